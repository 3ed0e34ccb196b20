"""INT8 trunk projection on the tensor cores (k3c_q8_gemv) against the CPU oracle.

The kernel splits activations into four int8 terms and accumulates exactly in int32, so it
lands much closer to the oracle's double-accumulated result than the reference's fp32 sum
does; the bar here is 2e-6 of max|y| (the reference-facing bar is 1e-5)."""
import numpy as np
import pytest

from conftest import maxrel

pytestmark = pytest.mark.gpu

TOL = 2e-6


@pytest.fixture(scope="module")
def dev():
    import torch
    return torch.device("cuda:0")


def T(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def run(k3, x_dev, wq, ws, ldw, in_, out, ntok, ldx):
    import torch
    y = torch.full((ntok, out), float("nan"), dtype=torch.float32, device=x_dev.device)
    rc = k3.lib().k3c_q8_gemv(y.data_ptr(), out, x_dev.data_ptr(), k3._dtype_code(x_dev), ldx, ntok,
                              wq.data_ptr(), ws.data_ptr(), ldw, in_, out, k3._stream())
    assert rc == 0, k3.lib().k3c_last_error()
    return y.cpu().numpy()


@pytest.mark.parametrize("in_,out,ntok,dtype,pad", [
    (100, 70, 1, "f32", 0),        # one K tile, one partial row tile, no split-K
    (300, 260, 5, "bf16", 0),      # ragged K tile and row tile
    (1000, 129, 33, "f32", 3),     # three token blocks, rows not 16-byte aligned (scalar loads)
    (7168, 2048, 20, "bf16", 5),   # two token blocks, unaligned bf16 rows
    (7168, 7168, 16, "bf16", 0),   # the trunk shape of the decode benchmark
])
def test_q8_tc_vs_oracle(k3, ora, dev, in_, out, ntok, dtype, pad):
    import torch
    g = k3.synth.rng(100 + in_ + ntok)
    _, _, rows = k3.synth.q8_matrix(g, out, in_)
    wq, ws, ldw = k3.q8_pack(T(rows, dev), in_, out)
    ldx = in_ + pad
    xf = np.zeros((ntok, ldx), np.float32)
    xf[:, :in_] = g.standard_normal((ntok, in_), dtype=np.float32)
    if dtype == "bf16":
        xb = k3.synth.bf16_bits(xf)
        xf = k3.synth.bf16_to_f32(xb)
        xd = T(xb.view(np.int16), dev).view(torch.bfloat16)
    else:
        xd = T(xf, dev)
    got = run(k3, xd, wq, ws, ldw, in_, out, ntok, ldx)
    for t in range(ntok):
        assert maxrel(got[t], ora.matmul_q8(xf[t, :in_], rows, in_, out)) < TOL, t
    again = run(k3, xd, wq, ws, ldw, in_, out, ntok, ldx)
    assert np.array_equal(got.view(np.uint32), again.view(np.uint32))   # deterministic


def test_q8_tc_wide_dynamic_range(k3, ora, dev):
    """Activations spanning 2^-40 .. 2^40 within one token, and an all-zero token."""
    g = k3.synth.rng(7)
    in_, out, ntok = 2048, 384, 4
    _, _, rows = k3.synth.q8_matrix(g, out, in_)
    wq, ws, ldw = k3.q8_pack(T(rows, dev), in_, out)
    xf = (g.standard_normal((ntok, in_)) * np.exp2(g.integers(-40, 41, (ntok, in_)))).astype(np.float32)
    xf[2] = 0.0
    got = run(k3, T(xf, dev), wq, ws, ldw, in_, out, ntok, in_)
    assert np.all(got[2] == 0.0)
    for t in (0, 1, 3):
        assert maxrel(got[t], ora.matmul_q8(xf[t], rows, in_, out)) < TOL, t


def test_q8_tc_nonfinite_token(k3, ora, dev):
    """A token holding inf yields NaN outputs; the other tokens are unaffected."""
    g = k3.synth.rng(9)
    in_, out, ntok = 512, 256, 3
    _, _, rows = k3.synth.q8_matrix(g, out, in_)
    wq, ws, ldw = k3.q8_pack(T(rows, dev), in_, out)
    xf = g.standard_normal((ntok, in_), dtype=np.float32)
    xf[1, 77] = np.inf
    got = run(k3, T(xf, dev), wq, ws, ldw, in_, out, ntok, in_)
    assert np.all(np.isnan(got[1]))
    for t in (0, 2):
        assert maxrel(got[t], ora.matmul_q8(xf[t], rows, in_, out)) < TOL, t


@pytest.mark.parametrize("in_,out,ntok", [(7168, 7168, 16), (1000, 129, 33), (300, 260, 1)])
def test_q8_caller_scratch_equals_pooled(k3, dev, in_, out, ntok):
    """k3c_q8_gemv_ws with caller-owned scratch (offset by 8 bytes: the entry point aligns it)
    gives the bits of k3c_q8_gemv; a buffer too short is refused with K3C_EINVAL before any
    launch."""
    import torch
    g = k3.synth.rng(900 + ntok)
    _, _, rows = k3.synth.q8_matrix(g, out, in_)
    wq, ws, ldw = k3.q8_pack(T(rows, dev), in_, out)
    xb = k3.synth.bf16_bits(g.standard_normal((ntok, in_), dtype=np.float32))
    xd = T(xb.view(np.int16), dev).view(torch.bfloat16)
    want = run(k3, xd, wq, ws, ldw, in_, out, ntok, in_)
    need = k3.q8_gemv_scratch(ntok, in_, out)
    buf = torch.empty(need + 8, dtype=torch.uint8, device=dev)
    y = torch.full((ntok, out), float("nan"), dtype=torch.float32, device=dev)
    L = k3.lib()
    rc = L.k3c_q8_gemv_ws(y.data_ptr(), out, xd.data_ptr(), k3.K3C_BF16, in_, ntok, wq.data_ptr(), ws.data_ptr(),
                          ldw, in_, out, buf.data_ptr() + 8, need, k3._stream())
    assert rc == 0, L.k3c_last_error()
    assert np.array_equal(y.cpu().numpy().view(np.uint32), want.view(np.uint32))
    rc = L.k3c_q8_gemv_ws(y.data_ptr(), out, xd.data_ptr(), k3.K3C_BF16, in_, ntok, wq.data_ptr(), ws.data_ptr(),
                          ldw, in_, out, buf.data_ptr(), need - 257, k3._stream())
    assert rc == -1   # K3C_EINVAL
    y2 = k3.q8_gemv(xd, wq, ws, ldw, in_, out, scratch=buf)
    assert np.array_equal(y2.cpu().numpy().view(np.uint32), want.view(np.uint32))
