"""Tensor-core router logits (csrc/router_tc.cu: exact int8 digit products plus residual
lists) against the oracle router and against the fp64 CUDA-core logits on the same inputs:
indices exact, scores equal to the fp64 path and within 2 ulp of the oracle. Covers ragged
token/expert/hidden counts, the split-K slices small batches get, and the rows that take the
residual lists or the double-dot fallback (outliers, NaN, infinity, zero rows)."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    import torch
    return torch.device("cuda:0")


def _bf16(k3, a, dev):
    import torch
    b = k3.synth.bf16_bits(a)
    return k3.synth.bf16_to_f32(b), torch.from_numpy(b.view(np.int16)).to(dev).view(torch.bfloat16)


def _run(k3, x, W, bias, K, tc):
    old = os.environ.get("K3C_ROUTER_TC")
    os.environ["K3C_ROUTER_TC"] = "1" if tc else "0"
    try:
        idx, w, sc = k3.router(x, W, bias, K)
        return idx.cpu().numpy(), w.cpu().numpy(), sc.cpu().numpy()
    finally:
        if old is None:
            del os.environ["K3C_ROUTER_TC"]
        else:
            os.environ["K3C_ROUTER_TC"] = old


def _same_scores(s1, s0):
    same = (s1.view(np.uint32) == s0.view(np.uint32)) | (np.isnan(s1) & np.isnan(s0))
    assert same.all(), np.argwhere(~same)[:5]


@pytest.mark.parametrize("ntok,E,hidden", [
    (64, 384, 7168),      # one token tile, many K slices
    (300, 200, 7168),     # ragged token and expert tiles
    (1000, 384, 4000),    # partial last K block
    (257, 96, 1040),
])
def test_router_tc_matches_fp64_and_oracle(k3, ora, dev, ntok, E, hidden):
    import torch
    g = k3.synth.rng(900 + ntok)
    wf, W = _bf16(k3, (g.standard_normal((E, hidden)) * 0.02).astype(np.float32), dev)
    xf, x = _bf16(k3, g.standard_normal((ntok, hidden)).astype(np.float32), dev)
    bias_np = (g.standard_normal(E) * 0.01).astype(np.float32)
    bias = torch.from_numpy(bias_np).to(dev)
    K = 8
    i1, w1, s1 = _run(k3, x, W, bias, K, tc=True)
    i0, w0, s0 = _run(k3, x, W, bias, K, tc=False)
    assert np.array_equal(i1, i0)
    assert np.array_equal(w1.view(np.uint32), w0.view(np.uint32))
    _same_scores(s1, s0)
    rng = np.random.default_rng(0)
    for t in sorted(rng.choice(ntok, size=min(24, ntok), replace=False).tolist()):
        ri, rw = ora.router(xf[t], wf, bias_np, K)
        assert np.array_equal(i1[t], ri), t
        np.testing.assert_allclose(w1[t], rw, rtol=1e-6)
        np.testing.assert_array_max_ulp(s1[t], ora.router_scores(xf[t], wf), maxulp=2)


def test_router_tc_special_rows(k3, ora, dev):
    """Rows whose residual lists overflow (one huge element among ordinary ones), rows with
    a few dozen tiny elements (lists within capacity), NaN, infinity, all-zero and subnormal
    rows, in both operands."""
    import torch
    g = k3.synth.rng(77)
    E, H, T, K = 384, 7168, 200, 8
    wf = (g.standard_normal((E, H)) * 0.02).astype(np.float32)
    xf = g.standard_normal((T, H)).astype(np.float32)
    xf[3, 100] = 2.0 ** 20                      # every other element falls off the digits
    xf[4, :40] = 1e-6                           # forty residual entries
    xf[5, 7] = np.nan
    xf[6, 9] = np.inf
    xf[7] = 0.0
    xf[8, 5] = -2.0 ** 100
    wf[10, 0] = 1000.0                          # expert list overflow
    wf[11, 100:150] = 1e-9                      # fifty residual entries
    wf[12] = 0.0
    wf[13, :] = 2.0 ** -130                     # subnormal row
    xf, x = _bf16(k3, xf, dev)
    wf, W = _bf16(k3, wf, dev)
    bias_np = (g.standard_normal(E) * 0.01).astype(np.float32)
    bias = torch.from_numpy(bias_np).to(dev)
    i1, w1, s1 = _run(k3, x, W, bias, K, tc=True)
    i0, w0, s0 = _run(k3, x, W, bias, K, tc=False)
    assert np.array_equal(i1, i0)
    _same_scores(s1, s0)
    for t in (0, 3, 4, 5, 6, 7, 8, 199):
        ri, rw = ora.router(xf[t], wf, bias_np, K)
        assert np.array_equal(i1[t], ri), t
