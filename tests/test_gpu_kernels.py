"""GPU parity of libk3cuda.so against the CPU oracle and the reference's golden vectors.

Tolerances: dequantised weights and router indices bit-exact;
expert/GEMV outputs within 1e-5 relative (fp32 activations, fp32 accumulate) using the
reference's own metric max|got-want| / max|want|.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import maxrel

pytestmark = pytest.mark.gpu

TOL_F32 = 1e-5


@pytest.fixture(scope="module")
def dev():
    import torch
    return torch.device("cuda:0")


def T(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


# ------------------------------------------------------------------------ dequant
def test_dequant_exact_on_checkpoint_bytes(golden, k3, dev):
    g = golden("mxfp4_ckpt.npz")
    out = k3.mxfp4_dequant(T(g["packed"], dev), T(g["scales"], dev), 32).cpu().numpy()
    assert np.array_equal(out.view(np.uint32), g["expected"].view(np.uint32))


@pytest.mark.parametrize("name", ["g32", "g32_wide", "g16", "g64", "g24_tail", "edges"])
def test_dequant_exact_vs_reference(golden, k3, dev, name):
    g = golden("ref_kernels.npz")
    p, s = g[f"mx_{name}_packed"], g[f"mx_{name}_scales"]
    out = k3.mxfp4_dequant(T(p, dev), T(s, dev), int(g[f"mx_{name}_group"])).cpu().numpy()
    assert np.array_equal(out.view(np.uint32), g[f"mx_{name}_deq"].view(np.uint32))


# --------------------------------------------------------------------------- GEMV
@pytest.mark.parametrize("name", ["g32", "g32_wide", "g16", "g64", "g24_tail", "edges"])
def test_gemv_vs_reference_golden(golden, k3, dev, name):
    g = golden("ref_kernels.npz")
    p, s, x, y = (g[f"mx_{name}_{k}"] for k in ("packed", "scales", "x", "y"))
    got = k3.mxfp4_gemv(T(x, dev), T(p, dev), T(s, dev), int(g[f"mx_{name}_group"]))
    got = got.cpu().numpy()[0]
    fin = np.isfinite(y)
    assert np.array_equal(np.isfinite(got), fin)
    assert np.array_equal(got[~fin], y[~fin], equal_nan=True)
    assert maxrel(got[fin], y[fin]) < TOL_F32


@pytest.mark.parametrize("rows,in_,ntok", [(2048, 7168, 1), (7168, 2048, 1), (33, 7168, 3),
                                           (16, 64, 5), (129, 2048, 9), (1, 32, 1)])
def test_gemv_batched_vs_oracle(k3, ora, dev, rows, in_, ntok):
    g = k3.synth.rng(rows * 31 + in_ + ntok)
    p, s = k3.synth.mxfp4_matrix(g, rows, in_)
    x = g.standard_normal((ntok, in_), dtype=np.float32)
    got = k3.mxfp4_gemv(T(x, dev), T(p, dev), T(s, dev)).cpu().numpy()
    for t in range(ntok):
        want = ora.matmul_mxfp4(x[t], p, s)
        assert maxrel(got[t], want) < TOL_F32, t


def test_dropin_matmul_and_dequant_host_pointers(k3, ora):
    """The reference's own entry points, host pointers in and out."""
    L = k3.lib()
    g = k3.synth.rng(5)
    for rows, in_, group in [(300, 7168, 32), (17, 96, 16), (5, 70, 24)]:
        p = g.integers(0, 256, (rows, in_ // 2), dtype=np.uint8)
        s = g.integers(110, 140, (rows, (in_ + group - 1) // group), dtype=np.uint8)
        s[0, 0] = 255
        x = g.standard_normal(in_, dtype=np.float32)
        y = np.empty(rows, np.float32)
        L.k3_matmul_mxfp4(y.ctypes.data, x.ctypes.data, p.ctypes.data, s.ctypes.data, in_, rows,
                          group)
        assert maxrel(y, ora.matmul_mxfp4(x, p, s, group)) < TOL_F32
        d = np.empty((rows, in_), np.float32)
        L.k3_mxfp4_dequant(d.ctypes.data, p.ctypes.data, s.ctypes.data, rows, in_ // 2, group)
        assert np.array_equal(d.view(np.uint32), ora.mxfp4_dequant(p, s, group).view(np.uint32))


# ----------------------------------------------------------------------------- q8
@pytest.mark.parametrize("name", ["q8a", "q8b"])
def test_q8_vs_reference_golden(golden, k3, dev, name):
    g = golden("ref_kernels.npz")
    rows, x, y = g[f"{name}_rows"], g[f"{name}_x"], g[f"{name}_y"]
    in_, out = int(g[f"{name}_in"]), y.shape[0]
    wq, ws, ldw = k3.q8_pack(T(rows, dev), in_, out)
    got = k3.q8_gemv(T(x, dev), wq, ws, ldw, in_, out).cpu().numpy()[0]
    assert maxrel(got, y) < TOL_F32


def test_q8_trunk_shape_bf16_input(k3, ora, dev):
    import torch
    g = k3.synth.rng(8)
    H = 7168
    _, _, rows = k3.synth.q8_matrix(g, H, H)
    xf, xb = k3.synth.activations(g, 3, H)
    wq, ws, ldw = k3.q8_pack(T(rows, dev), H, H)
    xt = T(xb.view(np.int16), dev).view(torch.bfloat16)
    got = k3.q8_gemv(xt, wq, ws, ldw, H, H).cpu().numpy()
    for t in range(3):
        assert maxrel(got[t], ora.matmul_q8(xf[t], rows, H, H)) < TOL_F32
    y = np.empty(H, np.float32)                       # drop-in entry point, host pointers
    k3.lib().k3_matmul_q8(y.ctypes.data, xf[0].ctypes.data, rows.ctypes.data, H, H)
    assert maxrel(y, ora.matmul_q8(xf[0], rows, H, H)) < TOL_F32


# ------------------------------------------------------------------------- router
def test_router_select_bit_exact_on_same_scores(k3, ora, dev):
    """Indices must match the reference bit-exactly on the same scores (ties, NaN, -inf,
    fewer finite candidates than topk)."""
    g = k3.synth.rng(9)
    E, K = 384, 8
    cases = []
    s = g.random((6, E), dtype=np.float32)
    s[1, 10:20] = s[1, 5]                  # a 11-way tie
    s[2, :] = 0.5                          # everything tied
    s[3, ::3] = np.nan                     # NaN is never selected
    s[4, :] = -np.inf
    s[4, 7] = 0.25                          # one finite candidate, topk 8
    s[5, 100] = np.inf
    bias = (g.standard_normal(E, dtype=np.float32) * 0.01).astype(np.float32)
    for b in (None, bias):
        for renorm, scale in ((1, 1.0), (0, 2.5)):
            idx, w = k3.router_select(T(s, dev), None if b is None else T(b, dev), K, renorm, scale)
            idx, w = idx.cpu().numpy(), w.cpu().numpy()
            for t in range(s.shape[0]):
                ri, rw = ora.router_select(s[t], b, K, renorm, scale)
                assert np.array_equal(idx[t], ri), (t, idx[t], ri)
                # bitwise, except that NaN (inf * 0 after renorm of an inf score) matches
                # NaN whatever its payload: the GPU's canonical NaN is 0x7fffffff
                nan = np.isnan(rw)
                assert np.array_equal(np.isnan(w[t]), nan), t
                assert np.array_equal(w[t][~nan].view(np.uint32), rw[~nan].view(np.uint32)), t


def test_router_fixture_sets_and_weights(golden, k3, dev):
    g = golden("router_fixture.npz")
    K = int(g["top_k"])
    idx, w, _ = k3.router(T(g["x"], dev), T(g["W"], dev), T(g["bias"], dev), K)
    idx, w = idx.cpu().numpy(), w.cpu().numpy()
    for t in range(g["x"].shape[0]):
        assert set(idx[t].tolist()) == set(g["topk_idx"][t].tolist())
        for a in range(K):
            b = list(g["topk_idx"][t]).index(idx[t][a])
            ref = g["topk_weight"][t][b]
            assert abs(w[t][a] - ref) <= 1e-5 + 1e-4 * abs(ref)


def test_router_full_shape_matches_reference(golden, k3, ora, dev):
    import torch
    g = golden("ref_router_full.npz")
    r = k3.synth.rng(int(g["seed"]))
    wf, wb = k3.synth.router_weights(r)
    xf, xb = k3.synth.activations(r, 16)
    W = T(wb.view(np.int16), dev).view(torch.bfloat16)
    X = T(xb.view(np.int16), dev).view(torch.bfloat16)
    idx, w, sc = k3.router(X, W, None, 8)
    assert np.array_equal(idx.cpu().numpy(), g["idx"])
    np.testing.assert_array_max_ulp(w.cpu().numpy(), g["wt"], maxulp=1)
    # Scores: the device exp is correctly rounded, libm expf is within ~0.5 ulp; one ulp of
    # exp can become two after 1/(1+e). Indices (above) are the exact-parity boundary.
    sref = np.stack([ora.router_scores(xf[t], wf) for t in range(16)])
    np.testing.assert_array_max_ulp(sc.cpu().numpy(), sref, maxulp=2)


@pytest.mark.parametrize("ntok,hidden,wdt,xdt", [
    (1, 7168, "bf16", "bf16"), (2, 7168, "bf16", "f32"), (3, 1000, "f32", "bf16"),
    (7, 7168, "bf16", "bf16"), (16, 700, "f32", "f32"), (21, 7168, "bf16", "bf16"),
])
def test_router_token_blockings(k3, ora, dev, ntok, hidden, wdt, xdt):
    """Every tokens-per-block specialisation (1, 2, 4, 8, 16, and several blocks), ragged
    hidden sizes (a partial last K chunk, rows not 16-byte aligned) and all dtype pairs:
    indices exact, scores within 2 ulp of the oracle's correctly rounded ones."""
    import torch
    g = k3.synth.rng(500 + ntok)
    E, K = 384, 8
    wf = (g.standard_normal((E, hidden)) * 0.02).astype(np.float32)
    xf = g.standard_normal((ntok, hidden)).astype(np.float32)
    bias = (g.standard_normal(E) * 0.01).astype(np.float32)
    dev_t = {}
    for name, a, dt in (("W", wf, wdt), ("x", xf, xdt)):
        if dt == "bf16":
            b = k3.synth.bf16_bits(a)
            a[...] = k3.synth.bf16_to_f32(b)
            dev_t[name] = T(b.view(np.int16), dev).view(torch.bfloat16)
        else:
            dev_t[name] = T(a, dev)
    idx, w, sc = k3.router(dev_t["x"], dev_t["W"], T(bias, dev), K)
    idx, w, sc = idx.cpu().numpy(), w.cpu().numpy(), sc.cpu().numpy()
    for t in range(ntok):
        ri, rw = ora.router(xf[t], wf, bias, K)
        assert np.array_equal(idx[t], ri), t
        np.testing.assert_allclose(w[t], rw, rtol=1e-6)   # from scores within 2 ulp
        np.testing.assert_array_max_ulp(sc[t], ora.router_scores(xf[t], wf), maxulp=2)


def test_dropin_router_host_pointers(golden, k3, ora):
    g = golden("ref_kernels.npz")
    L = k3.lib()
    X, W, bias = g["rt_x"], g["rt_W"], g["rt_bias"]     # keep the arrays alive across calls
    for renorm in (0, 1):
        for t in range(X.shape[0]):
            idx = np.empty(6, np.int32)
            w = np.empty(6, np.float32)
            xt = np.ascontiguousarray(X[t])
            L.k3_router(idx.ctypes.data, w.ctypes.data, xt.ctypes.data, W.ctypes.data,
                        bias.ctypes.data, 64, 24, 6, renorm, 2.5)
            assert np.array_equal(idx, g[f"rt_idx_r{renorm}"][t])
            np.testing.assert_array_max_ulp(w, g[f"rt_wt_r{renorm}"][t], maxulp=1)


# -------------------------------------------------------------------- expert FFN
@pytest.mark.parametrize("ntok,act", [(1, 0), (3, 0), (2, 1)])
def test_expert_ffn_config0_shape(k3, ora, dev, ntok, act):
    """one 7168 -> 2048 -> 7168 MXFP4 expert, fp32 x ~ N(0,1)."""
    g = k3.synth.rng(100 + ntok)
    e = k3.synth.expert(g)
    x = g.standard_normal((ntok, 7168), dtype=np.float32)
    de = k3.DeviceExpert.from_host(e, dev)
    y = k3.expert_ffn(T(x, dev), de, 7168, 2048, act).cpu().numpy()
    want = ora.expert_ffn(x, e, 7168, 2048, act)
    assert maxrel(y, want) < TOL_F32


def test_expert_ffn_vs_reference_golden(golden, k3, dev):
    g = golden("ref_kernels.npz")
    H, I, E, K, Tn = (int(v) for v in g["moe_dims"])
    keys = k3.DeviceExpert.KEYS
    e0 = {k: g[f"moe_e0_{k}"] for k in keys}
    de = k3.DeviceExpert.from_host(e0, dev)
    y = k3.expert_ffn(T(g["moe_x"], dev), de, H, I, 0).cpu().numpy()
    assert maxrel(y, g["ffn_y"]) < TOL_F32
    y = k3.expert_ffn(T(g["moe_x"], dev), de, H, I, 1).cpu().numpy()
    assert maxrel(y, g["ffn_y_situ"]) < TOL_F32


# -------------------------------------------------------------------- MoE decode
def test_moe_decode_vs_reference_golden(golden, k3, dev):
    g = golden("ref_kernels.npz")
    H, I, E, K, Tn = (int(v) for v in g["moe_dims"])
    keys = k3.DeviceExpert.KEYS
    ex = [{k: g[f"moe_e{i}_{k}"] for k in keys} for i in range(E + 1)]
    layer = k3.MoeLayer.from_host(ex[:E], ex[E], g["moe_W"], None, H, I, K, device=dev)
    out, idx, wt = layer.decode(T(g["moe_x"], dev))
    assert np.array_equal(idx.cpu().numpy(), g["moe_idx"])
    np.testing.assert_array_max_ulp(wt.cpu().numpy(), g["moe_wt"], maxulp=1)
    assert maxrel(out.cpu().numpy(), g["moe_out"]) < TOL_F32


@pytest.mark.parametrize("ntok", [1, 4, 16])
def test_moe_decode_config1_shape(k3, ora, dev, ntok):
    """BASELINE config[1] shapes (hidden 7168, inter 2048, top-8, 1 shared expert, bf16 x and
    bf16 router W) with 48 distinct experts tiled over the 384 expert ids to bound memory."""
    import torch
    g = k3.synth.rng(200 + ntok)
    H, I, E, K = 7168, 2048, 384, 8
    distinct = [k3.synth.expert(g) for _ in range(48)]
    shared = k3.synth.expert(g)
    experts = [distinct[i % 48] for i in range(E)]
    xf, xb = k3.synth.activations(g, ntok)
    wf, wb = k3.synth.router_weights(g, E, H)
    dev_distinct = [k3.DeviceExpert.from_host(e, dev) for e in distinct]
    layer = k3.MoeLayer([dev_distinct[i % 48] for i in range(E)],
                        k3.DeviceExpert.from_host(shared, dev),
                        T(wb.view(np.int16), dev).view(torch.bfloat16), None, H, I, K, device=dev)
    drops = torch.zeros(1, dtype=torch.int32, device=dev)
    out, idx, wt = layer.decode(T(xb.view(np.int16), dev), drops=drops)
    ro, ri, rw = ora.moe_layer(xf, wf, None, experts, shared, H, I, K)
    assert drops.item() == 0
    assert np.array_equal(idx.cpu().numpy(), ri)
    np.testing.assert_array_max_ulp(wt.cpu().numpy(), rw, maxulp=1)
    assert maxrel(out.cpu().numpy(), ro) < TOL_F32


def test_moe_decode_counts_drops_for_missing_experts(k3, ora, dev):
    """A selected expert with no resident weights is skipped and counted
    (src/core/k3_ops.c:616-626)."""
    import torch
    H, I, E, K, Tn = 256, 128, 8, 2, 3
    g = k3.synth.rng(300)
    experts = [k3.synth.expert(g, H, I) for _ in range(E)]
    xf, _ = k3.synth.activations(g, Tn, H)
    wf, _ = k3.synth.router_weights(g, E, H)
    wf = (wf * 30).astype(np.float32)
    devs = [k3.DeviceExpert.from_host(e, dev) for e in experts]
    _, ri, rw = ora.moe_layer(xf, wf, None, experts, None, H, I, K)
    missing = int(ri[0, 0])
    layer = k3.MoeLayer([None if i == missing else d for i, d in enumerate(devs)], None,
                        T(wf, dev), None, H, I, K, device=dev)
    drops = torch.zeros(1, dtype=torch.int32, device=dev)
    out, idx, wt = layer.decode(T(xf, dev), drops=drops)
    assert drops.item() == int((ri == missing).sum())
    # the output equals the oracle computed with that expert's contribution removed
    want = np.zeros((Tn, H), np.float32)
    for t in range(Tn):
        for j in range(K):
            if ri[t, j] == missing:
                continue
            want[t] += rw[t, j] * ora.expert_ffn(xf[t], experts[ri[t, j]], H, I)[0]
    assert maxrel(out.cpu().numpy(), want) < TOL_F32
