"""Pin the CPU oracle (oracle/k3_oracle.c) to the reference before trusting it.

Three anchors, in order of authority:
  1. the reference's own golden vectors (released-checkpoint MXFP4 bytes and the
     torch-generated router fixture, converted into tests/golden/ by make_golden.py);
  2. outputs of the reference's own kernels recorded in tests/golden/ref_*.npz;
  3. live calls into oracle/_ref/libk3ref.so when it is present.
"""
import numpy as np
import pytest

from conftest import maxrel


def test_dequant_exact_on_checkpoint_bytes(golden, ora):
    # tests/unit/test_ops.c:743-796 of the reference: EXACT equality, no tolerance.
    g = golden("mxfp4_ckpt.npz")
    out = ora.mxfp4_dequant(g["packed"], g["scales"], int(g["group"]))
    assert np.array_equal(out.view(np.uint32), g["expected"].view(np.uint32))
    # the swapped nibble order gives the recorded wrong values: the check can fail
    sw = ora.mxfp4_dequant(
        ((g["packed"] >> 4) | (g["packed"] << 4)).astype(np.uint8), g["scales"], 32)
    assert np.array_equal(sw.ravel()[:64], g["swapped_first64"])
    assert not np.array_equal(out.ravel()[:64], g["swapped_first64"])


def test_e2m1_negative_zero(ora):
    L = ora.lib()
    assert np.signbit(np.float32(L.ora_e2m1(8))) and L.ora_e2m1(8) == 0.0
    assert [L.ora_e2m1(c) for c in range(16)] == [0, .5, 1, 1.5, 2, 3, 4, 6,
                                                 -0.0, -.5, -1, -1.5, -2, -3, -4, -6]
    assert L.ora_e8m0(255) == 0.0 and L.ora_e8m0(127) == 1.0
    assert L.ora_e8m0(0) == np.ldexp(np.float32(1), -127)


def test_router_fixture(golden, ora):
    # tests/unit/test_ops.c:350-401: index SETS equal, weights atol 1e-5 rtol 1e-4
    # (tests/fixtures/ops/MANIFEST.json tolerance block).
    g = golden("router_fixture.npz")
    K = int(g["top_k"])
    changed = 0
    for t in range(g["x"].shape[0]):
        idx, w = ora.router(g["x"][t], g["W"], g["bias"], K)
        assert set(idx.tolist()) == set(g["topk_idx"][t].tolist())
        for a in range(K):
            b = list(g["topk_idx"][t]).index(idx[a])
            assert abs(w[a] - g["topk_weight"][t][b]) <= 1e-5 + 1e-4 * abs(g["topk_weight"][t][b])
        nb, _ = ora.router(g["x"][t], g["W"], None, K)
        changed += set(nb.tolist()) != set(idx.tolist())
    assert changed == int(g["rows_where_bias_changed_selection"])


@pytest.mark.parametrize("name", ["g32", "g32_wide", "g16", "g64", "g24_tail", "edges"])
def test_gemv_matches_reference_kernel(golden, ora, name):
    g = golden("ref_kernels.npz")
    p, s, x, y = (g[f"mx_{name}_{k}"] for k in ("packed", "scales", "x", "y"))
    grp = int(g[f"mx_{name}_group"])
    got = ora.matmul_mxfp4(x, p, s, grp)
    fin = np.isfinite(y)
    assert np.array_equal(np.isfinite(got), fin)          # the 2^127*6 row is inf in both
    assert np.array_equal(got[~fin], y[~fin], equal_nan=True)  # inf / NaN rows agree
    assert maxrel(got[fin], y[fin]) < 1e-6                 # test_expert.c:219 contract
    deq = ora.mxfp4_dequant(p, s, grp)
    assert np.array_equal(deq.view(np.uint32), g[f"mx_{name}_deq"].view(np.uint32))


@pytest.mark.parametrize("name", ["q8a", "q8b"])
def test_q8_matches_reference_kernel(golden, ora, name):
    g = golden("ref_kernels.npz")
    in_ = int(g[f"{name}_in"])
    y = ora.matmul_q8(g[f"{name}_x"], g[f"{name}_rows"], in_, g[f"{name}_y"].shape[0])
    assert maxrel(y, g[f"{name}_y"]) < 1e-5


def test_router_small_matches_reference(golden, ora):
    g = golden("ref_kernels.npz")
    X, W, bias = g["rt_x"], g["rt_W"], g["rt_bias"]     # keep the arrays alive across calls
    for renorm in (0, 1):
        for t in range(X.shape[0]):
            idx = np.empty(6, np.int32)
            w = np.empty(6, np.float32)
            ora.lib().ora_router(idx, w, np.ascontiguousarray(X[t]), W, bias.ctypes.data,
                                 64, 24, 6, renorm, 2.5)
            assert np.array_equal(idx, g[f"rt_idx_r{renorm}"][t])
            assert np.array_equal(w.view(np.uint32), g[f"rt_wt_r{renorm}"][t].view(np.uint32))


def test_router_full_shape_matches_reference(golden, ora, k3):
    g = golden("ref_router_full.npz")
    r = k3.synth.rng(int(g["seed"]))
    wf, wb = k3.synth.router_weights(r)
    xf, xb = k3.synth.activations(r, 16)
    chk = [int(wb.astype(np.uint64).sum()), int(xb.astype(np.uint64).sum())]
    assert chk == [int(v) for v in g["input_checksum"]], "synthetic generator drifted"
    for t in range(16):
        idx, w = ora.router(xf[t], wf, None, 8)
        assert np.array_equal(idx, g["idx"][t])
        assert np.array_equal(w.view(np.uint32), g["wt"][t].view(np.uint32))


def _moe_fixture(g):
    H, I, E, K, T = (int(v) for v in g["moe_dims"])
    keys = ("gate_p", "gate_s", "up_p", "up_s", "down_p", "down_s")
    ex = [{k: g[f"moe_e{i}_{k}"] for k in keys} for i in range(E + 1)]
    return H, I, E, K, T, ex[:E], ex[E]


def test_expert_and_moe_match_reference(golden, ora):
    g = golden("ref_kernels.npz")
    H, I, E, K, T, experts, shared = _moe_fixture(g)
    y = ora.expert_ffn(g["moe_x"], experts[0], H, I, act=0)
    assert maxrel(y, g["ffn_y"]) < 1e-6
    y = ora.expert_ffn(g["moe_x"], experts[0], H, I, act=1)
    assert maxrel(y, g["ffn_y_situ"]) < 1e-6
    o, idx, wt = ora.moe_layer(g["moe_x"], g["moe_W"], None, experts, shared, H, I, K)
    assert np.array_equal(idx, g["moe_idx"])
    assert np.array_equal(wt, g["moe_wt"])
    assert maxrel(o, g["moe_out"]) < 1e-6


@pytest.mark.skipif("not __import__('oracle.oracle', fromlist=['x']).ref_available()")
def test_live_reference_random_cases(ora, k3):
    """Fresh random shapes against the reference's own kernels, when its build is here."""
    r = k3.synth.rng(77)
    for rows, in_ in [(3, 64), (130, 2048), (7, 7168)]:
        p, s = k3.synth.mxfp4_matrix(r, rows, in_, 60, 190)
        s[:, ::7] = 255                     # NaN scale groups are skipped
        x = r.standard_normal(in_, dtype=np.float32)
        a = ora.matmul_mxfp4(x, p, s)
        b = ora.matmul_mxfp4(x, p, s, use_ref=True)
        assert np.isfinite(b).all()
        assert maxrel(a, b) < 1e-6
