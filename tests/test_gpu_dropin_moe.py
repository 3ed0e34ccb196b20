"""GPU parity of the MoE-layer drop-ins k3_moe / k3_moe_prefill (include/k3/k3.h:381-426 of the
reference; include/k3c.h here) against the reference's OWN k3_moe / k3_moe_prefill
(oracle/_ref, src/core/k3_ops.c:556-808) called on the same K3MoeW / K3Cfg and the same expert
source, and of the reference's own unit tests and kernel benchmark linked against
libk3cuda.so.

Bars: outputs within 2e-2 relative (max|got-want| / max|want|) on the tensor-core expert
kernels (measured ~1e-5 with three activation terms), 1e-5 on the fp32 engine
(K3C_DROPIN_FP32=1: k3_matmul_mxfp4's own order for the experts, k3_matmul's for the trunk);
the expert-source call sequence, the idx/wt left to the caller and the k3_expert_drops count
equal to the reference's exactly.
"""
import os
import re
import subprocess

import numpy as np
import pytest

from conftest import ROOT, latent_layer_from_npz, maxrel
from dropin_util import HostSource, MoeArgs, ours, reference

pytestmark = pytest.mark.gpu

REF_DIR = os.path.join(ROOT, "oracle", "_ref")
TOL_TC = 2e-2
TOL_FP32 = 1e-5


def _need_ref(ora):
    if not ora.ref_available():
        pytest.skip("oracle/_ref not built")


def _bin(name):
    p = os.path.join(REF_DIR, name)
    if not os.path.exists(p):
        pytest.skip(f"{name} not built (oracle/Makefile, needs the reference tree)")
    return p


def _layer(k3, seed, H=512, L=256, I=256, E=16, K=4, n_shared=1, wdt=1):
    g = k3.synth.rng(seed)
    return k3.synth.latent_layer(g, H, L, I, E, K, n_shared=n_shared, wdt=wdt), g


# ------------------------------------------------------------- the reference's own programs
def test_reference_unit_tests_through_library():
    """tests/unit/test_ops.c of the reference, linked so that every k3_* entry point this
    library defines (and the calls the reference's k3_ops.c makes to them internally: k3_moe
    from the decoder layer, k3_matmul from MLA/KDA, ...) runs on the GPU: the same tests pass
    as in the CPU build, including t_moe, t_router, t_mxfp4 (EXACT) and t_matmul_bf16."""
    cpu = subprocess.run([_bin("test_ops_cpu"), os.path.join(REF_DIR, "fixtures", "ops")],
                         capture_output=True, text=True, timeout=600)
    gpu = subprocess.run([_bin("test_ops_gpu"), os.path.join(REF_DIR, "fixtures", "ops")],
                         capture_output=True, text=True, timeout=900)
    print(gpu.stdout[-3000:], gpu.stderr[-2000:])
    assert cpu.returncode == 0, cpu.stdout[-2000:]
    assert gpu.returncode == 0, gpu.stdout[-2000:] + gpu.stderr[-2000:]

    def passed(s):
        return sorted(re.findall(r"^\s*PASS\s+(\S+)", s, re.M))

    assert passed(gpu.stdout) == passed(cpu.stdout)
    for name in ("moe", "router", "mxfp4", "matmul_bf16", "layer_kda", "layer_mla", "mla"):
        assert name in passed(gpu.stdout), name
    summary = re.search(r"(\d+) passed, (\d+) failed, (\d+) skipped", gpu.stdout)
    assert summary and summary.group(2) == "0" and summary.group(3) == "0"


def test_reference_bench_kernels_hashes_equal():
    """benchmarks/bench_kernels.c of the reference: the FNV-1a hashes of its bf16 trunk matmul
    (12288 x 7168) and its MXFP4 expert matmul (3072 x 3584) outputs are the CPU build's,
    bit for bit, with both kernels running on the GPU."""
    cpu = subprocess.run([_bin("bench_kernels_cpu")], capture_output=True, text=True, timeout=900)
    gpu = subprocess.run([_bin("bench_kernels_gpu")], capture_output=True, text=True, timeout=900)
    print(gpu.stdout)
    assert cpu.returncode == 0 and gpu.returncode == 0, gpu.stderr[-2000:]
    hc = re.findall(r"(\w+)\s+OUTPUT FNV1a = ([0-9a-f]+)", cpu.stdout)
    hg = re.findall(r"(\w+)\s+OUTPUT FNV1a = ([0-9a-f]+)", gpu.stdout)
    assert len(hc) == 2 and hg == hc


# ------------------------------------------------------------------------ k3_moe drop-in
def test_k3_moe_fp32_bank_fixture(k3, ora, golden):
    """The reference's published ops/moe.json layer (fp32 resident bank, SiTU in its caps,
    a bias that reorders the top-k): within test_ops.c's tolerance of the published output
    and within 1e-5 of the reference's own k3_moe, last token's idx/wt equal."""
    _need_ref(ora)
    f = golden("moe_latent_fixture.npz")
    layer = latent_layer_from_npz(f)
    a = MoeArgs(k3, layer)
    out, idx, wt, d = ours(k3, a, f["x"])
    rout, ridx, rwt, rd = reference(ora, a, f["x"])
    want = f["want"]
    assert (np.abs(out - want) <= 1e-4 + 1e-3 * np.abs(want)).all()
    err = maxrel(out, rout)
    print(f"k3_moe bank fixture: maxrel vs reference {err:.3e}")
    assert err <= TOL_FP32
    assert np.array_equal(idx, ridx) and np.array_equal(wt.view(np.uint32), rwt.view(np.uint32))
    assert d == rd == 0


@pytest.mark.parametrize("T,fp32", [(1, False), (5, False), (5, True), (40, False)])
def test_k3_moe_streamed_source(k3, ora, T, fp32, monkeypatch):
    """MXFP4 experts at the latent width from a host expert source (the reference's
    K3ExpertSrc contract), bf16 trunk: same routing, same source calls (getmany of the top-k,
    then get of each, token by token), output within the bar of the engine."""
    _need_ref(ora)
    if fp32:
        monkeypatch.setenv("K3C_DROPIN_FP32", "1")
    layer, g = _layer(k3, 300 + T)
    x = g.standard_normal((T, layer["hidden"]), dtype=np.float32)
    s_ours, s_ref = HostSource(k3, layer["experts"]), HostSource(k3, layer["experts"])
    out, idx, wt, d = ours(k3, MoeArgs(k3, layer, s_ours.src, layer_id=3), x)
    rout, ridx, rwt, rd = reference(ora, MoeArgs(k3, layer, s_ref.src, layer_id=3), x)
    err = maxrel(out, rout)
    print(f"k3_moe streamed T={T} {'fp32' if fp32 else 'tensor-core'}: maxrel {err:.3e}")
    assert err <= (TOL_FP32 if fp32 else TOL_TC)
    assert s_ours.log == s_ref.log
    assert np.array_equal(idx, ridx) and np.array_equal(wt.view(np.uint32), rwt.view(np.uint32))
    assert d == rd == 0


def test_k3_moe_cache_only(k3, ora):
    """The draft model's cache-only routing (k3_ops.c:580-593): resident() filters the top-k,
    the kept weights are renormalised, the experts come through resident(), nothing is counted
    as a drop; idx/wt left compacted exactly as the reference leaves them."""
    _need_ref(ora)
    layer, g = _layer(k3, 411, E=16, K=6)
    x = g.standard_normal((6, layer["hidden"]), dtype=np.float32)
    res = {e for e in range(16) if e % 3 != 1}
    s_ours, s_ref = HostSource(k3, layer["experts"], resident=res), HostSource(k3, layer["experts"], resident=res)
    out, idx, wt, d = ours(k3, MoeArgs(k3, layer, s_ours.src, cache_only=1), x)
    rout, ridx, rwt, rd = reference(ora, MoeArgs(k3, layer, s_ref.src, cache_only=1), x)
    assert s_ours.log == s_ref.log
    assert any(op == "resident" and not q for op, _, e, q in s_ours.log if e not in res)
    assert np.array_equal(idx, ridx) and np.array_equal(wt.view(np.uint32), rwt.view(np.uint32))
    assert d == rd == 0
    err = maxrel(out, rout)
    print(f"k3_moe cache-only: maxrel {err:.3e}")
    assert err <= TOL_TC


@pytest.mark.parametrize("T", [65, 100])
def test_k3_moe_prefill_batched(k3, ora, T):
    """k3_moe_prefill's batched source pattern (k3_ops.c:689-715): per 64-token chunk one
    getmany of its distinct experts in first-seen order and one get per distinct expert; a
    final one-token chunk goes through k3_moe and is the only writer of idx/wt."""
    _need_ref(ora)
    layer, g = _layer(k3, 500 + T)
    x = g.standard_normal((T, layer["hidden"]), dtype=np.float32)
    s_ours, s_ref = HostSource(k3, layer["experts"]), HostSource(k3, layer["experts"])
    out, idx, wt, d = ours(k3, MoeArgs(k3, layer, s_ours.src), x, prefill=True)
    rout, ridx, rwt, rd = reference(ora, MoeArgs(k3, layer, s_ref.src), x, prefill=True)
    assert s_ours.log == s_ref.log
    assert sum(1 for op, *_ in s_ours.log if op == "getmany") >= 2
    assert np.array_equal(idx, ridx) and np.array_equal(wt.view(np.uint32), rwt.view(np.uint32))
    err = maxrel(out, rout)
    print(f"k3_moe_prefill T={T}: maxrel {err:.3e}")
    assert err <= TOL_TC and d == rd == 0


@pytest.mark.parametrize("prefill", [False, True])
def test_k3_moe_failed_get_is_a_counted_drop(k3, ora, prefill):
    """A get() that fails is skipped and counted in k3_expert_drops, per token in k3_moe and
    once per chunk in the batched k3_moe_prefill, as the reference counts it. k3_moe skips the
    pair in both implementations, so every output agrees. The reference's batched path leaves
    the failed expert's contribution rows unwritten and still sums them (k3_ops.c:786-790):
    those tokens are the ones it reports as CORRUPT and their output is undefined there, so
    only the other tokens are compared."""
    _need_ref(ora)
    layer, g = _layer(k3, 77)
    x = g.standard_normal((9, layer["hidden"]), dtype=np.float32)
    hit = reference(ora, MoeArgs(k3, layer, HostSource(k3, layer["experts"]).src), x)[1]
    bad = int(hit[0])
    s_ours, s_ref = HostSource(k3, layer["experts"], fail={bad}), HostSource(k3, layer["experts"], fail={bad})
    out, idx, wt, d = ours(k3, MoeArgs(k3, layer, s_ours.src), x, prefill=prefill)
    rout, ridx, rwt, rd = reference(ora, MoeArgs(k3, layer, s_ref.src), x, prefill=prefill)
    assert s_ours.log == s_ref.log
    assert d == rd and d >= 1
    routed = np.stack([ora.router(x[t], layer["router_w"], layer["router_bias"], int(layer["topk"]))[0]
                       for t in range(len(x))])
    clean = ~(routed == bad).any(1)
    assert clean.any() and not clean.all()
    rows = clean if prefill else np.ones(len(x), bool)
    assert np.isfinite(out).all()
    assert maxrel(out[rows], rout[rows]) <= TOL_TC


def test_k3_moe_int8_trunk(k3, ora):
    """The draft model's K3_WI8 trunk rows through the drop-in (exact int32 sums here, float
    sums in the reference, which states no determinism contract for them)."""
    _need_ref(ora)
    layer, g = _layer(k3, 91, wdt=2, n_shared=2)
    x = g.standard_normal((3, layer["hidden"]), dtype=np.float32)
    s1, s2 = HostSource(k3, layer["experts"]), HostSource(k3, layer["experts"])
    out, idx, wt, _ = ours(k3, MoeArgs(k3, layer, s1.src), x)
    rout, ridx, rwt, _ = reference(ora, MoeArgs(k3, layer, s2.src), x)
    assert np.array_equal(idx, ridx)
    assert maxrel(out, rout) <= TOL_TC


def test_k3_moe_keep_weights(k3, ora):
    """k3c_dropin_keep_weights(1): weights uploaded once and reused; same result as the
    default per-call upload; forgetting them frees the copies."""
    _need_ref(ora)
    L = k3.lib()
    layer, g = _layer(k3, 93)
    x = g.standard_normal((2, layer["hidden"]), dtype=np.float32)
    a = MoeArgs(k3, layer, HostSource(k3, layer["experts"]).src)
    base = ours(k3, a, x)[0]
    L.k3c_dropin_keep_weights(1)
    try:
        o1 = ours(k3, a, x)[0]
        o2 = ours(k3, a, x)[0]
    finally:
        L.k3c_dropin_keep_weights(0)
        L.k3c_dropin_forget_weights()
    assert np.array_equal(o1, base) and np.array_equal(o2, base)


def _pool_from_layer(k3, layer, n_slots):
    """An HBM expert pool whose host side holds the layer's experts as pinned pool-format runs."""
    import torch
    Lw, I = int(layer["latent"]), int(layer["inter"])
    run = k3.pool_run_bytes(Lw, I)
    host = []
    for e in layer["experts"]:
        dev = torch.empty(run, dtype=torch.uint8, device="cuda")
        k3.pool_pack(dev, k3.DeviceExpert.from_host(e, "cuda").q(), Lw, I)
        torch.cuda.synchronize()
        host.append(dev.cpu().pin_memory())
    pool = k3.ExpertPool(Lw, I, 4, len(layer["experts"]), n_slots, lambda layer_, e: host[e])
    return pool, host


def test_k3_moe_pool_source(k3, ora):
    """k3c_pool_source as the layer's K3ExpertSrc: the experts are used in their pool slots
    (no staging copy), hits/misses counted per get as the reference's cache counts them, the
    access trace records every request, pins released once the kernels are enqueued."""
    _need_ref(ora)
    import ctypes as C
    import torch
    L = k3.lib()
    layer, g = _layer(k3, 61, E=16, K=4)
    x = g.standard_normal((4, layer["hidden"]), dtype=np.float32)
    pool, host = _pool_from_layer(k3, layer, n_slots=12)
    src = L.k3c_pool_source_create(pool.p, C.c_void_p(torch.cuda.current_stream().cuda_stream))
    try:
        a = MoeArgs(k3, layer, src, layer_id=2)
        out, idx, wt, d = ours(k3, a, x)
        s_ref = HostSource(k3, layer["experts"])
        rout, ridx, rwt, rd = reference(ora, MoeArgs(k3, layer, s_ref.src, layer_id=2), x)
        assert np.array_equal(idx, ridx) and d == rd == 0
        err = maxrel(out, rout)
        print(f"k3_moe pool source: maxrel {err:.3e}")
        assert err <= TOL_TC
        gets = [(lay, e) for op, lay, e, *_ in s_ref.log if op == "get"]
        st = pool.stats()
        assert st["hits"] + st["misses"] == len(gets)
        n = L.k3c_pool_trace(pool.p, None, 0)
        tr = np.empty(n, np.int32)
        L.k3c_pool_trace(pool.p, tr.ctypes.data, n)
        assert [tuple(v) for v in tr.reshape(-1, 2).tolist()] == gets
        # every pin released: all 12 slots can be taken by other experts of another layer
        ids = np.arange(12, dtype=np.int32)
        run_of = pool.run_table()
        pool.acquire(1, ids, run_of)
        pool.release(1, ids)
    finally:
        L.k3c_pool_source_destroy(C.c_void_p(src))
        pool.close()
