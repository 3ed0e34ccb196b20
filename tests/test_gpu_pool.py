"""HBM expert pool (k3c_pool_*) against the restated cache bookkeeping (oracle/cache_model.py)
and the resident-expert decode path."""
import numpy as np
import pytest

from oracle.cache_model import CacheModel

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    import torch
    return torch.device("cuda:0")


def T(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


class HostRuns:
    """Pinned host pool-format runs, one per (layer, expert) key, packed on the device from
    random experts and copied back (so the bytes are exactly the pool format)."""

    def __init__(self, k3, dev, H, I, n_layers, n_experts, seed):
        import torch
        self.n_experts = n_experts
        g = k3.synth.rng(seed)
        self.experts, self.runs = [], []
        rb = k3.pool_run_bytes(H, I)
        dev_run = torch.empty(rb, dtype=torch.uint8, device=dev)
        for _ in range(n_layers * n_experts):
            e = k3.synth.expert(g, H, I)
            k3.pool_pack(dev_run, k3.DeviceExpert.from_host(e, dev).q(), H, I)
            self.experts.append(e)
            self.runs.append(dev_run.cpu().pin_memory())

    def __call__(self, layer, expert):
        return self.runs[layer * self.n_experts + expert]


def test_pool_bookkeeping_matches_cache_model(k3, dev):
    """Slot choice, hits, misses, evictions and prefetch accounting, request by request."""
    import torch
    H, I, NL, NE, NS = 256, 128, 2, 8, 5
    host = HostRuns(k3, dev, H, I, NL, NE, seed=1)
    pool = k3.ExpertPool(H, I, NL, NE, NS, host)
    model = CacheModel(NL, NE, NS)
    rng = np.random.default_rng(3)
    for step in range(60):
        layer = int(rng.integers(NL))
        ids = rng.choice(NE, size=int(rng.integers(1, 5)), replace=False).tolist()
        if step % 7 == 3:
            assert pool.getmany(layer, ids) == model.getmany(layer, ids)
        got = pool.acquire(layer, ids).tolist()
        assert got == model.acquire(layer, ids), step
        for e, s in zip(ids, got):
            assert pool.resident(layer, e) == s
        pool.release(layer, ids)
        model.release(layer, ids)
    torch.cuda.synchronize()
    st, ms = pool.stats(), model.stats()
    for k in ("hits", "misses", "evictions", "prefetch_reads"):
        assert st[k] == ms[k], k
    assert st["bytes_h2d"] == (ms["misses"] + ms["prefetch_reads"]) * k3.pool_run_bytes(H, I)
    assert st["true_hit_rate"] == pytest.approx(ms["true_hit_rate"])
    pool.close()


def test_pool_slots_hold_the_host_bytes(k3, dev):
    import torch
    H, I, NL, NE, NS = 256, 128, 1, 6, 4
    host = HostRuns(k3, dev, H, I, NL, NE, seed=2)
    pool = k3.ExpertPool(H, I, NL, NE, NS, host)
    rb = k3.pool_run_bytes(H, I)
    for ids in ([0, 1, 2], [3, 4], [5, 0, 1]):
        slots = pool.acquire(0, ids)
        for e, s in zip(ids, slots):
            got = pool.slot_tensor(s)[:rb].cpu().numpy()   # ordered after the copy
            assert np.array_equal(got, host(0, e).numpy())
        pool.release(0, ids)
    pool.close()


def test_pool_all_pinned_is_reported(k3, dev):
    H, I, NL, NE, NS = 256, 128, 1, 6, 2
    host = HostRuns(k3, dev, H, I, NL, NE, seed=4)
    pool = k3.ExpertPool(H, I, NL, NE, NS, host)
    pool.acquire(0, [0, 1])
    with pytest.raises(k3.K3CError, match="pinned"):
        pool.acquire(0, [2])
    pool.release(0, [0, 1])
    pool.acquire(0, [2])          # now evicts the least recently used
    pool.release(0, [2])
    pool.close()


def test_streamed_decode_matches_resident_layers(k3, dev):
    """Several layers through a pool that holds fewer slots than one layer's experts plus
    the next one's, back to back without host syncs: every layer's output equals the same
    layer run with all of its experts resident."""
    import torch
    H, I, NL, NE, K, NS = 256, 128, 4, 8, 3, 7
    host = HostRuns(k3, dev, H, I, NL, NE, seed=5)
    g = k3.synth.rng(6)
    shared = [k3.synth.expert(g, H, I) for _ in range(NL)]
    # the shared experts live in the pool too, pinned: they get the keys of extra experts
    host_sh = []
    rb = k3.pool_run_bytes(H, I)
    dev_run = torch.empty(rb, dtype=torch.uint8, device=dev)
    for e in shared:
        k3.pool_pack(dev_run, k3.DeviceExpert.from_host(e, dev).q(), H, I)
        host_sh.append(dev_run.cpu().pin_memory())

    def src(layer, expert):
        return host_sh[layer] if expert == NE else host(layer, expert)

    pool = k3.ExpertPool(H, I, NL, NE + 1, NS + NL, src)
    wf, wb = k3.synth.router_weights(g, NE, H)
    W = T(wb.view(np.int16), dev).view(torch.bfloat16)
    xf, xb = k3.synth.activations(g, 2, H)
    x0 = T(xb.view(np.int16), dev).view(torch.bfloat16)
    # routing for every layer from the resident reference layers
    refs, routes = [], []
    x = x0
    for l in range(NL):
        lay = k3.PoolMoeLayer.pack([k3.DeviceExpert.from_host(e, dev) for e in host.experts[l * NE:(l + 1) * NE]],
                                   k3.DeviceExpert.from_host(shared[l], dev), W, None, H, I, K, dev)
        out, idx, wt = lay.decode(x)
        refs.append(out.clone())
        routes.append((idx.clone(), wt.clone()))
        x = out.to(torch.bfloat16)
    torch.cuda.synchronize()
    shared_slots = [pool.pin(l, NE) for l in range(NL)]
    run_ofs = [pool.run_table() for _ in range(NL)]
    layers = [pool.layer(W, H, I, K, NE, run_ofs[l], shared_slot=shared_slots[l]) for l in range(NL)]
    outs = []
    x = x0
    for l in range(NL):
        idx, wt = routes[l]
        ids = sorted(set(idx.cpu().numpy().ravel().tolist()))
        pool.acquire(l, ids, run_of=run_ofs[l])
        out = layers[l].decode_routed(x, idx, wt)
        pool.release(l, ids)
        outs.append(out)
        x = out.to(torch.bfloat16)
    torch.cuda.synchronize()
    for l in range(NL):
        assert np.array_equal(outs[l].cpu().numpy().view(np.uint32), refs[l].cpu().numpy().view(np.uint32)), l
    st = pool.stats()
    assert st["evictions"] > 0
    pool.close()


def test_streamed_prefill_matches_resident_layers(k3, dev):
    """The reference's streamed prefill (k3_moe_prefill with an expert source,
    src/core/k3_ops.c:689-808: each distinct expert of the chunk fetched once): layers of 40
    tokens whose distinct experts are acquired through a pool that cannot hold all layers at
    once, run by the routed prefill kernels; every output equals the resident layer's bit for
    bit, and the pool evicts on the way."""
    import torch
    H, I, NL, NE, K, T_ = 256, 128, 3, 8, 3, 40
    host = HostRuns(k3, dev, H, I, NL, NE, seed=15)
    g = k3.synth.rng(16)
    pool = k3.ExpertPool(H, I, NL, NE, NE + 2, host)
    wf, wb = k3.synth.router_weights(g, NE, H)
    W = T(wb.view(np.int16), dev).view(torch.bfloat16)
    _, xb = k3.synth.activations(g, T_, H)
    x0 = T(xb.view(np.int16), dev).view(torch.bfloat16)
    refs, routes, x = [], [], x0
    for l in range(NL):
        lay = k3.PoolMoeLayer.pack([k3.DeviceExpert.from_host(e, dev) for e in host.experts[l * NE:(l + 1) * NE]],
                                   None, W, None, H, I, K, dev)
        out, idx, wt = lay.prefill(x)
        refs.append(out.clone())
        routes.append((idx.clone(), wt.clone()))
        x = out.to(torch.bfloat16)
    torch.cuda.synchronize()
    run_ofs = [pool.run_table() for _ in range(NL)]
    layers = [pool.layer(W, H, I, K, NE, run_ofs[l]) for l in range(NL)]
    outs, x = [], x0
    for l in range(NL):
        idx, wt = routes[l]
        ids = sorted(set(idx.cpu().numpy().ravel().tolist()))
        pool.acquire(l, ids, run_of=run_ofs[l])
        outs.append(layers[l].prefill_routed(x, idx, wt))
        pool.release(l, ids)
        x = outs[-1].to(torch.bfloat16)
    torch.cuda.synchronize()
    for l in range(NL):
        assert np.array_equal(outs[l].cpu().numpy().view(np.uint32), refs[l].cpu().numpy().view(np.uint32)), l
    assert pool.stats()["evictions"] > 0
    pool.close()


def test_cache_only_routing(k3, ora, dev):
    """The draft model's cache-only routing (src/core/k3_ops.c:580-593): kept entries and their
    renormalised weights equal a host restatement bit for bit, and the layer run with them
    equals the oracle's sum over the resident experts (plus the shared expert)."""
    import torch
    from conftest import maxrel
    H, I, E, K, T_ = 256, 128, 16, 4, 8
    g = k3.synth.rng(21)
    experts = [k3.synth.expert(g, H, I) for _ in range(E)]
    shared = k3.synth.expert(g, H, I)
    wf, wb = k3.synth.router_weights(g, E, H)
    wf = (wf * 20).astype(np.float32)
    wb = k3.synth.bf16_bits(wf)
    W = T(wb.view(np.int16), dev).view(torch.bfloat16)
    xf, xb = k3.synth.activations(g, T_, H)
    x = T(xb.view(np.int16), dev).view(torch.bfloat16)
    full = k3.PoolMoeLayer.pack([k3.DeviceExpert.from_host(e, dev) for e in experts],
                                k3.DeviceExpert.from_host(shared, dev), W, None, H, I, K, dev)
    _, idx, wt = full.decode(x)
    resident = np.array([e % 3 != 0 for e in range(E)])
    run_of = T(np.where(resident, np.arange(E), -1).astype(np.int32), dev)
    idx2, wt2 = idx.clone(), wt.clone()
    k3.route_cache_only(idx2, wt2, run_of, full.c.n_runs)
    hi, hw = idx.cpu().numpy(), wt.cpu().numpy()
    want_i = np.full_like(hi, -1)
    want_w = np.zeros_like(hw)
    for t in range(T_):
        kept = [(e, w) for e, w in zip(hi[t], hw[t]) if resident[e]]
        s = np.float32(0)
        for _, w in kept:
            s = np.float32(s + w)
        for j, (e, w) in enumerate(kept):
            want_i[t, j] = e
            want_w[t, j] = np.float32(w / s) if s > 0 else w
    assert np.array_equal(idx2.cpu().numpy(), want_i)
    assert np.array_equal(wt2.cpu().numpy().view(np.uint32), want_w.view(np.uint32))
    draft = k3.PoolMoeLayer(full.arena, full.c.n_runs, run_of, full.c.shared_run, W, None, H, I, K)
    out = draft.decode_routed(x, idx2, wt2).cpu().numpy()
    want = np.zeros((T_, H), np.float32)
    for t in range(T_):
        for j in range(K):
            if want_i[t, j] >= 0:
                y = ora.expert_ffn(xf[t:t + 1], experts[want_i[t, j]], H, I)[0]
                want[t] = want[t] + np.float32(want_w[t, j]) * y
        want[t] = want[t] + ora.expert_ffn(xf[t:t + 1], shared, H, I)[0]
    assert (want_i < 0).any()
    assert maxrel(out, want) < 2e-2


def _decode_want(ora, xf, experts, shared, idx, wt, H, I):
    """Host restatement of a routed decode: sum over the kept entries in top-k order, then the
    shared expert (src/core/k3_ops.c:641-654)."""
    T_, K = idx.shape
    want = np.zeros((T_, H), np.float32)
    for t in range(T_):
        for j in range(K):
            if idx[t, j] >= 0:
                y = ora.expert_ffn(xf[t:t + 1], experts[idx[t, j]], H, I)[0]
                want[t] = want[t] + np.float32(wt[t, j]) * y
        if shared is not None:
            want[t] = want[t] + ora.expert_ffn(xf[t:t + 1], shared, H, I)[0]
    return want


def test_acquire_resident_with_getmany_in_flight(k3, ora, dev):
    """The draft model's resident set from the pool (k3c_pool_acquire_resident): with a batch
    prefetch still copying, the run table it writes holds every expert with a slot, the slots
    are pinned (no eviction until release) and the stream waits for their copies, no hit or
    miss is counted; cache-only routing over that table and the routed decode equal a host
    restatement over the same resident set."""
    import ctypes as C
    import torch
    from conftest import maxrel
    H, I, NE, NS, K, T_ = 256, 128, 16, 10, 4, 6
    host = HostRuns(k3, dev, H, I, 1, NE, seed=31)
    pool = k3.ExpertPool(H, I, 1, NE, NS, host)
    L = k3.lib()
    pool.acquire(0, [0, 1, 2], None)
    pool.release(0, [0, 1, 2])
    assert pool.getmany(0, [5, 6, 7, 8]) == 4              # copies on the pool's stream
    before = pool.stats()
    run_of = pool.run_table()
    ids = np.empty(NE, np.int32)
    n = L.k3c_pool_acquire_resident(pool.p, 0, ids.ctypes.data, NE, C.c_void_p(run_of.data_ptr()),
                                    k3._stream())
    assert n == 7 and sorted(ids[:n].tolist()) == [0, 1, 2, 5, 6, 7, 8]
    after = pool.stats()
    assert (after["hits"], after["misses"]) == (before["hits"], before["misses"])
    # pinned: filling the other experts cannot evict them (3 free slots only)
    with pytest.raises(k3.K3CError):
        pool.acquire(0, [9, 10, 11, 12], None)
    # the layer over the pool arena, routing filtered to the resident set
    g = k3.synth.rng(32)
    wf, wb = k3.synth.router_weights(g, NE, H)
    wf = (wf * 20).astype(np.float32)
    wb = k3.synth.bf16_bits(wf)
    W = T(wb.view(np.int16), dev).view(torch.bfloat16)
    xf, xb = k3.synth.activations(g, T_, H)
    x = T(xb.view(np.int16), dev).view(torch.bfloat16)
    layer = pool.layer(W, H, I, K, NE, run_of)
    idx, wt, _ = k3.router(x, W, None, K)
    hi, hw = idx.cpu().numpy(), wt.cpu().numpy()
    k3.route_cache_only(idx, wt, run_of, NS)
    out = layer.decode_routed(x, idx, wt).cpu().numpy()
    resident = set(ids[:n].tolist())
    want_i = np.full_like(hi, -1)
    want_w = np.zeros_like(hw)
    for t in range(T_):
        kept = [(e, w) for e, w in zip(hi[t], hw[t]) if e in resident]
        s = np.float32(0)
        for _, w in kept:
            s = np.float32(s + w)
        for j, (e, w) in enumerate(kept):
            want_i[t, j], want_w[t, j] = e, (np.float32(w / s) if s > 0 else w)
    assert np.array_equal(idx.cpu().numpy(), want_i)
    assert np.array_equal(wt.cpu().numpy().view(np.uint32), want_w.view(np.uint32))
    experts = [host.experts[e] for e in range(NE)]
    assert maxrel(out, _decode_want(ora, xf, experts, None, want_i, want_w, H, I)) < 2e-2
    pool.release(0, ids[:n])
    pool.acquire(0, [9, 10, 11, 12], None)                # unpinned: room again
    pool.close()


def test_route_cache_only_respects_the_run_count(k3, dev):
    """An expert whose run index is at or past n_runs is not resident (the expert kernels'
    own test), so it is dropped from the routing and the kept weights renormalised without it."""
    idx = T(np.array([[0, 1, 2, 3]], np.int32), dev)
    wt = T(np.array([[0.4, 0.3, 0.2, 0.1]], np.float32), dev)
    run_of = T(np.array([0, 7, 1, 2], np.int32), dev)       # expert 1 -> run 7 >= n_runs 3
    k3.route_cache_only(idx, wt, run_of, 3)
    assert idx.cpu().numpy().tolist() == [[0, 2, 3, -1]]
    s = np.float32(np.float32(np.float32(0.4) + np.float32(0.2)) + np.float32(0.1))
    want = np.array([np.float32(0.4) / s, np.float32(0.2) / s, np.float32(0.1) / s, 0], np.float32)
    assert np.array_equal(wt.cpu().numpy()[0].view(np.uint32), want.view(np.uint32))


def test_source_without_bytes_fails_that_expert_only(k3, dev):
    """A host source that has no bytes for some experts (the reference's failed read,
    src/cache/k3_cache.c:197-216): the request fails with K3C_ENOTFOUND, the miss is counted,
    no slot is taken (the expert stays absent, nothing else is evicted), and the other experts
    fill normally."""
    H, I, NE, NS = 256, 128, 8, 4
    host = HostRuns(k3, dev, H, I, 1, NE, seed=41)
    pool = k3.ExpertPool(H, I, 1, NE, NS, lambda layer, e: None if e in (3, 5) else host(layer, e))
    pool.acquire(0, [0, 1], None)
    pool.release(0, [0, 1])
    with pytest.raises(k3.K3CError, match="no host bytes"):
        pool.acquire(0, [3], None)
    assert pool.resident(0, 3) == -1
    assert pool.resident(0, 0) >= 0 and pool.resident(0, 1) >= 0   # nothing evicted
    assert pool.getmany(0, [5, 6]) == 1                       # 5 fails, 6 is copied
    assert pool.resident(0, 5) == -1 and pool.resident(0, 6) >= 0
    st = pool.stats()
    assert st["misses"] == 3 and st["prefetch_reads"] == 1
    pool.close()


def test_trace_histogram_pin_and_reset(k3, dev, tmp_path):
    """The reference cache's bookkeeping around the counters: every get request is traced as
    an int32 (layer, expert) pair and counted in the histogram (k3_cache.c:235-249), the dumps
    have the reference's formats (k3_cache_dump_trace, k3_cache_dump_hist), a pinned slot is
    never chosen as a victim (k3_cache_pin), and a reset clears the counters together."""
    import ctypes as C
    import json
    H, I, NL, NE, NS = 256, 128, 2, 6, 3
    host = HostRuns(k3, dev, H, I, NL, NE, seed=51)
    pool = k3.ExpertPool(H, I, NL, NE, NS, host)
    L = k3.lib()
    reqs = [(0, [1, 2]), (1, [4]), (0, [1]), (1, [0, 5])]
    for layer, ids in reqs:
        pool.acquire(layer, ids, None)
        pool.release(layer, ids)
    flat = [v for layer, ids in reqs for e in ids for v in (layer, e)]
    n = L.k3c_pool_trace(pool.p, None, 0)
    tr = np.empty(n, np.int32)
    L.k3c_pool_trace(pool.p, tr.ctypes.data, n)
    assert tr.tolist() == flat
    hist = np.empty(NL * NE, np.uint32)
    assert L.k3c_pool_hist(pool.p, hist.ctypes.data) == 0
    assert hist[0 * NE + 1] == 2 and hist[1 * NE + 4] == 1 and hist.sum() == len(flat) // 2
    p = str(tmp_path / "trace.bin")
    assert L.k3c_pool_dump_trace(pool.p, p.encode()) == 0
    assert np.fromfile(p, np.int32).tolist() == flat
    ph = str(tmp_path / "hist.json")
    assert L.k3c_pool_dump_hist(pool.p, ph.encode()) == 0
    d = json.load(open(ph))
    assert d["n_layers"] == NL and d["n_experts"] == NE and d["counts"]["0,1"] == 2 and "0,3" not in d["counts"]
    # pin (1, 5): three more distinct experts cannot evict it
    assert L.k3c_pool_set_pin(pool.p, 1, 5, 1) == 1
    assert L.k3c_pool_set_pin(pool.p, 0, 3, 1) == 0          # not resident
    for e in (2, 3, 4):
        pool.acquire(0, [e], None)
        pool.release(0, [e])
    assert pool.resident(1, 5) >= 0
    L.k3c_pool_set_pin(pool.p, 1, 5, 0)
    L.k3c_pool_reset_stats(pool.p)
    st = pool.stats()
    assert st["hits"] == st["misses"] == st["evictions"] == st["prefetch_reads"] == st["bytes_h2d"] == 0
    pool.close()
