"""Expert parallelism on two GPUs: each rank's output against the single-GPU tensor-core
prefill of the same layer on its tokens.
- NCCL all-to-all path (ep.ExpertParallel): same activation terms, only the order in which
  the per-rank partial sums are added differs (1e-5).
- Peer-memory path (ep.FusedExpertParallel: token rows read and every pair's bf16 output row
  stored at its token's owner over NVLink by this library's kernels): every pair row is the
  single-GPU one and the owner's combine is the single-GPU combine, so the output equals the
  single-GPU layer (within 1e-5, bit for bit in practice), for two layer calls in a row with
  different token counts per rank."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = pytest.mark.gpu


def _worker(rank, world, port, err):
    sys.path.insert(0, ROOT)
    import datetime
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    try:
        from __graft_entry__ import load_package
        k3 = load_package()
        H, I, E, K, T = 256, 128, 8, 2, 200 + 37 * rank
        g = k3.synth.rng(31)                               # the same model on every rank
        experts = [k3.synth.expert(g, H, I) for _ in range(E)]
        shared = k3.synth.expert(g, H, I)
        wf, wb = k3.synth.router_weights(g, E, H)
        wf = (wf * 20).astype(np.float32)
        wb = k3.synth.bf16_bits(wf)
        W = torch.from_numpy(wb.view(np.int16)).to(dev).view(torch.bfloat16)
        full = k3.PoolMoeLayer.pack([k3.DeviceExpert.from_host(e, dev) for e in experts],
                                    k3.DeviceExpert.from_host(shared, dev), W, None, H, I, K, dev, terms=2)
        per = E // world
        owner = torch.arange(E, device=dev) // per
        run_of = torch.full((E,), -1, dtype=torch.int32, device=dev)
        run_of[rank * per:(rank + 1) * per] = full.run_of[rank * per:(rank + 1) * per]
        none = torch.full((E,), -1, dtype=torch.int32, device=dev)
        lr = k3.PoolMoeLayer(full.arena, E + 1, run_of, -1, W, None, H, I, K, terms=2)
        lsh = k3.PoolMoeLayer(full.arena, E + 1, none, E, W, None, H, I, K, terms=2)
        route, routed, sh = k3.ep.gpu_layer_fns(k3, lr, lsh, W, None, K)
        ep = k3.ep.ExpertParallel(owner, route, routed, sh)
        xb = k3.synth.bf16_bits(k3.synth.rng(500 + rank).standard_normal((T, H)).astype(np.float32))
        x = torch.from_numpy(xb.view(np.int16)).to(dev).view(torch.bfloat16)
        y = ep.forward(x)
        want, _, _ = full.prefill(x)
        torch.cuda.synchronize()
        y, want = y.cpu().numpy(), want.cpu().numpy()
        rel = np.abs(y - want).max() / np.abs(want).max()
        assert rel < 1e-5, rel
    except Exception as e:
        err.put(f"rank {rank}: {e!r}")
        raise
    finally:
        dist.destroy_process_group()


def _fused_worker(rank, world, port, err):
    sys.path.insert(0, ROOT)
    import datetime
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    ep = None
    try:
        from __graft_entry__ import load_package
        k3 = load_package()
        H, I, E, K = 256, 128, 8, 2
        g = k3.synth.rng(31)                               # the same model on every rank
        experts = [k3.synth.expert(g, H, I) for _ in range(E)]
        shared = k3.synth.expert(g, H, I)
        wf, wb = k3.synth.router_weights(g, E, H)
        wb = k3.synth.bf16_bits((wf * 20).astype(np.float32))
        W = torch.from_numpy(wb.view(np.int16)).to(dev).view(torch.bfloat16)
        full = k3.PoolMoeLayer.pack([k3.DeviceExpert.from_host(e, dev) for e in experts],
                                    k3.DeviceExpert.from_host(shared, dev), W, None, H, I, K, dev, terms=2)
        per = E // world
        run_of = torch.full((E,), -1, dtype=torch.int32, device=dev)
        run_of[rank * per:(rank + 1) * per] = full.run_of[rank * per:(rank + 1) * per]
        layer = k3.PoolMoeLayer(full.arena, E + 1, run_of, E, W, None, H, I, K, terms=2)
        ep = k3.ep.FusedExpertParallel(k3, layer, t_max=300)
        for call, T in enumerate((200 + 37 * rank, 131 - 50 * rank)):
            xb = k3.synth.bf16_bits(k3.synth.rng(700 + 10 * call + rank).standard_normal((T, H)).astype(np.float32))
            x = torch.from_numpy(xb.view(np.int16)).to(dev).view(torch.bfloat16)
            y = ep.forward(x)
            want, _, _ = full.prefill(x)
            torch.cuda.synchronize()
            y, want = y.cpu().numpy(), want.cpu().numpy()
            rel = np.abs(y - want).max() / np.abs(want).max()
            assert rel < 1e-5, (call, rel)
    except Exception as e:
        err.put(f"rank {rank}: {e!r}")
        raise
    finally:
        if ep is not None:
            ep.close()
        dist.destroy_process_group()


def test_ep_fused_two_gpus_equals_single_gpu():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    err = mp.get_context("spawn").SimpleQueue()
    mp.start_processes(_fused_worker, args=(2, 29652, err), nprocs=2, join=True, start_method="spawn")
    assert err.empty()


def test_ep_two_gpus_matches_single_gpu():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    err = mp.get_context("spawn").SimpleQueue()
    mp.start_processes(_worker, args=(2, 29650, err), nprocs=2, join=True, start_method="spawn")
    assert err.empty()


def test_ep_fused_one_rank_equals_single_gpu():
    """The peer-memory path's kernels (id gather, token quantisation from the x buffer, pair
    rows into the receive buffer, owner combine) on a one-rank group: the output equals the
    single-GPU layer bit for bit."""
    import datetime
    import torch
    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    from __graft_entry__ import load_package
    k3 = load_package()
    dev = torch.device("cuda:0")
    torch.cuda.set_device(0)
    dist.init_process_group("gloo", init_method="tcp://127.0.0.1:29661", rank=0, world_size=1,
                            timeout=datetime.timedelta(seconds=60))
    ep = None
    try:
        H, I, E, K = 512, 256, 16, 4
        g = k3.synth.rng(77)
        experts = [k3.synth.expert(g, H, I) for _ in range(E)]
        shared = k3.synth.expert(g, H, I)
        wf, wb = k3.synth.router_weights(g, E, H)
        W = torch.from_numpy(wb.view(np.int16)).to(dev).view(torch.bfloat16)
        full = k3.PoolMoeLayer.pack([k3.DeviceExpert.from_host(e, dev) for e in experts],
                                    k3.DeviceExpert.from_host(shared, dev), W, None, H, I, K, dev, terms=2)
        ep = k3.ep.FusedExpertParallel(k3, full, t_max=400)
        for call, T in enumerate((333, 97)):
            xb = k3.synth.bf16_bits(k3.synth.rng(800 + call).standard_normal((T, H)).astype(np.float32))
            x = torch.from_numpy(xb.view(np.int16)).to(dev).view(torch.bfloat16)
            y = ep.forward(x)
            want, _, _ = full.prefill(x)
            torch.cuda.synchronize()
            y, want = y.cpu().numpy(), want.cpu().numpy()
            assert np.array_equal(y, want), (call, np.abs(y - want).max())
    finally:
        if ep is not None:
            ep.close()
        dist.destroy_process_group()


def _emulated_ranks(k3, W_, H, I, E, K, counts, t_max, seed, replicate=0):
    """W_ ranks of the peer-memory expert-parallel layer emulated on ONE GPU: every rank's
    buffers are device tensors of cuda:0 and the three steps run for all ranks in turn on one
    stream (step 1 of every rank, then step 2 of every rank, then step 3), which orders them
    as the two barriers do. No kernel waits on another (the step-2 kernels read only x, idx
    and wt, which step 2 never writes, and store into the receive buffers, which only step 3
    reads). `replicate` experts are held by every rank with their pairs run by the tokens'
    owners (k3c_ep_peers.local_only). Returns each rank's output and the single-GPU layer's on
    the same tokens."""
    import ctypes as C
    import torch
    dev = torch.device("cuda:0")
    L = k3.lib()
    g = k3.synth.rng(seed)
    experts = [k3.synth.expert(g, H, I) for _ in range(E)]
    shared = k3.synth.expert(g, H, I)
    wf, _ = k3.synth.router_weights(g, E, H)
    wb = k3.synth.bf16_bits((wf * 20).astype(np.float32))
    Wr = torch.from_numpy(wb.view(np.int16)).to(dev).view(torch.bfloat16)
    full = k3.PoolMoeLayer.pack([k3.DeviceExpert.from_host(e, dev) for e in experts],
                                k3.DeviceExpert.from_host(shared, dev), Wr, None, H, I, K, dev, terms=2)
    owner = np.random.default_rng(seed).permutation(np.arange(E) % W_)     # scattered placement
    rep = np.zeros(E, bool)
    rep[np.random.default_rng(seed + 1).permutation(E)[:replicate]] = True
    expert_rank = torch.from_numpy(owner.astype(np.int32)).to(dev)
    local_only = torch.from_numpy(rep.astype(np.uint8)).to(dev)
    layers = []
    for q in range(W_):
        run_of = full.run_of.clone()
        run_of[torch.from_numpy((owner != q) & ~rep).to(dev)] = -1
        layers.append(k3.PoolMoeLayer(full.arena, E + 1, run_of, E, Wr, None, H, I, K, terms=2))
    xb = [torch.zeros((t_max, H), dtype=torch.bfloat16, device=dev) for _ in range(W_)]
    idx = [torch.zeros((t_max, K), dtype=torch.int32, device=dev) for _ in range(W_)]
    wt = [torch.zeros((t_max, K), dtype=torch.float32, device=dev) for _ in range(W_)]
    recv = [torch.zeros((t_max, K + 1, H), dtype=torch.int16, device=dev) for _ in range(W_)]
    peers = []
    for q in range(W_):
        p = k3.EpPeersC()
        p.world, p.rank, p.t_max = W_, q, t_max
        p.x_dtype = k3._dtype_code(xb[0])
        p.local_only = local_only.data_ptr() if replicate else None
        for r in range(W_):
            p.ntok[r] = counts[r]
            p.x[r], p.idx[r], p.wt[r], p.recv[r] = (xb[r].data_ptr(), idx[r].data_ptr(), wt[r].data_ptr(),
                                                    recv[r].data_ptr())
        peers.append(p)
    xs = []
    for q in range(W_):                                     # step 1: tokens and their routing
        T = counts[q]
        x = torch.from_numpy(k3.synth.bf16_bits(k3.synth.rng(900 + q).standard_normal((T, H)).astype(np.float32))
                             .view(np.int16)).to(dev).view(torch.bfloat16)
        xs.append(x)
        xb[q][:T].copy_(x)
        c = layers[q].c
        rn = L.k3c_router_scratch(H, E, T)
        rs = torch.empty(rn, dtype=torch.uint8, device=dev)
        k3._check(L.k3c_router_ws(idx[q].data_ptr(), wt[q].data_ptr(), None, xb[q].data_ptr(), k3._dtype_code(xb[q]),
                                  C.c_void_p(c.router_w), c.router_dtype, C.c_void_p(c.router_bias), H, E, K,
                                  c.renorm, c.routed_scale, T, rs.data_ptr(), rn, k3._stream()), "k3c_router_ws")
    keep = []
    for q in range(W_):                                     # step 2: every rank's experts
        c = layers[q].c
        need = L.k3c_moe_prefill_ep_scratch(C.byref(c), C.byref(peers[q]))
        assert need > 0, L.k3c_last_error()
        ws = torch.empty(need, dtype=torch.uint8, device=dev)
        keep.append(ws)
        k3._check(L.k3c_moe_prefill_ep_experts(C.byref(c), C.byref(peers[q]), ws.data_ptr(), need, k3._stream()),
                  "k3c_moe_prefill_ep_experts")
    outs = []
    for q in range(W_):                                     # step 3: each rank's combine
        out = torch.empty((counts[q], H), dtype=torch.float32, device=dev)
        k3._check(L.k3c_moe_ep_combine(out.data_ptr(), C.byref(peers[q]), H, K, expert_rank.data_ptr(), E, 1,
                                       k3._stream()), "k3c_moe_ep_combine")
        outs.append(out)
    wants = [full.prefill(xs[q])[0] if counts[q] else torch.empty((0, H), device=dev) for q in range(W_)]
    torch.cuda.synchronize()
    return [o.cpu().numpy() for o in outs], [w.cpu().numpy() for w in wants]


@pytest.mark.parametrize("W_,H,I,E,K,counts,t_max,replicate", [
    (2, 256, 128, 8, 2, (200, 131), 256, 0),
    (4, 512, 256, 16, 4, (97, 300, 0, 1), 320, 0),
    (8, 256, 128, 16, 2, (40, 33, 64, 1, 17, 64, 5, 29), 64, 0),
    (4, 512, 256, 16, 4, (97, 300, 0, 1), 320, 3),
    (8, 256, 128, 16, 2, (40, 33, 64, 1, 17, 64, 5, 29), 64, 5),
])
def test_ep_emulated_ranks_equal_single_gpu(k3, W_, H, I, E, K, counts, t_max, replicate):
    """The multi-rank indexing of the peer-memory path (pair rows stored at row t % t_max of
    rank t / t_max's receive buffer, token rows read from the owners' buffers, ragged and empty
    ranks, replicated experts whose pairs run at their tokens' owners) on one GPU: every rank's
    output equals the single-GPU layer bit for bit."""
    outs, wants = _emulated_ranks(k3, W_, H, I, E, K, list(counts), t_max, seed=40 + W_, replicate=replicate)
    for q, (o, w) in enumerate(zip(outs, wants)):
        assert np.array_equal(o, w), (q, np.abs(o - w).max() if o.size else 0)
