"""Expert-parallel dispatch and combine (kimi-k3-in-rust_b200/ep.py) on two gloo ranks on the
CPU, with the oracle as the compute step: every rank's output equals the single-process
oracle MoE layer on its tokens (within fp32 reassociation: partial sums are added per rank)."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _worker(rank, world, port, seed, skew, err):
    sys.path.insert(0, ROOT)
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from __graft_entry__ import load_package
        from oracle import oracle as ora
        k3 = load_package()
        H, I, E, K, T = 64, 32, 8, 3, 7
        g = k3.synth.rng(seed)                         # same model on every rank
        experts = [k3.synth.expert(g, H, I) for _ in range(E)]
        shared = k3.synth.expert(g, H, I)
        wf = (g.standard_normal((E, H)) * 0.5).astype(np.float32)
        bias = np.zeros(E, np.float32)
        if skew:
            bias[5] = 10.0                             # every token picks expert 5 first
        owner = np.array([e % world for e in range(E)], np.int64)
        xs = [k3.synth.rng(1000 + r).standard_normal((T + r, H)).astype(np.float32) for r in range(world)]
        x = torch.from_numpy(xs[rank])

        def route(xt):
            idx = np.empty((xt.shape[0], K), np.int32)
            wt = np.empty((xt.shape[0], K), np.float32)
            for t in range(xt.shape[0]):
                idx[t], wt[t] = ora.router(xt[t].numpy(), wf, bias, K)
            return torch.from_numpy(idx), torch.from_numpy(wt)

        def routed(xt, idx, wt):
            out = np.zeros((xt.shape[0], H), np.float32)
            for t in range(xt.shape[0]):
                for k in range(K):
                    e = int(idx[t, k])
                    if owner[e] == rank:
                        y = ora.expert_ffn(xt[t].numpy()[None, :], experts[e], H, I)[0]
                        out[t] = out[t] + np.float32(wt[t, k]) * y
            return torch.from_numpy(out)

        def shared_fn(xt):
            return torch.from_numpy(ora.expert_ffn(xt.numpy(), shared, H, I).astype(np.float32))

        ep = k3.ep.ExpertParallel(torch.from_numpy(owner), route, routed, shared_fn)
        y = ep.forward(x).numpy()
        want, _, _ = ora.moe_layer(xs[rank], wf, bias, experts, shared, H, I, K)
        rel = np.abs(y - want).max() / np.abs(want).max()
        assert rel < 1e-5, rel
        assert ep.last["sent_tokens"] >= x.shape[0]    # every token has a home rank at least
    except Exception as e:  # report through the queue, then re-raise
        err.put(f"rank {rank}: {e!r}")
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("skew", [False, True])
def test_ep_dispatch_combine_two_ranks(skew):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    err = ctx.SimpleQueue()
    port = 29600 + (7 if skew else 3)
    mp.start_processes(_worker, args=(2, port, 11, skew, err), nprocs=2, join=True, start_method="spawn")
    assert err.empty()


def test_balanced_placement():
    """Equal expert counts per rank; Zipf loads spread much more evenly than contiguous ranges."""
    import sys
    sys.path.insert(0, ROOT)
    from __graft_entry__ import load_package
    k3 = load_package()
    E, W = 384, 8
    rng = np.random.default_rng(2)
    marg = k3.synth.zipf_topk_marginal(E, 1.1, 8, samples=8192).numpy()   # reachable top-8 loads
    load = marg[rng.permutation(E)]
    owner, lists = k3.ep.balanced_placement(load, W)
    assert sorted(sum(lists, [])) == list(range(E))
    assert all(len(v) == E // W for v in lists)
    assert all(owner[e] == r for r, v in enumerate(lists) for e in v)
    sums = np.array([load[v].sum() for v in lists])
    contiguous = load.reshape(W, -1).sum(1)
    assert sums.max() / sums.mean() < contiguous.max() / contiguous.mean()
    assert sums.max() / sums.mean() < 1.3
