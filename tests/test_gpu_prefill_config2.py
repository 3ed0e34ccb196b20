"""GPU parity of the tcgen05 MoE prefill on the exact layer bench.py measures for BASELINE
config[2]: 4096 bf16 tokens, 384 distinct MXFP4 experts plus a shared expert (7168 -> 2048 ->
7168), the bf16 router with the selection bias fitted to Zipf(1.1) popularity
(synth.zipf_router), activations as two E4M3 terms.

The whole layer runs once; at least 128 of its tokens are checked against the reference's
k3_moe composition (oracle/_ref when built: the reference's own k3_router and
k3_matmul_mxfp4; otherwise the oracle restatement), indices exact and outputs within the
bf16 bar of 2e-2 relative (max|got-want| / max|want|). The tokens are chosen from the layer's
slot structure (each expert's pairs in (token, k) order, 128 per slot): the hottest expert's
first and last slots, the pairs on either side of its slot boundaries, the partial last
slots of many lightly used experts, the tokens with the most pairs in multi-slot experts,
the first and last token, and random ones.
"""
import numpy as np
import pytest

from conftest import maxrel

pytestmark = pytest.mark.gpu

TOL_BF16 = 2e-2
H, I, E, K, T = 7168, 2048, 384, 8, 4096
M = 128   # pair rows per slot


@pytest.fixture(scope="module")
def dev():
    import torch
    return torch.device("cuda:0")


def _sample_tokens(idx, rng):
    counts = np.bincount(idx.ravel(), minlength=E)
    flat = idx.ravel()
    pairs_of = {}
    order = np.argsort(flat, kind="stable")        # pair indices grouped by expert, (t, k) order
    starts = np.concatenate([[0], np.cumsum(counts)])
    for e in range(E):
        pairs_of[e] = order[starts[e]:starts[e + 1]]
    pick = {0, T - 1}
    hot = int(np.argmax(counts))
    ph = pairs_of[hot]
    last0 = ((len(ph) - 1) // M) * M
    pick.update((ph[last0:] // K)[:: max(1, (len(ph) - last0) // 16)][:16].tolist())    # last slot
    pick.update((ph[:M] // K)[::16].tolist())                                            # first slot
    for e in np.argsort(-counts)[:3]:                                                    # boundaries
        pe = pairs_of[int(e)]
        for b in range(M, len(pe), M):
            pick.update((pe[b - 1:b + 1] // K).tolist())
    light = [e for e in np.argsort(counts) if 0 < counts[e] < M]                         # tail slots
    for e in light[:: max(1, len(light) // 40)][:40]:
        pick.add(int(pairs_of[int(e)][-1] // K))
    multi = counts[idx] > M                                                              # many slots
    pick.update(np.argsort(-multi.sum(1), kind="stable")[:16].tolist())
    rest = np.setdiff1d(np.arange(T), np.array(sorted(pick)))
    need = max(0, 144 - len(pick))
    pick.update(rng.choice(rest, need, replace=False).tolist())
    return np.array(sorted(pick)), counts, hot


def test_prefill_config2_bench_layer(k3, ora, dev):
    import torch
    ref_runs, arena = k3.synth.device_bank(k3, E + 1, H, I, dev, seed=2024)
    W, bias, _ = k3.synth.zipf_router(dev, E, H, K)
    layer = k3.PoolMoeLayer(arena, E + 1, torch.arange(E, dtype=torch.int32, device=dev), E, W, bias,
                            H, I, K, terms=2)
    g = torch.Generator(device=dev)
    g.manual_seed(4096)
    x = torch.randn((T, H), generator=g, device=dev).to(torch.bfloat16)
    drops = torch.zeros(1, dtype=torch.int32, device=dev)
    out, idx, wt = layer.prefill(x, drops=drops)
    torch.cuda.synchronize()
    assert drops.item() == 0
    assert bool(torch.isfinite(out).all())
    idx = idx.cpu().numpy()
    sel, counts, hot = _sample_tokens(idx, np.random.default_rng(7))
    n_slots = int(sum((c + M - 1) // M for c in counts))
    print(f"config2 layer: {int((counts > 0).sum())} experts hit, hottest {hot} with {counts[hot]} pairs "
          f"({(counts[hot] + M - 1) // M} slots), {n_slots} routed slots, "
          f"{int(((counts % M) > 0).sum())} partial; checking {len(sel)} tokens")
    assert len(sel) >= 128
    assert counts[hot] > 4 * M                    # the fitted Zipf bias gives a multi-slot head
    xf = x[torch.from_numpy(sel).to(dev)].float().cpu().numpy()
    wf = W.float().cpu().numpy()
    bh = bias.cpu().numpy()
    shared = k3.synth.host_expert(ref_runs, E, H, I)
    use_ref = ora.ref_available()
    got = out.cpu().numpy()[sel]
    want = np.empty_like(got)
    host = {}                                       # each needed expert copied to the host once
    for c0 in range(0, len(sel), 16):
        rows = slice(c0, min(c0 + 16, len(sel)))
        need = sorted(set(idx[sel[rows]].ravel().tolist()))
        for e in need:
            if e not in host:
                host[e] = k3.synth.host_expert(ref_runs, e, H, I)
        experts = [host.get(e, host[need[0]]) for e in range(E)]   # the others are never selected
        ro, ri, _ = ora.moe_layer(xf[rows], wf, bh, experts, shared, H, I, K, use_ref=use_ref)
        assert np.array_equal(ri, idx[sel[rows]]), f"routing differs in tokens {sel[rows]}"
        want[rows] = ro
    err = maxrel(got, want)
    print(f"config2 layer vs {'reference' if use_ref else 'oracle'}: maxrel {err:.3e} over {len(sel)} tokens")
    assert err < TOL_BF16
