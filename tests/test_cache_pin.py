"""Pins the cache bookkeeping restatement (oracle/cache_model.py, the model the GPU pool's
counters and slot choices are tested against) to the reference's OWN expert cache: the
reference's k3_cache (src/cache/k3_cache.c, compiled into oracle/_ref) replays a seeded
request sequence over a small checkpoint and, after every request, its key_of table must equal
the model's, slot for slot; the counters, the (layer, expert) access trace and the request
histogram must match at the end.

The sequence mixes get (admit, k3_cache.c:60-108), batch getmany (:131-234), pin and unpin
(:375-383), with evictions under a hot/cold id mix. Each getmany asks for distinct ids in
ascending order over a checkpoint whose experts lie in id order, so the reference's
disk-offset issue order is the request order and its two clock ticks per slot (reserve,
publish) order the slots as the model's single tick does -- the one adaptation of the model
that the pool relies on. User pins stay below nslot - topk - 1, so every request finds a slot
(the constructor's nslot >= topk + 1 guarantee)."""
import os

import numpy as np
import pytest

from ckpt_util import expert_tensors, write_shard
from oracle.cache_model import CacheModel

NL, NE, TOPK, NSLOT = 2, 12, 4, 7


def _checkpoint(d):
    g = np.random.default_rng(5)
    tensors = [("model.embed_filler", g.integers(0, 256, 123, dtype=np.uint8), None)]
    for layer in range(NL):
        for e in range(NE):
            tensors += expert_tensors(g, layer, e, 64, 32)[0]
    os.makedirs(d, exist_ok=True)
    write_shard(os.path.join(d, "model-00001-of-00001.safetensors"), tensors)


def _records(seed, n):
    g = np.random.default_rng(seed)
    hot = np.array([1, 4, 7])
    recs = []
    for _ in range(n):
        r = g.random()
        layer = int(g.integers(0, NL))
        if r < 0.55:
            e = int(g.choice(hot)) if g.random() < 0.5 else int(g.integers(0, NE))
            recs.append((0, layer, [e]))
        elif r < 0.85:
            k = int(g.integers(1, TOPK + 1))
            recs.append((1, layer, sorted(g.choice(NE, k, replace=False).tolist())))
        else:
            recs.append((2 if g.random() < 0.6 else 3, layer, [int(g.integers(0, NE))]))
    return recs


def _model_replay(recs):
    m = CacheModel(NL, NE, NSLOT)
    user = set()   # slots pinned by pin records (the reference's pinned flag)
    keys, rcs, trace = [], [], []
    hist = [0] * (NL * NE)
    for kind, layer, ids in recs:
        key = layer * NE + ids[0]
        if kind == 0:
            trace.append((layer, ids[0]))
            hist[key] += 1
            m.acquire(layer, ids)
            m.release(layer, ids)
            rc = 0
        elif kind == 1:
            rc = m.getmany(layer, ids)
        else:
            s = m.slot_of.get(key, -1)
            rc = int(s >= 0)
            if s >= 0 and kind == 2 and s not in user:
                user.add(s)
                m.pins[s] += 1
            elif s >= 0 and kind == 3 and s in user:
                user.discard(s)
                m.pins[s] -= 1
        keys.append(list(m.key_of))
        rcs.append(rc)
    return m, keys, rcs, trace, hist


def _limit_pins(recs):
    """Drop pin records that would pin more than nslot - topk - 1 slots at once (tracked on
    the model, which holds the same slots as the reference at every step)."""
    m = CacheModel(NL, NE, NSLOT)
    user, out = set(), []
    for kind, layer, ids in recs:
        key = layer * NE + ids[0]
        if kind == 0:
            m.acquire(layer, ids)
            m.release(layer, ids)
        elif kind == 1:
            m.getmany(layer, ids)
        else:
            s = m.slot_of.get(key, -1)
            if kind == 2 and s >= 0 and s not in user:
                if len(user) >= NSLOT - TOPK - 1:
                    continue
                user.add(s)
                m.pins[s] += 1
            elif kind == 3 and s >= 0 and s in user:
                user.discard(s)
                m.pins[s] -= 1
        out.append((kind, layer, ids))
    return out


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_cache_model_matches_reference_cache(ora, tmp_path, seed):
    if not ora.ref_available():
        pytest.skip("oracle/_ref not built (needs the reference tree)")
    import __graft_entry__ as ge
    k3 = ge.load_package()
    d = str(tmp_path / "ckpt")
    _checkpoint(d)
    recs = _limit_pins(_records(seed, 400))
    cfg = k3.K3CfgC()
    cfg.n_layers, cfg.n_experts, cfg.topk, cfg.first_dense = NL, NE, TOPK, 0
    ref = ora.ref_cache_replay(d, cfg, NSLOT, recs)
    assert ref is not None, "the reference cache did not open the checkpoint"
    m, keys, rcs, trace, hist = _model_replay(recs)
    for i, (want, got) in enumerate(zip(ref["key_of"], keys)):
        assert got == want, f"record {i} {recs[i]}: model slots {got}, reference {want}"
    assert rcs == ref["rc"]
    st = m.stats()
    for k in ("hits", "misses", "evictions", "prefetch_reads"):
        assert st[k] == ref[k], (k, st[k], ref[k])
    assert trace == ref["trace"]
    assert hist == ref["hist"]
    assert ref["evictions"] > 20 and ref["prefetch_reads"] > 20 and ref["hits"] > 20
