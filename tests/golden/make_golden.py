"""Regenerate the golden fixtures in tests/golden/. Run in the container that has the
reference tree (it reads the reference's fixture files and calls the reference's own
kernels compiled into oracle/_ref/libk3ref.so); the outputs are committed so the tests
need neither on the GPU box.

    python tests/golden/make_golden.py [/path/to/reference]

Writes:
  mxfp4_ckpt.npz   from tests/fixtures/mxfp4.json: released-checkpoint MXFP4 bytes (64 rows
                   x 3584 of layers.1 experts.0 w1), the reference's exact dequantised
                   values, and the first 64 values a swapped nibble order would give.
  router_fixture.npz from tests/fixtures/ops/router.json: 6 rows, 8 experts, top-2, hidden
                   128, a bias that changes the selection on 5 rows.
  ref_kernels.npz  outputs of the reference's k3_matmul_mxfp4 / k3_matmul_q8 / k3_router
                   / refh_expert_ffn / refh_moe_layer on small seeded inputs (inputs
                   stored alongside), incl. edge cases (scale 255, scale 0, odd groups).
  ref_router_full.npz the reference's k3_router at the BASELINE shape (384 x 7168, top-8)
                   on 16 seeded bf16 tokens; inputs are regenerated from the seed, a
                   checksum of them is stored to catch generator drift.
  moe_latent_fixture.npz from tests/fixtures/ops/moe.json: the K3 latent MoE layer
                   (hidden 128, latent 64, inter 48, 8 experts, top-2, 2 shared, fp32 expert
                   bank and trunk) with its published output, plus the reference's own
                   k3_moe output on the same inputs.
  ref_latent.npz   the reference's own k3_moe on a seeded latent layer with MXFP4 experts
                   (through an in-memory expert source) and a bf16 trunk (hidden 256,
                   latent 128, inter 128, 8 experts, top-2, 2 shared), 3 tokens; the layer
                   is regenerated from the seed by synth.latent_layer and a checksum of its
                   bytes is stored to catch generator drift.
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import __graft_entry__ as ge  # noqa: E402
from oracle import oracle as ora  # noqa: E402

synth = ge.load_package().synth


def _arr(o):
    return np.asarray(o["data"] if isinstance(o, dict) else o)


def fixture_mxfp4(ref_root):
    d = json.load(open(os.path.join(ref_root, "tests/fixtures/mxfp4.json")))
    rows, pcols = d["rows"], d["packed_cols"]
    packed = _arr(d["packed"]).astype(np.uint8).reshape(rows, pcols)
    scales = _arr(d["scales"]).astype(np.uint8).reshape(rows, d["scale_cols"])
    expected = _arr(d["expected"]).astype(np.float32).reshape(rows, pcols * 2)
    swapped = np.asarray(d["expected_swapped_nibbles"]["first64"], np.float32)
    np.savez_compressed(os.path.join(HERE, "mxfp4_ckpt.npz"), packed=packed, scales=scales,
                        expected=expected, swapped_first64=swapped,
                        group=np.int32(d["group_size"]))


def fixture_router(ref_root):
    r = json.load(open(os.path.join(ref_root, "tests/fixtures/ops/router.json")))
    E, K = r["n_experts"], r["top_k"]
    W = _arr(r["gate_weight"]).astype(np.float32).reshape(E, -1)
    x = _arr(r["in"]).astype(np.float32).reshape(-1, W.shape[1])
    np.savez_compressed(
        os.path.join(HERE, "router_fixture.npz"), W=W, bias=_arr(r["bias"]).astype(np.float32),
        x=x, topk_idx=_arr(r["topk_idx"]).astype(np.int32).reshape(-1, K),
        topk_weight=_arr(r["topk_weight"]).astype(np.float32).reshape(-1, K), top_k=np.int32(K),
        rows_where_bias_changed_selection=np.int32(r["rows_where_bias_changed_selection"]))


def ref_kernels():
    R = ora.ref()
    out = {}
    # MXFP4 GEMV cases: (name, rows, in, group, scale range, seed, edits)
    cases = [("g32", 64, 512, 32, (118, 124), 11), ("g32_wide", 33, 7168, 32, (118, 124), 12),
             ("g16", 17, 96, 16, (120, 130), 13), ("g64", 9, 256, 64, (100, 140), 14),
             ("g24_tail", 5, 70, 24, (110, 125), 15), ("edges", 16, 256, 32, (0, 254), 16)]
    for name, rows, in_, group, (lo, hi), seed in cases:
        g = synth.rng(seed)
        packed = g.integers(0, 256, size=(rows, in_ // 2), dtype=np.uint8)
        ngrp = (in_ + group - 1) // group
        scales = g.integers(lo, hi + 1, size=(rows, ngrp), dtype=np.uint8)
        if name == "edges":
            scales[0, :] = 255          # NaN scale: whole row contributes nothing
            scales[1, ::2] = 255        # every other group skipped
            scales[2, :] = 0            # 2^-127, an fp32 subnormal
            scales[3, :] = 254          # 2^127 * 6 overflows to inf exactly
            scales[4, 3] = 255
        x = g.standard_normal(in_, dtype=np.float32)
        y = np.empty(rows, np.float32)
        R.k3_matmul_mxfp4(y, x, packed, scales, in_, rows, group)
        deq = np.empty((rows, in_), np.float32)
        R.k3_mxfp4_dequant(deq, packed, scales, rows, in_ // 2, group)
        out.update({f"mx_{name}_packed": packed, f"mx_{name}_scales": scales,
                    f"mx_{name}_x": x, f"mx_{name}_y": y, f"mx_{name}_deq": deq,
                    f"mx_{name}_group": np.int32(group)})
    # INT8 per-row GEMV (reference row layout), incl. a ragged `in`
    for name, outn, in_, seed in [("q8a", 48, 512, 21), ("q8b", 7, 131, 22)]:
        g = synth.rng(seed)
        _, _, rows = synth.q8_matrix(g, outn, in_)
        x = g.standard_normal(in_, dtype=np.float32)
        y = np.empty(outn, np.float32)
        R.k3_matmul_q8(y, x, rows, in_, outn)
        out.update({f"{name}_rows": rows, f"{name}_x": x, f"{name}_y": y,
                    f"{name}_in": np.int32(in_)})
    # Router, small: ties and NaN-free; bias on; renorm on/off
    g = synth.rng(31)
    W = (g.standard_normal((24, 64), dtype=np.float32) * 0.3).astype(np.float32)
    x = g.standard_normal((5, 64), dtype=np.float32)
    bias = (g.standard_normal(24, dtype=np.float32) * 0.05).astype(np.float32)
    W[7] = W[3]                         # exact tie between experts 3 and 7
    for renorm in (0, 1):
        idx = np.empty((5, 6), np.int32)
        wt = np.empty((5, 6), np.float32)
        for t in range(5):
            i1 = np.empty(6, np.int32)
            w1 = np.empty(6, np.float32)
            R.k3_router(i1, w1, x[t], W, bias.ctypes.data, 64, 24, 6, renorm, 2.5)
            idx[t], wt[t] = i1, w1
        out[f"rt_idx_r{renorm}"], out[f"rt_wt_r{renorm}"] = idx, wt
    out.update(rt_W=W, rt_x=x, rt_bias=bias)
    # One expert FFN and a small MoE layer through the reference's kernels
    H, I, E, K, T = 256, 128, 12, 3, 4
    g = synth.rng(41)
    experts = [synth.expert(g, H, I) for _ in range(E)]
    shared = synth.expert(g, H, I)
    xf, _ = synth.activations(g, T, H)
    wf, _ = synth.router_weights(g, E, H)
    wf = (wf * 20).astype(np.float32)   # spread the logits so routing is decisive
    y_ffn = ora.expert_ffn(xf, experts[0], H, I, act=0, use_ref=True)
    y_ffn_situ = ora.expert_ffn(xf, experts[0], H, I, act=1, use_ref=True)
    o, idx, wt = ora.moe_layer(xf, wf, None, experts, shared, H, I, K, use_ref=True)
    for e_i, e in enumerate(experts + [shared]):
        for k, v in e.items():
            out[f"moe_e{e_i}_{k}"] = v
    out.update(moe_x=xf, moe_W=wf, moe_out=o, moe_idx=idx, moe_wt=wt, ffn_y=y_ffn,
               ffn_y_situ=y_ffn_situ, moe_dims=np.array([H, I, E, K, T], np.int32))
    np.savez_compressed(os.path.join(HERE, "ref_kernels.npz"), **out)


def ref_router_full():
    g = synth.rng(51)
    wf, wb = synth.router_weights(g)
    xf, xb = synth.activations(g, 16)
    idx = np.empty((16, 8), np.int32)
    wt = np.empty((16, 8), np.float32)
    for t in range(16):
        idx[t], wt[t] = ora.router(xf[t], wf, None, 8, use_ref=True)
    chk = np.array([int(wb.astype(np.uint64).sum()), int(xb.astype(np.uint64).sum())],
                   np.uint64)
    np.savez_compressed(os.path.join(HERE, "ref_router_full.npz"), idx=idx, wt=wt,
                        seed=np.int32(51), input_checksum=chk)


def fixture_moe_latent(ref_root):
    r = json.load(open(os.path.join(ref_root, "tests/fixtures/ops/moe.json")))
    H, Lw, I, E = r["hidden"], r["latent"], r["moe_inter"], r["n_experts"]
    f = lambda k: _arr(r[k]).astype(np.float32)   # noqa: E731
    layer = dict(router_w=f("gate_weight").reshape(E, H),
                 router_bias=f("e_score_correction_bias"),
                 w1=np.stack([f(f"experts_{e}_w1_weight").reshape(I, Lw) for e in range(E)]),
                 w3=np.stack([f(f"experts_{e}_w3_weight").reshape(I, Lw) for e in range(E)]),
                 w2=np.stack([f(f"experts_{e}_w2_weight").reshape(Lw, I) for e in range(E)]),
                 latent_norm=f("norm_weight"), down=f("down_weight").reshape(Lw, H),
                 up=f("up_weight").reshape(H, Lw),
                 sh1=f("shared_w1_weight").reshape(-1, H), sh3=f("shared_w3_weight").reshape(-1, H),
                 sh2=f("shared_w2_weight").reshape(H, -1), wdt=0, hidden=H, latent=Lw, inter=I,
                 n_shared=r["n_shared"], n_experts=E, topk=r["top_k"], renorm=int(r["renorm"]),
                 latent_norm_on=int(r["latent_norm"]), routed_scale=float(r["routed_scale"]),
                 rms_eps=float(r["rms_eps"]), situ_b1=float(r["situ_b1"]),
                 situ_b2=float(r["situ_b2"]))
    x = f("in").reshape(-1, H)
    want = f("out").reshape(-1, H)
    ref_out, ref_idx, ref_wt = ora.moe_latent(x, layer, use_ref=True)
    arrays = {k: v for k, v in layer.items() if isinstance(v, np.ndarray)}
    scalars = {k: np.asarray(v) for k, v in layer.items() if not isinstance(v, np.ndarray)}
    np.savez_compressed(os.path.join(HERE, "moe_latent_fixture.npz"), x=x, want=want,
                        ref_out=ref_out, ref_idx=ref_idx, ref_wt=ref_wt, **arrays, **scalars)


LATENT_CASE = dict(seed=61, hidden=256, latent=128, inter=128, n_experts=8, topk=2, n_shared=2,
                   ntok=3)


def latent_case():
    """The seeded latent layer and tokens of ref_latent.npz (shared with the tests)."""
    c = LATENT_CASE
    g = synth.rng(c["seed"])
    layer = synth.latent_layer(g, c["hidden"], c["latent"], c["inter"], c["n_experts"],
                               c["topk"], c["n_shared"], wdt=1)
    x, _ = synth.activations(g, c["ntok"], c["hidden"], bf16=False)
    return layer, x


def layer_checksum(layer):
    h = np.uint64(1469598103934665603)
    parts = [layer[k] for k in ("router_w", "router_bias", "latent_norm", "down", "up", "sh1",
                                "sh3", "sh2")]
    parts += [e[k] for e in layer["experts"] for k in sorted(e)]
    total = 0
    for a in parts:
        total = (total * 1000003 + int(np.frombuffer(np.ascontiguousarray(a).tobytes(),
                                                     np.uint8).astype(np.uint64).sum())) % (1 << 61)
    return np.int64(total + int(h % 7))


def ref_latent():
    layer, x = latent_case()
    out, idx, wt = ora.moe_latent(x, layer, use_ref=True)
    np.savez_compressed(os.path.join(HERE, "ref_latent.npz"), x=x, out=out, idx=idx, wt=wt,
                        checksum=layer_checksum(layer))


def main():
    ref_root = sys.argv[1] if len(sys.argv) > 1 else "/root/reference"
    fixture_mxfp4(ref_root)
    fixture_router(ref_root)
    ref_kernels()
    ref_router_full()
    fixture_moe_latent(ref_root)
    ref_latent()
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f"{f}: {os.path.getsize(os.path.join(HERE, f))} bytes")


if __name__ == "__main__":
    main()
