"""Seeded synthetic inputs with the BASELINE configs' shapes and value distributions.

There is no checkpoint and no dataset on the GPU box; every workload is synthetic:

  * MXFP4 matrices: packed bytes uniform over 0..255 (so each E2M1 code is uniform over
    all 16 values) and one E8M0 scale byte per 32 input elements, uniform in [118, 124];
  * activations ~ N(0, 1), rounded to bf16 where the config says bf16;
  * router weights ~ N(0, 0.02) in bf16;
  * INT8 trunk weights uniform in [-127, 127] with one fp32 row scale ~ U(1e-3, 1e-2).

numpy's PCG64 stream is the generator, so a seed names the same bytes on every host.
"""
from __future__ import annotations

import numpy as np

HIDDEN = 7168
INTER = 2048
N_EXPERTS = 384
TOPK = 8
GROUP = 32
SCALE_LO, SCALE_HI = 118, 124


def rng(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(seed))


def bf16_bits(a: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns, round to nearest even (finite inputs)."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return r.astype(np.uint16)


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    """bf16 bits -> fp32: a left shift by 16, exact (the reference's k3_bf16f)."""
    return (np.ascontiguousarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


def mxfp4_matrix(g: np.random.Generator, rows: int, cols: int,
                 scale_lo: int = SCALE_LO, scale_hi: int = SCALE_HI):
    """(packed [rows][cols/2] u8, scales [rows][cols/32] u8) in the reference layout."""
    packed = g.integers(0, 256, size=(rows, cols // 2), dtype=np.uint8)
    scales = g.integers(scale_lo, scale_hi + 1, size=(rows, (cols + GROUP - 1) // GROUP),
                        dtype=np.uint8)
    return packed, scales


def expert(g: np.random.Generator, hidden: int = HIDDEN, inter: int = INTER, **kw) -> dict:
    """One routed expert: gate/up [inter][hidden], down [hidden][inter], all MXFP4."""
    gp, gs = mxfp4_matrix(g, inter, hidden, **kw)
    up, us = mxfp4_matrix(g, inter, hidden, **kw)
    dp, ds = mxfp4_matrix(g, hidden, inter, **kw)
    return dict(gate_p=gp, gate_s=gs, up_p=up, up_s=us, down_p=dp, down_s=ds)


def expert_bytes(hidden: int = HIDDEN, inter: int = INTER) -> int:
    """Algorithmic bytes of one MXFP4 expert: 3 matrices of packed nibbles + scales."""
    m = inter * hidden // 2 + inter * hidden // GROUP
    return 3 * m


def activations(g: np.random.Generator, ntok: int, hidden: int = HIDDEN, bf16=True):
    """x ~ N(0,1); returns (fp32 values, bf16 bits or None). With bf16=True the fp32 array
    holds exactly the bf16 values."""
    x = g.standard_normal((ntok, hidden), dtype=np.float32)
    if not bf16:
        return x, None
    b = bf16_bits(x)
    return bf16_to_f32(b), b


def router_weights(g: np.random.Generator, n_experts: int = N_EXPERTS,
                   hidden: int = HIDDEN):
    """W_r ~ N(0, 0.02) in bf16; returns (fp32 values, bf16 bits)."""
    w = g.standard_normal((n_experts, hidden), dtype=np.float32) * np.float32(0.02)
    b = bf16_bits(w)
    return bf16_to_f32(b), b


def q8_matrix(g: np.random.Generator, out: int, in_: int):
    """INT8 trunk matrix: (int8 [out][in], fp32 scales [out], reference row bytes).

    The reference row layout is [f32 scale][int8 * in], stride 4+in bytes
    (include/k3/k3.h:265-303)."""
    w = g.integers(-127, 128, size=(out, in_), dtype=np.int8)
    s = g.uniform(1e-3, 1e-2, size=out).astype(np.float32)
    rows = np.empty((out, 4 + in_), np.uint8)
    rows[:, :4] = s.view(np.uint8).reshape(out, 4)
    rows[:, 4:] = w.view(np.uint8)
    return w, s, rows


def zipf_bias(n_experts: int, s: float = 1.1, alpha: float = 0.0,
              perm: np.ndarray | None = None) -> np.ndarray:
    """Selection bias b_e = alpha * log(rank_e^-s): steers top-k popularity toward a Zipf
    law over experts (rank 1 most popular). perm maps rank -> expert id."""
    ranks = np.arange(1, n_experts + 1, dtype=np.float64)
    b = alpha * (-s) * np.log(ranks)
    out = np.empty(n_experts, np.float32)
    ids = np.arange(n_experts) if perm is None else perm
    out[ids] = b.astype(np.float32)
    return out


def zipf_topk_marginal(n_experts: int, s: float = 1.1, topk: int = 8, samples: int = 65536,
                       seed: int = 1, device="cpu"):
    """Expert popularity when every token draws topk distinct experts with Zipf(s) weights
    (rank r = expert id r-1), estimated by Gumbel-top-k sampling. Under top-k routing no
    expert can take more than 1/topk of the pairs, so this -- not the Zipf law itself -- is
    the reachable target."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    logw = -s * torch.log(torch.arange(1, n_experts + 1, dtype=torch.float64, device=device))
    u = torch.rand((samples, n_experts), generator=g, device=device, dtype=torch.float64)
    top = torch.topk(logw[None, :] - torch.log(-torch.log(u)), topk, dim=1).indices
    cnt = torch.bincount(top.reshape(-1), minlength=n_experts).to(torch.float64)
    return cnt / cnt.sum()


def zipf_fit_bias(scores, s: float = 1.1, topk: int = 8, iters: int = 1500, step: float = 0.05,
                  seed: int = 1):
    """Router selection bias (fp32, max 0) fitted so that top-k(score + bias) over the sample
    `scores` [tokens][experts] (a torch tensor of sigmoid router scores) reproduces
    zipf_topk_marginal: a Zipf(s) popularity over expert ids. The fixed form
    alpha*log(rank^-s) cannot reach it -- the bounded sigmoid scores cut its tail off -- so
    the bias is found by damped proportional updates in log space."""
    import torch
    T, E = scores.shape
    target = zipf_topk_marginal(E, s, topk, seed=seed, device=scores.device)
    sc = scores.to(torch.float64)
    b = torch.zeros(E, dtype=torch.float64, device=scores.device)
    eps = 1.0 / (T * topk)
    for it in range(iters):
        top = torch.topk(sc + b[None, :], topk, dim=1).indices
        p = torch.bincount(top.reshape(-1), minlength=E).to(torch.float64) / (T * topk)
        b += step * torch.clamp(torch.log((target + eps) / (p + eps)), -1.0, 1.0) / (1 + it / 300)
        b -= b.max()
    return b.to(torch.float32)


def latent_layer(g: np.random.Generator, hidden: int, latent: int, inter: int,
                 n_experts: int, topk: int, n_shared: int = 2, wdt: int = 1,
                 scale_lo: int = SCALE_LO, scale_hi: int = SCALE_HI) -> dict:
    """One K3 latent MoE layer with the fields of the oracle's ora_latent: an fp32 router
    [n_experts][hidden] (spread so routing is decisive), routed MXFP4 experts at the latent
    width (``experts``), trunk matrices down [latent][hidden], up [hidden][latent],
    sh1/sh3 [inter*n_shared][hidden], sh2 [hidden][inter*n_shared] as bf16 bit patterns
    (wdt=1), fp32 (wdt=0), each ~N(0, 1/in), or per-row int8 in the reference's row layout
    [f32 scale][int8 * in] (wdt=2, the draft model's trunk; scale ~ 1/(64 sqrt(in)) so the
    rows have the same spread), and latent-norm weights near 1."""
    SI = inter * n_shared

    def trunk(out_, in_):
        if wdt == 2:
            w = g.integers(-127, 128, size=(out_, in_), dtype=np.int8)
            sc = (g.uniform(0.5, 1.5, out_) / (64 * np.sqrt(in_))).astype(np.float32)
            rows = np.empty((out_, 4 + in_), np.uint8)
            rows[:, :4] = sc.view(np.uint8).reshape(out_, 4)
            rows[:, 4:] = w.view(np.uint8)
            return rows
        w = g.standard_normal((out_, in_), dtype=np.float32) * np.float32(1.0 / np.sqrt(in_))
        return bf16_bits(w) if wdt == 1 else w

    router = g.standard_normal((n_experts, hidden), dtype=np.float32) * np.float32(0.4)
    if wdt == 1:
        router = bf16_to_f32(bf16_bits(router))
    return dict(
        router_w=router.astype(np.float32),
        router_bias=(g.standard_normal(n_experts, dtype=np.float32) * 0.05).astype(np.float32),
        experts=[expert(g, latent, inter, scale_lo=scale_lo, scale_hi=scale_hi)
                 for _ in range(n_experts)],
        latent_norm=(1.0 + 0.1 * g.standard_normal(latent, dtype=np.float32)).astype(np.float32),
        down=trunk(latent, hidden), up=trunk(hidden, latent),
        sh1=trunk(SI, hidden) if SI else None, sh3=trunk(SI, hidden) if SI else None,
        sh2=trunk(hidden, SI) if SI else None,
        wdt=wdt, hidden=hidden, latent=latent, inter=inter, n_shared=n_shared,
        n_experts=n_experts, topk=topk, renorm=1, latent_norm_on=1,
        routed_scale=1.0, rms_eps=1e-5, situ_b1=4.0, situ_b2=25.0)


def zipf_router(device, n_experts: int = N_EXPERTS, hidden: int = HIDDEN, topk: int = TOPK,
                s: float = 1.1, seed: int = 77, sample: int = 2048, perm_seed: int = 5,
                iters: int = 600):
    """The Zipf(s)-skewed router of BASELINE configs [2] and [3], generated on `device`:
    W_r ~ N(0, 0.02) in bf16 and a selection bias fitted (zipf_fit_bias) on a separate sample
    of `sample` bf16 tokens so that expert popularity follows Zipf(s) over a fixed random
    permutation of the expert ids. The same seeds give the same tensors on every process of
    one device type. Returns (W bf16 [E][H], bias fp32 [E], the sample tokens bf16)."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    W = (torch.randn((n_experts, hidden), generator=g, device=device) * 0.02).to(torch.bfloat16)
    smp = torch.randn((sample, hidden), generator=g, device=device).to(torch.bfloat16)
    scores = torch.sigmoid(smp.float() @ W.float().T)
    perm = torch.randperm(n_experts, generator=torch.Generator().manual_seed(perm_seed)).to(device)
    b_rank = zipf_fit_bias(scores[:, perm], s=s, topk=topk, iters=iters)
    bias = torch.empty_like(b_rank)
    bias[perm] = b_rank
    return W, bias, smp


def device_bank(k3, n: int, hidden: int = HIDDEN, inter: int = INTER, device="cuda", seed: int = 4242):
    """n MXFP4 experts generated on the device with the BASELINE distributions (packed bytes
    uniform over 0..255, scale bytes uniform in [118, 124]) in the reference's expert-run
    layout, and the same experts packed into pool-format runs for the tensor-core kernels.
    The same seed gives the same bytes on every process of one device type, so ranks that
    each hold a share of the experts agree on every expert's weights.
    Returns (ref_runs uint8 [n][run], arena uint8 [n * pool_run_bytes])."""
    import torch
    lay, run = k3.expert_run_layout(hidden, inter)
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    ref = torch.empty((n, run), dtype=torch.uint8, device=device)
    for name, (off, nb) in lay.items():
        seg = ref[:, off:off + nb]
        if name.endswith("_p"):
            seg.random_(0, 256, generator=g)
        else:
            seg.random_(SCALE_LO, SCALE_HI + 1, generator=g)
    stride = k3.pool_run_bytes(hidden, inter)
    arena = torch.empty(n * stride, dtype=torch.uint8, device=device)
    for i, q in enumerate(k3.experts_from_blob(ref, n, hidden, inter)):
        k3.pool_pack(arena[i * stride:(i + 1) * stride], q, hidden, inter)
    return ref, arena


def host_expert(ref_runs, i: int, hidden: int = HIDDEN, inter: int = INTER, layout=None) -> dict:
    """Expert i of a device_bank as the host dict of expert(): numpy uint8 arrays in the
    reference layout (gate/up [inter][hidden/2] + [inter][hidden/32], down [hidden][inter/2] +
    [hidden][inter/32])."""
    if layout is None:
        parts = [("gate_p", inter * hidden // 2), ("gate_s", inter * hidden // 32),
                 ("down_p", hidden * inter // 2), ("down_s", hidden * inter // 32),
                 ("up_p", inter * hidden // 2), ("up_s", inter * hidden // 32)]
        off, layout = 0, {}
        for name, nb in parts:
            layout[name] = (off, nb)
            off += nb
    run = ref_runs[i].cpu().numpy()
    shapes = {"gate_p": (inter, hidden // 2), "gate_s": (inter, hidden // GROUP),
              "up_p": (inter, hidden // 2), "up_s": (inter, hidden // GROUP),
              "down_p": (hidden, inter // 2), "down_s": (hidden, inter // GROUP)}
    return {k: np.ascontiguousarray(run[o:o + nb].reshape(shapes[k])) for k, (o, nb) in layout.items()}
