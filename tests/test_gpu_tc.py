"""GPU parity of the tcgen05 block-scaled MoE path (k3c_moe_decode_tc) and of the pool
format it reads.

Activations enter the tensor core as J E4M3 terms with power-of-two block scales, so the
path is exact in the weights and approximates the activations to ~4J bits relative to each
32-element block maximum. The BASELINE tolerance for bf16-activation runs is 2e-2 relative
(max|got-want| / max|want|); router indices must match exactly.
"""
import numpy as np
import pytest

from conftest import maxrel

pytestmark = pytest.mark.gpu

TOL_BF16 = 2e-2


@pytest.fixture(scope="module")
def dev():
    import torch
    return torch.device("cuda:0")


def T(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _atoms(scales, rows, groups):
    """[rows][groups] scale bytes -> [rows/128][groups/4][512] atoms, byte
    16*(m%32) + 4*(m//32) + g for row m and group g of a tile."""
    t = scales.reshape(rows // 128, 128, groups // 4, 4).transpose(0, 2, 1, 3)  # rt,kt,m,g
    t = t.reshape(rows // 128, groups // 4, 4, 32, 4).transpose(0, 1, 3, 2, 4)   # rt,kt,i,q,g
    return t.reshape(-1)


def pool_layout_ref(e, H, I):
    """numpy restatement of the pool-format run (see csrc/moe_tc.cu)."""
    R = np.arange(2 * I)
    m = R % 128
    which = (m >= 64)[:, None]
    row = 64 * (R // 128) + (m & 63)
    gup = np.where(which, e["up_p"][row], e["gate_p"][row]).copy()
    gus = np.where(which, e["up_s"][row], e["gate_s"][row]).copy()
    dp, ds = e["down_p"].copy(), e["down_s"].copy()
    for p, s in ((gup, gus), (dp, ds)):
        bad = s == 255
        p.reshape(p.shape[0], -1, 16)[bad] = 0
        s[bad] = 127
    return np.concatenate([gup.ravel(), _atoms(gus, 2 * I, H // 32), dp.ravel(),
                           _atoms(ds, H, I // 32)])


def test_pool_pack_is_the_documented_layout(k3, dev):
    import torch
    H, I = 256, 256
    g = k3.synth.rng(11)
    e = k3.synth.expert(g, H, I, scale_lo=110, scale_hi=130)
    e["gate_s"][3, 2] = 255
    e["down_s"][7, 5] = 255
    run = torch.zeros(k3.pool_run_bytes(H, I), dtype=torch.uint8, device=dev)
    k3.pool_pack(run, k3.DeviceExpert.from_host(e, dev).q(), H, I)
    got = run.cpu().numpy()
    assert np.array_equal(got, pool_layout_ref(e, H, I))


def _small_layer(k3, dev, H, I, E, K, terms, seed, shared=True):
    import torch
    g = k3.synth.rng(seed)
    experts = [k3.synth.expert(g, H, I) for _ in range(E)]
    sh = k3.synth.expert(g, H, I) if shared else None
    wf, wb = k3.synth.router_weights(g, E, H)
    wf = (wf * 20).astype(np.float32)          # decisive routing at small hidden sizes
    wb = k3.synth.bf16_bits(wf)
    wf = k3.synth.bf16_to_f32(wb)
    devs = [k3.DeviceExpert.from_host(e, dev) for e in experts]
    W = T(wb.view(np.int16), dev).view(torch.bfloat16)
    layer = k3.PoolMoeLayer.pack(devs, k3.DeviceExpert.from_host(sh, dev) if shared else None,
                                 W, None, H, I, K, dev, terms=terms)
    return layer, experts, sh, wf, g


@pytest.mark.parametrize("terms", [3])
def test_tc_decode_small_vs_oracle(k3, ora, dev, terms):
    H, I, E, K, Tn = 256, 128, 8, 2, 3
    layer, experts, sh, wf, g = _small_layer(k3, dev, H, I, E, K, terms, seed=21)
    xf, xb = k3.synth.activations(g, Tn, H)
    out, idx, wt = layer.decode(T(xb.view(np.int16), dev))
    ro, ri, rw = ora.moe_layer(xf, wf, None, experts, sh, H, I, K)
    assert np.array_equal(idx.cpu().numpy(), ri)
    err = maxrel(out.cpu().numpy(), ro)
    print(f"tc small terms={terms}: maxrel {err:.3e}")
    assert err < TOL_BF16


def test_tc_decode_error_shrinks_with_terms(k3, ora, dev):
    H, I, E, K, Tn = 512, 256, 8, 2, 4
    errs = []
    for terms in (1, 2, 3):
        layer, experts, sh, wf, g = _small_layer(k3, dev, H, I, E, K, terms, seed=33)
        xf, xb = k3.synth.activations(g, Tn, H)
        out, idx, wt = layer.decode(T(xb.view(np.int16), dev))
        ro, ri, rw = ora.moe_layer(xf, wf, None, experts, sh, H, I, K)
        errs.append(maxrel(out.cpu().numpy(), ro))
    print("tc maxrel by terms:", errs)
    assert errs[0] > errs[1] > errs[2]
    assert errs[2] < 5e-3


@pytest.mark.parametrize("ntok", [1, 16])
def test_tc_decode_config1_shape(k3, ora, dev, ntok):
    """BASELINE config[1] shapes: hidden 7168, inter 2048, 384 experts (24 distinct runs
    tiled over the ids), top-8, shared expert, bf16 x and router."""
    import torch
    H, I, E, K, D = 7168, 2048, 384, 8, 24
    g = k3.synth.rng(500 + ntok)
    distinct = [k3.synth.expert(g) for _ in range(D)]
    sh = k3.synth.expert(g)
    wf, wb = k3.synth.router_weights(g, E, H)
    xf, xb = k3.synth.activations(g, ntok, H)
    devs = [k3.DeviceExpert.from_host(e, dev) for e in distinct]
    W = T(wb.view(np.int16), dev).view(torch.bfloat16)
    layer = k3.PoolMoeLayer.pack(devs, k3.DeviceExpert.from_host(sh, dev), W, None, H, I, K, dev,
                                 expert_map=[i % D for i in range(E)], terms=3)
    drops = torch.zeros(1, dtype=torch.int32, device=dev)
    out, idx, wt = layer.decode(T(xb.view(np.int16), dev), drops=drops)
    ro, ri, rw = ora.moe_layer(xf, wf, None, [distinct[i % D] for i in range(E)], sh, H, I, K)
    assert drops.item() == 0
    assert np.array_equal(idx.cpu().numpy(), ri)
    err = maxrel(out.cpu().numpy(), ro)
    print(f"tc config1 ntok={ntok}: maxrel {err:.3e}")
    assert err < TOL_BF16
