"""The K3 latent MoE layer and its trunk operations on the GPU against the oracle and the
reference's own outputs: trunk matmuls bit-exact (k3_matmul / k3_matmul_bf16 order), the
layer within the decode tolerance with exact routing."""
import ctypes as C

import numpy as np
import pytest

from conftest import maxrel

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    import torch
    return torch.device("cuda:0")


def T(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


@pytest.mark.parametrize("out_,in_", [(37, 7168), (64, 35), (5, 16), (3, 7), (130, 2048),
                                      (1000, 3584)])
@pytest.mark.parametrize("ntok", [1, 3, 16, 32])
def test_mmw_bit_exact(k3, ora, dev, out_, in_, ntok):
    g = k3.synth.rng(out_ * 7 + in_ * 3 + ntok)
    W = g.standard_normal((out_, in_), dtype=np.float32)
    x = g.standard_normal((ntok, in_), dtype=np.float32)
    Wb = k3.synth.bf16_bits(W)
    yf = k3.mmw(T(x, dev), T(W, dev), k3.WF32).cpu().numpy()
    yb = k3.mmw(T(x, dev), T(Wb.view(np.int16), dev), k3.WBF16).cpu().numpy()
    for t in range(ntok):
        assert np.array_equal(yf[t].view(np.uint32), ora.matmul_f32(x[t], W).view(np.uint32))
        assert np.array_equal(yb[t].view(np.uint32), ora.matmul_bf16(x[t], Wb).view(np.uint32))


def test_mmw_accumulate_and_strides(k3, ora, dev):
    import torch
    g = k3.synth.rng(5)
    W = g.standard_normal((96, 200), dtype=np.float32)
    x = g.standard_normal((4, 200), dtype=np.float32)
    base = g.standard_normal((4, 160), dtype=np.float32)
    out = T(base, dev)
    # write into columns 40..135 of a wider row, adding to what is there
    view = out[:, 40:136]
    L = k3.lib()
    xd, Wd = T(x, dev), T(W, dev)          # held: the kernel reads them after this line
    rc = L.k3c_mmw(C.c_void_p(view.data_ptr()), 160, C.c_void_p(xd.data_ptr()), 200, 4,
                   C.c_void_p(Wd.data_ptr()), k3.WF32, 200, 96, 1,
                   C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    got = out.cpu().numpy()
    for t in range(4):
        want = (base[t, 40:136] + ora.matmul_f32(x[t], W)).astype(np.float32)
        assert np.array_equal(got[t, 40:136], want)
        assert np.array_equal(got[t, :40], base[t, :40]) and np.array_equal(got[t, 136:], base[t, 136:])


def test_host_dropin_trunk_matmuls(k3, ora):
    g = k3.synth.rng(9)
    L = k3.lib()
    for out_, in_ in [(300, 7168), (17, 45)]:
        W = g.standard_normal((out_, in_), dtype=np.float32)
        x = g.standard_normal(in_, dtype=np.float32)
        Wb = k3.synth.bf16_bits(W)
        y = np.empty(out_, np.float32)
        L.k3_matmul(y.ctypes.data, x.ctypes.data, W.ctypes.data, in_, out_)
        assert np.array_equal(y, ora.matmul_f32(x, W))
        L.k3_matmul_bf16(y.ctypes.data, x.ctypes.data, Wb.ctypes.data, in_, out_)
        assert np.array_equal(y, ora.matmul_bf16(x, Wb))


def test_rmsnorm_and_situ(k3, ora, dev):
    g = k3.synth.rng(11)
    x = (g.standard_normal((5, 3584), dtype=np.float32) * 3).astype(np.float32)
    w = (1 + 0.1 * g.standard_normal(3584, dtype=np.float32)).astype(np.float32)
    got = k3.rmsnorm(T(x, dev), T(w, dev), 1e-5).cpu().numpy()
    assert maxrel(got, ora.rmsnorm(x, w, 1e-5)) < 1e-6
    # both soft caps saturate over this range (the reference's situ_glu fixture spans
    # |z| 0.1..1000 for the same reason)
    gu = (np.sign(g.standard_normal((3, 2 * 1000))) *
          10 ** g.uniform(-1, 3, (3, 2 * 1000))).astype(np.float32)
    got = k3.situ_glu(T(gu, dev)).cpu().numpy()
    assert maxrel(got, ora.situ_glu(gu)) < 1e-6


def test_latent_layer_matches_reference_k3_moe(k3, golden, golden_gen, dev):
    # the reference's own k3_moe output (MXFP4 experts through an expert source, bf16 trunk)
    r = golden("ref_latent.npz")
    layer, x = golden_gen.latent_case()
    assert golden_gen.layer_checksum(layer) == r["checksum"]
    lat = k3.LatentMoeLayer.from_host(layer, dev, terms=3)
    out, idx, wt = lat.decode(T(x, dev))
    assert np.array_equal(idx.cpu().numpy(), r["idx"])
    assert np.array_equal(wt.cpu().numpy(), r["wt"])
    assert maxrel(out.cpu().numpy(), r["out"]) < 2e-2


@pytest.mark.parametrize("ntok,wdt", [(1, 1), (16, 1), (32, 0), (100, 1), (300, 0), (16, 2), (70, 2)])
def test_latent_layer_vs_oracle(k3, ora, dev, ntok, wdt):
    g = k3.synth.rng(100 + ntok)
    layer = k3.synth.latent_layer(g, 1024, 512, 256, 32, 4, n_shared=2, wdt=wdt)
    x = g.standard_normal((ntok, 1024), dtype=np.float32)
    want, widx, wwt = ora.moe_latent(x, layer)
    lat = k3.LatentMoeLayer.from_host(layer, dev, terms=3)
    import torch
    drops = torch.zeros(1, dtype=torch.int32, device=dev)
    out, idx, wt = lat.decode(T(x, dev), drops=drops)
    assert np.array_equal(idx.cpu().numpy(), widx)
    assert np.array_equal(wt.cpu().numpy(), wwt)
    assert int(drops.item()) == 0
    assert maxrel(out.cpu().numpy(), want) < 2e-2


@pytest.mark.parametrize("ntok", [8, 48])
@pytest.mark.parametrize("variant", ["no_shared", "no_norm", "no_bias"])
def test_latent_layer_optional_parts(k3, ora, dev, ntok, variant):
    """The layer's optional parts: no shared expert (n_shared = 0), no aggregate RMSNorm,
    no router bias; through the decode kernels (8 tokens) and the prefill kernels (48)."""
    g = k3.synth.rng(200 + ntok)
    layer = k3.synth.latent_layer(g, 512, 256, 128, 16, 4, n_shared=0 if variant == "no_shared" else 1,
                                  wdt=1)
    if variant == "no_norm":
        layer["latent_norm_on"] = 0
    if variant == "no_bias":
        layer["router_bias"] = None
    if variant == "no_shared":
        for k in ("sh1", "sh3", "sh2"):
            layer[k] = None
    x = g.standard_normal((ntok, 512), dtype=np.float32)
    want, widx, _ = ora.moe_latent(x, layer)
    out, idx, _ = k3.LatentMoeLayer.from_host(layer, dev).decode(T(x, dev))
    assert np.array_equal(idx.cpu().numpy(), widx)
    assert maxrel(out.cpu().numpy(), want) < 2e-2


@pytest.mark.parametrize("ntok", [8, 48])
def test_latent_layer_cache_only(k3, ora, dev, ntok):
    """The draft model's cache-only routing inside the latent layer (k3c_moe_latent_layer
    .cache_only): route among the experts with a run only, renormalise, count no drops --
    against the reference's own k3_moe with cache_only set and an expert source whose
    resident() reports the same set (src/core/k3_ops.c:580-593)."""
    if not ora.ref_available():
        pytest.skip("oracle/_ref not built")
    import torch
    from dropin_util import HostSource, MoeArgs, reference
    g = k3.synth.rng(600 + ntok)
    layer = k3.synth.latent_layer(g, 512, 256, 128, 16, 6, n_shared=1, wdt=1)
    x = g.standard_normal((ntok, 512), dtype=np.float32)
    resident = [e for e in range(16) if e % 4 != 2]
    lat = k3.LatentMoeLayer.from_host(layer, dev, cache_only=1)
    run_of = lat._keep[1]
    run_of.copy_(torch.tensor([e if e in resident else -1 for e in range(16)], dtype=torch.int32))
    drops = torch.zeros(1, dtype=torch.int32, device=dev)
    out, idx, wt = lat.decode(T(x, dev), drops=drops)
    src = HostSource(k3, layer["experts"], resident=set(resident))
    rout, ridx, rwt, rd = reference(ora, MoeArgs(k3, layer, src.src, cache_only=1), x)
    idx = idx.cpu().numpy()
    assert int(drops.item()) == 0 and rd == 0
    assert np.isin(idx[idx >= 0], resident).all() and (idx < 0).any()
    m = int((idx[-1] >= 0).sum())
    assert np.array_equal(idx[-1, :m], ridx[:m])
    assert np.array_equal(wt.cpu().numpy()[-1, :m].view(np.uint32), rwt[:m].view(np.uint32))
    assert maxrel(out.cpu().numpy(), rout) < 2e-2
