"""k3c_moe_decode_noalloc: MoE decode for callers that cannot allocate device memory.

Some callers of this library cannot call cudaMalloc: an engine that owns all device memory
and gives the library no allocator, or a decode loop whose host code must not block on an
allocation. For them k3c_moe_decode_noalloc takes its scratch from a fixed 8 MiB device
array inside the library instead of from the caller. These tests call it through the C ABI
and check that it returns what the existing entry point k3c_moe_decode returns, on two
calls in a row, and that it refuses a batch whose scratch would not fit.

This file is collected last on purpose (tests/test_zz_*), so that a run stopping at the
first failure has already run every other test. It passes alone in a fresh process too.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import maxrel

pytestmark = pytest.mark.gpu

TOL_F32 = 1e-5       # the tolerance every GPU parity test here uses
K3C_EINVAL = -1


def _bind(k3):
    L = k3.lib()
    fn = L.k3c_moe_decode_noalloc
    fn.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.POINTER(k3.MoeLayerC),
                   C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]
    fn.restype = C.c_int
    return L, fn


def _layer(k3, dev, H, I, E, K, distinct, seed):
    import torch
    g = k3.synth.rng(seed)
    uniq = [k3.synth.expert(g, H, I) for _ in range(distinct)]
    shared = k3.synth.expert(g, H, I)
    _, wb = k3.synth.router_weights(g, E, H)
    devs = [k3.DeviceExpert.from_host(e, dev) for e in uniq]
    W = torch.from_numpy(wb.view(np.int16)).to(dev).view(torch.bfloat16)
    layer = k3.MoeLayer([devs[i % distinct] for i in range(E)],
                        k3.DeviceExpert.from_host(shared, dev), W, None, H, I, K, device=dev)
    return layer, g


def _noalloc(k3, fn, layer, x):
    import torch
    ntok = x.shape[0]
    out = torch.empty((ntok, layer.c.hidden), dtype=torch.float32, device=x.device)
    idx = torch.empty((ntok, layer.c.topk), dtype=torch.int32, device=x.device)
    wt = torch.empty((ntok, layer.c.topk), dtype=torch.float32, device=x.device)
    rc = fn(C.c_void_p(out.data_ptr()), C.c_void_p(x.data_ptr()), k3.K3C_BF16, ntok,
            C.byref(layer.c), C.c_void_p(idx.data_ptr()), C.c_void_p(wt.data_ptr()), None,
            C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, k3.lib().k3c_last_error()
    torch.cuda.synchronize()
    return out, idx, wt


@pytest.mark.parametrize("H,I,E,K,distinct,ntok", [(1024, 512, 32, 4, 32, 6),
                                                   (7168, 2048, 384, 8, 16, 16)])
def test_noalloc_matches_moe_decode_on_two_calls(k3, H, I, E, K, distinct, ntok):
    import torch
    dev = torch.device("cuda:0")
    L, fn = _bind(k3)
    layer, g = _layer(k3, dev, H, I, E, K, distinct, seed=H + ntok)
    assert layer.scratch_bytes(ntok) <= 8 << 20
    for call in range(2):                 # two calls in a row, different tokens each time
        _, xb = k3.synth.activations(g, ntok, H)
        x = torch.from_numpy(xb.view(np.int16)).to(dev).view(torch.bfloat16)
        ref_out, ref_idx, ref_wt = layer.decode(x)        # existing entry point
        torch.cuda.synchronize()
        out, idx, wt = _noalloc(k3, fn, layer, x)
        assert torch.equal(idx, ref_idx), call
        assert maxrel(wt.cpu().numpy(), ref_wt.cpu().numpy()) < TOL_F32, call
        assert maxrel(out.cpu().numpy(), ref_out.cpu().numpy()) < TOL_F32, call


def test_noalloc_rejects_a_batch_beyond_the_static_maximum(k3):
    import torch
    dev = torch.device("cuda:0")
    L, fn = _bind(k3)
    layer, g = _layer(k3, dev, 7168, 2048, 384, 8, 4, seed=5)
    ntok = 64                             # ~23 MB of scratch, beyond the 8 MiB array
    assert layer.scratch_bytes(ntok) > 8 << 20
    x = torch.zeros((ntok, 7168), dtype=torch.bfloat16, device=dev)
    out = torch.full((ntok, 7168), 7.0, dtype=torch.float32, device=dev)
    rc = fn(C.c_void_p(out.data_ptr()), C.c_void_p(x.data_ptr()), k3.K3C_BF16, ntok,
            C.byref(layer.c), None, None, None, C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == K3C_EINVAL
    assert b"static maximum" in L.k3c_last_error()
    torch.cuda.synchronize()
    assert bool((out == 7.0).all())       # nothing was launched, the output is untouched
