"""k3b200 -- B200-native routed-expert hot path of the kimi-k3 engine.

The product is ``libk3cuda.so`` (sources in ``csrc/``, C ABI in ``include/k3c.h``). This
module is the thin Python host side over that ABI: it binds the ``k3c_*`` device entry
points with ctypes and uses torch only for device memory and the current CUDA stream.
There is no CPU fallback: every call goes through the CUDA library, and importing the
binding fails loudly when the library is missing.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import ep, synth  # noqa: F401

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libk3cuda.so")

K3C_F32, K3C_BF16 = 0, 1
ACT_SWIGLU, ACT_SITU = 0, 1


class K3ExpertQ(C.Structure):
    """Mirror of the reference's K3ExpertQ (include/k3/k3.h:323-327): gate, up, down as
    (packed, scale) pointer pairs, here device addresses."""

    _fields_ = [(n, C.c_void_p) for n in ("p1", "s1", "p3", "s3", "p2", "s2")]


class MoeLayerC(C.Structure):
    """Mirror of k3c_moe_layer (include/k3c.h)."""

    _fields_ = [("hidden", C.c_int), ("inter", C.c_int), ("n_experts", C.c_int),
                ("topk", C.c_int), ("renorm", C.c_int), ("act", C.c_int),
                ("routed_scale", C.c_float), ("router_w", C.c_void_p),
                ("router_dtype", C.c_int), ("router_bias", C.c_void_p),
                ("experts", C.c_void_p), ("shared", C.c_void_p)]


class MoePoolLayerC(C.Structure):
    """Mirror of k3c_moe_pool_layer (include/k3c.h)."""

    _fields_ = [("hidden", C.c_int), ("inter", C.c_int), ("n_experts", C.c_int),
                ("topk", C.c_int), ("renorm", C.c_int), ("act", C.c_int),
                ("routed_scale", C.c_float), ("router_w", C.c_void_p),
                ("router_dtype", C.c_int), ("router_bias", C.c_void_p),
                ("arena", C.c_void_p), ("run_stride", C.c_size_t), ("n_runs", C.c_int),
                ("run_of", C.c_void_p), ("shared_run", C.c_int), ("terms", C.c_int)]


class Q8MatC(C.Structure):
    """Mirror of k3c_q8_mat (include/k3c.h): a packed int8 trunk matrix on the device."""

    _fields_ = [("wq", C.c_void_p), ("wscale", C.c_void_p), ("ldw", C.c_int)]


class MoeLatentLayerC(C.Structure):
    """Mirror of k3c_moe_latent_layer (include/k3c.h)."""

    _fields_ = ([("hidden", C.c_int), ("experts", MoePoolLayerC)]
                + [(n, C.c_void_p) for n in ("router_w", "router_bias", "down", "up", "sh1", "sh3",
                                             "sh2", "latent_norm")]
                + [(n, C.c_int) for n in ("wdt", "n_shared", "latent_norm_on")]
                + [(n, C.c_float) for n in ("rms_eps", "situ_b1", "situ_b2")]
                + [("cache_only", C.c_int)])


class TensorC(C.Structure):
    """Mirror of k3c_tensor (include/k3c.h)."""

    _fields_ = [("shard", C.c_int), ("dtype", C.c_int), ("ndim", C.c_int), ("off", C.c_int64),
                ("nbytes", C.c_int64), ("shape", C.c_int64 * 4)]


class QMatC(C.Structure):
    """Mirror of k3c_qmat (the reference's K3QMat)."""

    _fields_ = [("p_off", C.c_int64), ("p_bytes", C.c_int64), ("s_off", C.c_int64),
                ("s_bytes", C.c_int64), ("rows", C.c_int), ("pcols", C.c_int), ("scols", C.c_int)]


class ExpertRunC(C.Structure):
    """Mirror of k3c_expert_run (the reference's K3ExpertRef)."""

    _fields_ = [("layer", C.c_int), ("expert", C.c_int), ("shard", C.c_int), ("off", C.c_int64),
                ("nbytes", C.c_int64), ("contiguous", C.c_int), ("m", QMatC * 3)]


EP_MAX = 8


class IpcHandleC(C.Structure):
    """Mirror of k3c_ipc_handle (include/k3c.h)."""

    _fields_ = [("bytes", C.c_ubyte * 64)]


class EpPeersC(C.Structure):
    """Mirror of k3c_ep_peers (include/k3c.h)."""

    _fields_ = [("world", C.c_int), ("rank", C.c_int), ("t_max", C.c_int), ("x_dtype", C.c_int),
                ("ntok", C.c_int * EP_MAX), ("x", C.c_void_p * EP_MAX), ("idx", C.c_void_p * EP_MAX),
                ("wt", C.c_void_p * EP_MAX), ("recv", C.c_void_p * EP_MAX), ("local_only", C.c_void_p),
                ("x_ready", C.c_void_p)]


class K3CError(RuntimeError):
    pass


class K3CfgC(C.Structure):
    """Mirror of the reference's K3Cfg (include/k3/k3.h:73-116; include/k3c.h)."""

    _fields_ = ([(n, C.c_int) for n in ("hidden", "n_layers", "vocab")] + [("rms_eps", C.c_float)]
                + [(n, C.c_int) for n in ("kda_heads", "kda_head_dim", "conv_k")] + [("gate_lb", C.c_float)]
                + [(n, C.c_int) for n in ("n_heads", "q_lora", "kv_lora", "qk_nope", "qk_rope", "v_head",
                                          "mla_out_gate", "n_experts", "topk", "n_shared", "latent",
                                          "moe_inter")]
                + [("routed_scale", C.c_float)]
                + [(n, C.c_int) for n in ("moe_renorm", "latent_norm", "first_dense", "dense_inter",
                                          "attn_res_block")]
                + [("situ_b1", C.c_float), ("situ_b2", C.c_float), ("n_full_attn", C.c_int),
                   ("full_attn", C.POINTER(C.c_int))])


class K3ExpertSrcC(C.Structure):
    """Mirror of the reference's K3ExpertSrc vtable (include/k3/k3.h:332-355)."""


SRC_GET_FN = C.CFUNCTYPE(C.c_int, C.POINTER(K3ExpertSrcC), C.c_int, C.c_int, C.POINTER(K3ExpertQ))
SRC_GETMANY_FN = C.CFUNCTYPE(C.c_int, C.POINTER(K3ExpertSrcC), C.c_int, C.POINTER(C.c_int), C.c_int)
K3ExpertSrcC._fields_ = [("get", SRC_GET_FN), ("getmany", SRC_GETMANY_FN), ("resident", SRC_GET_FN),
                         ("ctx", C.c_void_p)]


class K3MoeWC(C.Structure):
    """Mirror of the reference's K3MoeW (include/k3/k3.h:357-380; include/k3c.h): host addresses."""

    _fields_ = ([(n, C.c_void_p) for n in ("gate", "bias", "w1", "w3", "w2", "latent_norm", "down", "up",
                                           "sh1", "sh3", "sh2")]
                + [("wdt", C.c_int), ("src", C.POINTER(K3ExpertSrcC)), ("layer", C.c_int),
                   ("cache_only", C.c_int)])


_lib = None


# host bytes of (layer, expert): a pointer to its pool-format run in pinned memory, or NULL
POOL_SRC_FN = C.CFUNCTYPE(C.c_void_p, C.c_void_p, C.c_int, C.c_int)


class PoolStatsC(C.Structure):
    _fields_ = [("hits", C.c_longlong), ("misses", C.c_longlong), ("evictions", C.c_longlong),
                ("prefetch_reads", C.c_longlong), ("bytes_h2d", C.c_longlong)]


def lib():
    """Load libk3cuda.so (building it with make if this checkout has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        import subprocess
        subprocess.run(["make", "-s", "-C", os.path.join(HERE, "csrc")], check=True)
    L = C.CDLL(LIB_PATH)
    vp, i, f, sz = C.c_void_p, C.c_int, C.c_float, C.c_size_t
    sig = {
        "k3c_last_error": ([], C.c_char_p),
        "k3c_version": ([], C.c_char_p),
        "k3c_launch_count": ([], C.c_longlong),
        "k3c_timing_enable": ([i], None),
        "k3c_timing_read": ([C.POINTER(C.c_double), C.POINTER(C.c_longlong), i], i),
        "k3c_mxfp4_dequant": ([vp, vp, vp, i, i, i, vp], i),
        "k3c_mxfp4_gemv": ([vp, i, vp, i, i, vp, vp, i, i, i, vp], i),
        "k3c_q8_pack": ([vp, vp, i, vp, i, i, vp], i),
        "k3c_q8_gemv": ([vp, i, vp, i, i, i, vp, vp, i, i, i, vp], i),
        "k3c_q8_gemv_scratch": ([i, i, i], sz),
        "k3c_mmw_tc_scratch": ([i, i], sz),
        "k3c_mmw_tc": ([vp, i, vp, i, i, vp, i, i, i, vp, sz, vp], i),
        "k3c_q8_gemv_ws": ([vp, i, vp, i, i, i, vp, vp, i, i, i, vp, sz, vp], i),
        "k3c_router": ([vp, vp, vp, vp, i, vp, i, vp, i, i, i, i, f, i, vp], i),
        "k3c_router_select": ([vp, vp, vp, vp, i, i, i, f, i, vp], i),
        "k3c_expert_ffn_scratch": ([i, i, i], sz),
        "k3c_expert_ffn": ([vp, vp, i, C.POINTER(K3ExpertQ), i, i, i, vp, sz, vp], i),
        "k3c_moe_decode_scratch": ([C.POINTER(MoeLayerC), i], sz),
        "k3c_moe_decode": ([vp, vp, i, i, C.POINTER(MoeLayerC), vp, vp, vp, vp, sz, vp], i),
        "k3c_pool_run_bytes": ([i, i], sz),
        "k3c_pool_pack_expert": ([vp, C.POINTER(K3ExpertQ), i, i, vp], i),
        "k3c_moe_decode_tc_scratch": ([C.POINTER(MoePoolLayerC), i], sz),
        "k3c_moe_decode_tc": ([vp, vp, i, i, C.POINTER(MoePoolLayerC), vp, vp, vp, vp, sz, vp], i),
        "k3c_moe_decode_tc_routed": ([vp, vp, i, i, C.POINTER(MoePoolLayerC), vp, vp, vp, vp, sz, vp], i),
        "k3c_pool_create": ([i, i, i, i, i, POOL_SRC_FN, vp], vp),
        "k3c_pool_destroy": ([vp], None),
        "k3c_pool_arena": ([vp], vp),
        "k3c_pool_slot_stride": ([vp], sz),
        "k3c_pool_slots": ([vp], i),
        "k3c_pool_resident": ([vp, i, i], i),
        "k3c_pool_getmany": ([vp, i, vp, i], i),
        "k3c_pool_acquire": ([vp, i, vp, i, vp, vp, vp], i),
        "k3c_pool_release": ([vp, i, vp, i, vp], i),
        "k3c_pool_pin": ([vp, i, i, vp], i),
        "k3c_pool_stats": ([vp, C.POINTER(PoolStatsC)], i),
        "k3c_pool_sync": ([vp], i),
        "k3c_moe_prefill_tc_scratch": ([C.POINTER(MoePoolLayerC), i], sz),
        "k3c_moe_prefill_tc_routed": ([vp, vp, i, i, C.POINTER(MoePoolLayerC), vp, vp, vp, vp, sz, vp], i),
        "k3c_moe_prefill_tc": ([vp, vp, i, i, C.POINTER(MoePoolLayerC), vp, vp, vp, vp, sz, vp], i),
        "k3c_moe_combine": ([vp, vp, vp, vp, i, i, i, i, i, vp], i),
        "k3c_router_scratch": ([i, i, i], sz),
        "k3c_router_ws": ([vp, vp, vp, vp, i, vp, i, vp, i, i, i, i, f, i, vp, sz, vp], i),
        "k3c_ep_alloc": ([C.POINTER(vp), sz, C.POINTER(IpcHandleC)], i),
        "k3c_ep_free": ([vp], i),
        "k3c_ep_open": ([C.POINTER(vp), C.POINTER(IpcHandleC)], i),
        "k3c_ep_close": ([vp], i),
        "k3c_moe_prefill_ep_scratch": ([C.POINTER(MoePoolLayerC), C.POINTER(EpPeersC)], sz),
        "k3c_moe_prefill_ep_experts": ([C.POINTER(MoePoolLayerC), C.POINTER(EpPeersC), vp, sz, vp], i),
        "k3c_moe_ep_combine": ([vp, C.POINTER(EpPeersC), i, i, vp, i, i, vp], i),
        "k3_mxfp4_dequant": ([vp, vp, vp, i, i, i], None),
        "k3_matmul_mxfp4": ([vp, vp, vp, vp, i, i, i], None),
        "k3_matmul_q8": ([vp, vp, vp, i, i], None),
        "k3_router": ([vp, vp, vp, vp, vp, i, i, i, i, f], None),
        "k3_matmul": ([vp, vp, vp, i, i], None),
        "k3_matmul_bf16": ([vp, vp, vp, i, i], None),
        "k3c_mmw": ([vp, i, vp, i, i, vp, i, i, i, i, vp], i),
        "k3c_situ_glu": ([vp, vp, i, i, f, f, vp], i),
        "k3c_rmsnorm": ([vp, vp, vp, i, i, f, vp], i),
        "k3c_moe_latent_scratch": ([C.POINTER(MoeLatentLayerC), i], sz),
        "k3c_route_cache_only": ([vp, vp, i, i, vp, i, i, vp], i),
        "k3c_moe_latent_decode_routed": ([vp, vp, i, C.POINTER(MoeLatentLayerC), vp, vp, vp, vp, sz, vp], i),
        "k3c_pool_acquire_resident": ([vp, i, vp, i, vp, vp], i),
        "k3c_pool_trace": ([vp, vp, C.c_int64], C.c_int64),
        "k3c_pool_hist": ([vp, vp], i),
        "k3c_pool_dump_trace": ([vp, C.c_char_p], i),
        "k3c_pool_dump_hist": ([vp, C.c_char_p], i),
        "k3c_pool_set_pin": ([vp, i, i, i], i),
        "k3c_pool_reset_stats": ([vp], None),
        "k3c_pool_report": ([vp, C.c_char_p], None),
        "k3c_pool_source_create": ([vp, vp], vp),
        "k3c_pool_source_destroy": ([vp], None),
        "k3c_pool_source_release": ([vp], i),
        "k3c_pool_source_stream": ([vp], vp),
        "k3c_pool_source_pool": ([vp], vp),
        "k3c_pool_source_slot": ([vp, C.POINTER(K3ExpertQ)], i),
        "k3c_pool_shape": ([vp, C.POINTER(i), C.POINTER(i)], i),
        "k3_moe": ([vp, vp, C.POINTER(K3MoeWC), C.POINTER(K3CfgC), i, vp, vp, vp], None),
        "k3_moe_prefill": ([vp, vp, C.POINTER(K3MoeWC), C.POINTER(K3CfgC), i, vp, vp, vp], None),
        "k3_moe_scratch": ([C.POINTER(K3CfgC)], sz),
        "k3c_dropin_keep_weights": ([i], None),
        "k3c_dropin_forget_weights": ([], None),
        "k3c_selftest_wait": ([i, C.c_double, vp], i),
        "k3c_trunk_open": ([C.c_char_p], vp),
        "k3c_trunk_close": ([vp], None),
        "k3c_trunk_layers": ([vp], i),
        "k3c_trunk_find": ([vp, i, C.c_char_p, C.POINTER(TensorC)], i),
        "k3c_trunk_read": ([vp, C.POINTER(TensorC), vp, C.c_int64, C.POINTER(C.c_int64)], C.c_int64),
        "k3c_ckpt_open": ([C.c_char_p], vp),
        "k3c_ckpt_close": ([vp], None),
        "k3c_ckpt_shards": ([vp], i),
        "k3c_ckpt_direct": ([vp, i], i),
        "k3c_ckpt_find": ([vp, C.c_char_p, C.POINTER(TensorC)], i),
        "k3c_expert_ref": ([vp, i, i, C.POINTER(ExpertRunC)], i),
        "k3c_expert_read": ([vp, C.POINTER(ExpertRunC), vp, C.c_int64, C.POINTER(C.c_int64)], C.c_int64),
        "k3c_expert_upload": ([vp, C.POINTER(ExpertRunC), vp, vp, vp], i),
        "k3c_moe_latent_decode": ([vp, vp, i, C.POINTER(MoeLatentLayerC), vp, vp, vp, vp, sz, vp], i),
    }
    for name, (args, res) in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res
    _lib = L
    return L


def _check(rc: int, what: str):
    if rc != 0:
        raise K3CError(f"{what} failed ({rc}): {lib().k3c_last_error().decode()}")


def _stream():
    import torch
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _dtype_code(t):
    import torch
    if t.dtype == torch.float32:
        return K3C_F32
    if t.dtype in (torch.bfloat16, torch.int16, torch.uint16):
        return K3C_BF16
    raise K3CError(f"unsupported activation dtype {t.dtype}")


# ------------------------------------------------------------------ kernel wrappers


def mxfp4_dequant(packed, scales, group=32):
    import torch
    rows, pcols = packed.shape
    out = torch.empty((rows, 2 * pcols), dtype=torch.float32, device=packed.device)
    _check(lib().k3c_mxfp4_dequant(_ptr(out), _ptr(packed), _ptr(scales), rows, pcols, group,
                                   _stream()), "k3c_mxfp4_dequant")
    return out


def mxfp4_gemv(x, packed, scales, group=32):
    """y[t][r] = sum_k W[r][k] x[t][k]; x fp32 [ntok][in] on the device."""
    import torch
    x = x.contiguous()
    if x.dim() == 1:
        x = x.unsqueeze(0)
    ntok, in_ = x.shape
    rows = packed.shape[0]
    y = torch.empty((ntok, rows), dtype=torch.float32, device=x.device)
    _check(lib().k3c_mxfp4_gemv(_ptr(y), rows, _ptr(x), in_, ntok, _ptr(packed), _ptr(scales),
                                in_, rows, group, _stream()), "k3c_mxfp4_gemv")
    return y


def q8_pack(rows_u8, in_, out):
    """Reference row layout ([f32 scale][int8*in] per row, on the device) -> pool layout."""
    import torch
    ldw = (in_ + 31) // 32 * 32
    wq = torch.empty((out, ldw), dtype=torch.int8, device=rows_u8.device)
    ws = torch.empty(out, dtype=torch.float32, device=rows_u8.device)
    _check(lib().k3c_q8_pack(_ptr(wq), _ptr(ws), ldw, _ptr(rows_u8), in_, out, _stream()),
           "k3c_q8_pack")
    return wq, ws, ldw


def q8_gemv(x, wq, ws, ldw, in_, out, scratch=None):
    """scratch: a uint8 device tensor of at least q8_gemv_scratch(ntok, in_, out) bytes
    (k3c_q8_gemv_ws), or None for a per-call stream-ordered allocation (k3c_q8_gemv)."""
    import torch
    if x.dim() == 1:
        x = x.unsqueeze(0)
    x = x.contiguous()
    ntok = x.shape[0]
    y = torch.empty((ntok, out), dtype=torch.float32, device=x.device)
    if scratch is None:
        _check(lib().k3c_q8_gemv(_ptr(y), out, _ptr(x), _dtype_code(x), x.shape[1], ntok, _ptr(wq),
                                 _ptr(ws), ldw, in_, out, _stream()), "k3c_q8_gemv")
    else:
        _check(lib().k3c_q8_gemv_ws(_ptr(y), out, _ptr(x), _dtype_code(x), x.shape[1], ntok, _ptr(wq), _ptr(ws),
                                    ldw, in_, out, _ptr(scratch), scratch.numel() * scratch.element_size(),
                                    _stream()), "k3c_q8_gemv_ws")
    return y


def q8_gemv_scratch(ntok, in_, out):
    return int(lib().k3c_q8_gemv_scratch(ntok, in_, out))


def router(x, W, bias, topk, renorm=1, routed_scale=1.0):
    """Returns (idx [ntok][topk] int32, w [ntok][topk] fp32, scores [ntok][E] fp32)."""
    import torch
    if x.dim() == 1:
        x = x.unsqueeze(0)
    x = x.contiguous()
    ntok, H = x.shape
    E = W.shape[0]
    idx = torch.empty((ntok, topk), dtype=torch.int32, device=x.device)
    w = torch.empty((ntok, topk), dtype=torch.float32, device=x.device)
    sc = torch.empty((ntok, E), dtype=torch.float32, device=x.device)
    _check(lib().k3c_router(_ptr(idx), _ptr(w), _ptr(sc), _ptr(x), _dtype_code(x), _ptr(W),
                            _dtype_code(W), _ptr(bias), H, E, topk, renorm, routed_scale, ntok,
                            _stream()), "k3c_router")
    return idx, w, sc


def route_cache_only(idx, wt, run_of, n_runs):
    """k3c_route_cache_only in place on device idx/wt [ntok][topk] (the draft model's routing
    among resident experts); run_of: device int32 [n_experts], an expert is resident when
    0 <= run_of[e] < n_runs."""
    ntok, topk = idx.shape
    _check(lib().k3c_route_cache_only(_ptr(idx), _ptr(wt), ntok, topk, _ptr(run_of), run_of.numel(),
                                      int(n_runs), _stream()), "k3c_route_cache_only")
    return idx, wt


def router_select(scores, bias, topk, renorm=1, routed_scale=1.0):
    import torch
    ntok, E = scores.shape
    idx = torch.empty((ntok, topk), dtype=torch.int32, device=scores.device)
    w = torch.empty((ntok, topk), dtype=torch.float32, device=scores.device)
    _check(lib().k3c_router_select(_ptr(idx), _ptr(w), _ptr(scores.contiguous()), _ptr(bias), E,
                                   topk, renorm, routed_scale, ntok, _stream()),
           "k3c_router_select")
    return idx, w


class DeviceExpert:
    """One MXFP4 expert resident in device memory (reference layout per matrix)."""

    KEYS = ("gate_p", "gate_s", "up_p", "up_s", "down_p", "down_s")

    def __init__(self, tensors: dict):
        self.t = tensors

    @classmethod
    def from_host(cls, e: dict, device):
        import torch
        return cls({k: torch.from_numpy(np.ascontiguousarray(e[k])).to(device) for k in cls.KEYS})

    def q(self) -> K3ExpertQ:
        t = self.t
        return K3ExpertQ(t["gate_p"].data_ptr(), t["gate_s"].data_ptr(), t["up_p"].data_ptr(),
                         t["up_s"].data_ptr(), t["down_p"].data_ptr(), t["down_s"].data_ptr())


def expert_run_layout(hidden, inter):
    """Byte offsets of one expert's contiguous run, in the reference checkpoint's order
    w1.p w1.s w2.p w2.s w3.p w3.s (src/io/k3_load.c:82-105; w1 gate, w2 down, w3 up).
    Returns (dict name -> (offset, nbytes), total bytes)."""
    parts = [("gate_p", inter * hidden // 2), ("gate_s", inter * hidden // 32),
             ("down_p", hidden * inter // 2), ("down_s", hidden * inter // 32),
             ("up_p", inter * hidden // 2), ("up_s", inter * hidden // 32)]
    off, lay = 0, {}
    for name, nb in parts:
        lay[name] = (off, nb)
        off += nb
    return lay, off


def pool_layout(hidden, inter):
    """Byte offsets of the pool-format run read by the tensor-core path (csrc/moe_tc.cu):
    GU packed (gate/up rows interleaved per 64), GU scale atoms, D packed, D scale atoms.
    Returns (dict name -> (offset, nbytes), total bytes)."""
    H, I = hidden, inter
    parts = [("gu_p", I * H), ("gu_s", 2 * I * H // 32), ("d_p", H * I // 2),
             ("d_s", H * I // 32)]
    off, lay = 0, {}
    for name, nb in parts:
        lay[name] = (off, nb)
        off += nb
    return lay, off


def experts_from_blob(blob, n, hidden, inter, stride=None):
    """K3ExpertQ for n expert runs laid out back to back (every `stride` bytes) in one
    device uint8 tensor."""
    lay, total = expert_run_layout(hidden, inter)
    stride = stride or total
    base = blob.data_ptr()
    qs = []
    for i in range(n):
        b = base + i * stride
        qs.append(K3ExpertQ(b + lay["gate_p"][0], b + lay["gate_s"][0], b + lay["up_p"][0],
                            b + lay["up_s"][0], b + lay["down_p"][0], b + lay["down_s"][0]))
    return qs


def expert_table(qs, device):
    """Device array of K3ExpertQ built from a list of K3ExpertQ (None = not resident)."""
    import torch
    arr = np.zeros((len(qs), 6), np.uint64)
    for i, q in enumerate(qs):
        if q is not None:
            arr[i] = [q.p1 or 0, q.s1 or 0, q.p3 or 0, q.s3 or 0, q.p2 or 0, q.s2 or 0]
    return torch.from_numpy(arr.view(np.int64)).to(device)


def expert_ffn(x, expert: DeviceExpert, hidden, inter, act=ACT_SWIGLU):
    import torch
    if x.dim() == 1:
        x = x.unsqueeze(0)
    x = x.contiguous()
    ntok = x.shape[0]
    L = lib()
    nbytes = L.k3c_expert_ffn_scratch(ntok, hidden, inter)
    scratch = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
    y = torch.empty((ntok, hidden), dtype=torch.float32, device=x.device)
    q = expert.q()
    _check(L.k3c_expert_ffn(_ptr(y), _ptr(x), ntok, C.byref(q), hidden, inter, act,
                            _ptr(scratch), nbytes, _stream()), "k3c_expert_ffn")
    return y


class MoeLayer:
    """A non-latent MoE layer on the device: router (bf16 or fp32 W), routed MXFP4
    experts in an expert table, optional shared expert. decode() runs k3c_moe_decode."""

    def __init__(self, experts, shared, router_w, router_bias, hidden, inter, topk,
                 renorm=1, routed_scale=1.0, act=ACT_SWIGLU, device=None):
        """experts: list of DeviceExpert, K3ExpertQ (device addresses) or None (not
        resident); shared likewise or None."""
        import torch
        self.device = device
        self.experts = experts            # kept alive: the table holds their addresses
        self.shared = shared
        self.router_w = router_w
        self.router_bias = router_bias

        def q_of(e):
            return e.q() if isinstance(e, DeviceExpert) else e
        self.table = expert_table([q_of(e) for e in experts], device)
        self.shared_table = expert_table([q_of(shared)], device) if shared is not None else None
        self.c = MoeLayerC(hidden, inter, len(experts), topk, renorm, act, routed_scale,
                           router_w.data_ptr(), _dtype_code(router_w),
                           router_bias.data_ptr() if router_bias is not None else None,
                           self.table.data_ptr(),
                           self.shared_table.data_ptr() if shared is not None else None)
        self._scratch = torch.empty(0, dtype=torch.uint8, device=device)

    @classmethod
    def from_host(cls, experts, shared, router_w_bits, router_bias, hidden, inter, topk,
                  device, **kw):
        """experts/shared: host dicts of numpy arrays (synth.expert); router_w_bits: bf16 bits
        (uint16) or fp32 numpy array."""
        import torch
        dev = [DeviceExpert.from_host(e, device) for e in experts]
        sh = DeviceExpert.from_host(shared, device) if shared is not None else None
        if router_w_bits.dtype == np.uint16:
            W = torch.from_numpy(router_w_bits.view(np.int16)).to(device).view(torch.bfloat16)
        else:
            W = torch.from_numpy(np.ascontiguousarray(router_w_bits, np.float32)).to(device)
        b = None if router_bias is None else torch.from_numpy(
            np.ascontiguousarray(router_bias, np.float32)).to(device)
        return cls(dev, sh, W, b, hidden, inter, topk, device=device, **kw)

    def scratch_bytes(self, ntok):
        return lib().k3c_moe_decode_scratch(C.byref(self.c), ntok)

    def decode(self, x, out=None, idx=None, wt=None, drops=None):
        """x: [ntok][hidden] bf16 (or int16 bf16 bits) or fp32 device tensor."""
        import torch
        import torch as _t
        if x.dtype == _t.int16:
            x = x.view(_t.bfloat16)
        x = x.contiguous()
        ntok = x.shape[0]
        need = self.scratch_bytes(ntok)
        if self._scratch.numel() < need:
            self._scratch = torch.empty(need, dtype=torch.uint8, device=x.device)
        H, K = self.c.hidden, self.c.topk
        if out is None:
            out = torch.empty((ntok, H), dtype=torch.float32, device=x.device)
        if idx is None:
            idx = torch.empty((ntok, K), dtype=torch.int32, device=x.device)
        if wt is None:
            wt = torch.empty((ntok, K), dtype=torch.float32, device=x.device)
        _check(lib().k3c_moe_decode(_ptr(out), _ptr(x), _dtype_code(x), ntok, C.byref(self.c),
                                    _ptr(idx), _ptr(wt), _ptr(drops), _ptr(self._scratch),
                                    self._scratch.numel(), _stream()), "k3c_moe_decode")
        return out, idx, wt


def pool_run_bytes(hidden, inter):
    n = lib().k3c_pool_run_bytes(hidden, inter)
    if n == 0:
        raise K3CError(f"pool format needs hidden/inter multiples of 128 ({hidden}, {inter})")
    return n


def pool_pack(run, q: K3ExpertQ, hidden, inter):
    """Pack one expert (reference layout, device addresses) into a pool-format run (a
    device uint8 tensor view of pool_run_bytes bytes, 256-byte aligned)."""
    _check(lib().k3c_pool_pack_expert(_ptr(run), C.byref(q), hidden, inter, _stream()),
           "k3c_pool_pack_expert")


def device_view(ptr, shape, dtype):
    """A torch tensor over device memory this process did not allocate through torch (no
    copy; the memory must outlive the tensor). Only for local memory: a peer's memory is
    handed to this library's kernels by address, never to torch operations."""
    import torch
    nbytes = int(np.prod(shape)) * torch.empty(0, dtype=dtype).element_size()

    class _View:
        __cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (int(ptr), False),
                                    "version": 3}
    return torch.as_tensor(_View(), device="cuda").view(dtype).view(tuple(shape))


class PoolMoeLayer:
    """A non-latent MoE layer whose experts live in one HBM arena of pool-format runs and
    run on the tcgen05 block-scaled MMA path (k3c_moe_decode_tc)."""

    def __init__(self, arena, n_runs, run_of, shared_run, router_w, router_bias, hidden, inter,
                 topk, terms=3, renorm=1, routed_scale=1.0, act=ACT_SWIGLU):
        import torch
        self.arena = arena
        self.run_of = run_of
        self.router_w = router_w
        self.router_bias = router_bias
        self.stride = pool_run_bytes(hidden, inter)
        self.c = MoePoolLayerC(hidden, inter, run_of.numel(), topk, renorm, act, routed_scale,
                               router_w.data_ptr(), _dtype_code(router_w),
                               router_bias.data_ptr() if router_bias is not None else None,
                               arena.data_ptr(), self.stride, n_runs, run_of.data_ptr(),
                               shared_run, terms)
        self._scratch = torch.empty(0, dtype=torch.uint8, device=arena.device)

    @classmethod
    def pack(cls, experts, shared, router_w, router_bias, hidden, inter, topk, device,
             expert_map=None, **kw):
        """experts: list of K3ExpertQ / DeviceExpert (reference layout, distinct runs);
        expert_map: expert id -> index into `experts` (default identity); shared may be None."""
        import torch
        srcs = list(experts) + ([shared] if shared is not None else [])
        run = pool_run_bytes(hidden, inter)
        arena = torch.empty(len(srcs) * run, dtype=torch.uint8, device=device)
        for i, e in enumerate(srcs):
            q = e.q() if isinstance(e, DeviceExpert) else e
            pool_pack(arena[i * run:(i + 1) * run], q, hidden, inter)
        n_exp = len(expert_map) if expert_map is not None else len(experts)
        m = np.arange(n_exp) if expert_map is None else np.asarray(expert_map)
        run_of = torch.from_numpy(m.astype(np.int32)).to(device)
        shared_run = len(experts) if shared is not None else -1
        return cls(arena, len(srcs), run_of, shared_run, router_w, router_bias, hidden, inter,
                   topk, **kw)

    def scratch_bytes(self, ntok):
        return lib().k3c_moe_decode_tc_scratch(C.byref(self.c), ntok)

    def decode(self, x, out=None, idx=None, wt=None, drops=None):
        import torch
        if x.dtype == torch.int16:
            x = x.view(torch.bfloat16)
        x = x.contiguous()
        ntok = x.shape[0]
        need = self.scratch_bytes(ntok)
        if self._scratch.numel() < need:
            self._scratch = torch.empty(need, dtype=torch.uint8, device=x.device)
        H, K = self.c.hidden, self.c.topk
        if out is None:
            out = torch.empty((ntok, H), dtype=torch.float32, device=x.device)
        if idx is None:
            idx = torch.empty((ntok, K), dtype=torch.int32, device=x.device)
        if wt is None:
            wt = torch.empty((ntok, K), dtype=torch.float32, device=x.device)
        _check(lib().k3c_moe_decode_tc(_ptr(out), _ptr(x), _dtype_code(x), ntok,
                                       C.byref(self.c), _ptr(idx), _ptr(wt), _ptr(drops),
                                       _ptr(self._scratch), self._scratch.numel(), _stream()),
               "k3c_moe_decode_tc")
        return out, idx, wt

    def decode_routed(self, x, idx, wt, out=None, drops=None):
        """decode with the routing given (idx/wt [ntok][topk] on the device); the router is
        not run (k3c_moe_decode_tc_routed)."""
        import torch
        if x.dtype == torch.int16:
            x = x.view(torch.bfloat16)
        x = x.contiguous()
        ntok = x.shape[0]
        need = self.scratch_bytes(ntok)
        if self._scratch.numel() < need:
            self._scratch = torch.empty(need, dtype=torch.uint8, device=x.device)
        if out is None:
            out = torch.empty((ntok, self.c.hidden), dtype=torch.float32, device=x.device)
        _check(lib().k3c_moe_decode_tc_routed(_ptr(out), _ptr(x), _dtype_code(x), ntok,
                                              C.byref(self.c), _ptr(idx), _ptr(wt), _ptr(drops),
                                              _ptr(self._scratch), self._scratch.numel(), _stream()),
               "k3c_moe_decode_tc_routed")
        return out

    def prefill_routed(self, x, idx, wt, out=None, drops=None):
        """prefill with the routing given (k3c_moe_prefill_tc_routed); ids < 0 are skipped."""
        import torch
        if x.dtype == torch.int16:
            x = x.view(torch.bfloat16)
        x = x.contiguous()
        ntok = x.shape[0]
        need = lib().k3c_moe_prefill_tc_scratch(C.byref(self.c), max(ntok, 1))
        if self._scratch.numel() < need:
            self._scratch = torch.empty(need, dtype=torch.uint8, device=x.device)
        if out is None:
            out = torch.empty((ntok, self.c.hidden), dtype=torch.float32, device=x.device)
        if ntok == 0:
            return out
        _check(lib().k3c_moe_prefill_tc_routed(_ptr(out), _ptr(x), _dtype_code(x), ntok,
                                               C.byref(self.c), _ptr(idx), _ptr(wt), _ptr(drops),
                                               _ptr(self._scratch), self._scratch.numel(), _stream()),
               "k3c_moe_prefill_tc_routed")
        return out

    def prefill(self, x, out=None, idx=None, wt=None, drops=None):
        """Prefill over ntok tokens (k3c_moe_prefill_tc): expert-sorted tokens through the
        tcgen05 grouped expert kernels, combined in each token's top-k order."""
        import torch
        if x.dtype == torch.int16:
            x = x.view(torch.bfloat16)
        x = x.contiguous()
        ntok = x.shape[0]
        need = lib().k3c_moe_prefill_tc_scratch(C.byref(self.c), ntok)
        if self._scratch.numel() < need:
            self._scratch = torch.empty(need, dtype=torch.uint8, device=x.device)
        H, K = self.c.hidden, self.c.topk
        if out is None:
            out = torch.empty((ntok, H), dtype=torch.float32, device=x.device)
        if idx is None:
            idx = torch.empty((ntok, K), dtype=torch.int32, device=x.device)
        if wt is None:
            wt = torch.empty((ntok, K), dtype=torch.float32, device=x.device)
        _check(lib().k3c_moe_prefill_tc(_ptr(out), _ptr(x), _dtype_code(x), ntok,
                                        C.byref(self.c), _ptr(idx), _ptr(wt), _ptr(drops),
                                        _ptr(self._scratch), self._scratch.numel(), _stream()),
               "k3c_moe_prefill_tc")
        return out, idx, wt


class ExpertPool:
    """HBM expert pool (k3c_pool_*): the reference's expert cache with experts copied from
    pinned host memory. host_src(layer, expert) returns the pinned host uint8 tensor holding
    that expert's pool-format run (pool_run_bytes bytes), or None."""

    def __init__(self, hidden, inter, n_layers, n_experts, n_slots, host_src):
        self.hidden, self.inter, self.n_layers, self.n_experts = hidden, inter, n_layers, n_experts
        self._host_src = host_src

        def cb(ctx, layer, expert):
            t = self._host_src(layer, expert)
            return None if t is None else t.data_ptr()

        self._cb = POOL_SRC_FN(cb)          # kept alive as long as the pool
        self.p = lib().k3c_pool_create(hidden, inter, n_layers, n_experts, n_slots, self._cb, None)
        if not self.p:
            raise RuntimeError(f"k3c_pool_create: {lib().k3c_last_error().decode()}")
        self.n_slots = n_slots
        self.stride = lib().k3c_pool_slot_stride(self.p)
        self.arena_ptr = lib().k3c_pool_arena(self.p)

    def close(self):
        if self.p:
            lib().k3c_pool_destroy(self.p)
            self.p = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @staticmethod
    def _ids(ids):
        a = np.ascontiguousarray(np.asarray(ids, dtype=np.int32))
        return a, a.ctypes.data

    def getmany(self, layer, ids):
        a, p = self._ids(ids)
        rc = lib().k3c_pool_getmany(self.p, layer, p, len(a))
        if rc < 0:
            _check(rc, "k3c_pool_getmany")
        return rc

    def acquire(self, layer, ids, run_of=None):
        """Returns the slots (numpy); fills the device run table run_of if given."""
        a, p = self._ids(ids)
        slots = np.empty(len(a), np.int32)
        _check(lib().k3c_pool_acquire(self.p, layer, p, len(a), slots.ctypes.data, _ptr(run_of),
                                      _stream()), "k3c_pool_acquire")
        return slots

    def release(self, layer, ids):
        a, p = self._ids(ids)
        _check(lib().k3c_pool_release(self.p, layer, p, len(a), _stream()), "k3c_pool_release")

    def pin(self, layer, expert):
        rc = lib().k3c_pool_pin(self.p, layer, expert, _stream())
        if rc < 0:
            _check(rc, "k3c_pool_pin")
        return rc

    def resident(self, layer, expert):
        return lib().k3c_pool_resident(self.p, layer, expert)

    def stats(self):
        st = PoolStatsC()
        _check(lib().k3c_pool_stats(self.p, C.byref(st)), "k3c_pool_stats")
        d = {k: getattr(st, k) for k, _ in PoolStatsC._fields_}
        n = d["hits"] + d["misses"]
        d["hit_rate"] = d["hits"] / n if n else None
        d["true_hit_rate"] = max(d["hits"] - d["prefetch_reads"], 0) / n if n else None
        return d

    def sync(self):
        _check(lib().k3c_pool_sync(self.p), "k3c_pool_sync")

    def run_table(self):
        """A device run table for k3c_pool_acquire: int32 [n_experts of the pool], -1."""
        import torch
        return torch.full((self.n_experts,), -1, dtype=torch.int32, device="cuda")

    def slot_tensor(self, slot):
        """uint8 device view of one slot's bytes (no copy)."""
        import torch

        class _View:
            __cuda_array_interface__ = {"shape": (self.stride,), "typestr": "|u1",
                                        "data": (self.arena_ptr + int(slot) * self.stride, False),
                                        "version": 3}
        return torch.as_tensor(_View(), device="cuda")

    def layer(self, router_w, hidden, inter, topk, routed_experts, run_table, shared_slot=-1, **kw):
        """A PoolMoeLayer over this pool's slots for a layer routed over the first
        routed_experts ids of run_table (the table k3c_pool_acquire fills)."""
        return PoolMoeLayer(_PoolArena(self), self.n_slots, run_table[:routed_experts], shared_slot,
                            router_w, None, hidden, inter, topk, **kw)


class _PoolArena:
    """Adapter giving PoolMoeLayer the pool's arena pointer and device."""

    def __init__(self, pool):
        import torch
        self.pool = pool
        self.device = torch.device("cuda", torch.cuda.current_device())

    def data_ptr(self):
        return self.pool.arena_ptr


# ------------------------------------------------------------------ K3 latent MoE layer
WF32, WBF16, WI8 = 0, 1, 2


def mmw(x, W, wdt, out=None, accumulate=False):
    """k3c_mmw: y[t] = W x[t] for x [ntok][in] fp32 (ntok <= 32) and W [out][in] fp32
    (wdt=WF32) or bf16 bit patterns (WBF16, a torch int16/uint16/bfloat16 tensor), in the
    reference's k3_matmul summation order (bit-exact). accumulate adds into `out`."""
    import torch
    x = x.contiguous()
    ntok, in_ = x.shape
    out_ = W.shape[0]
    if out is None:
        out = torch.zeros((ntok, out_), dtype=torch.float32, device=x.device)
    _check(lib().k3c_mmw(_ptr(out), out.stride(0), _ptr(x), in_, ntok, _ptr(W), wdt, in_, out_,
                         1 if accumulate else 0, _stream()), "k3c_mmw")
    return out


def mmw_tc(x, W, out=None, accumulate=False, ldx=None):
    """k3c_mmw_tc: y[t] = W x[t] on the tensor cores for any number of tokens, W [out][in] bf16
    bit patterns (16-byte aligned, in a multiple of 8), x [ntok][>= in] fp32 (the first `in`
    columns; ldx its row stride). Two bf16 terms of x, fp32 accumulation: not bit-exact."""
    import torch
    ntok = x.shape[0]
    out_, in_ = W.shape
    ldx = x.stride(0) if ldx is None else ldx
    if out is None:
        out = torch.zeros((ntok, out_), dtype=torch.float32, device=x.device)
    n = int(lib().k3c_mmw_tc_scratch(ntok, in_))
    ws = torch.empty(max(n, 1), dtype=torch.uint8, device=x.device)
    _check(lib().k3c_mmw_tc(_ptr(out), out.stride(0), _ptr(x), ldx, ntok, _ptr(W), in_, out_,
                            1 if accumulate else 0, _ptr(ws), n, _stream()), "k3c_mmw_tc")
    return out


def rmsnorm(x, w, eps=1e-5, out=None):
    """k3c_rmsnorm over the rows of x [ntok][n] fp32."""
    import torch
    x = x.contiguous()
    if out is None:
        out = torch.empty_like(x)
    _check(lib().k3c_rmsnorm(_ptr(out), _ptr(x), _ptr(w), x.shape[1], x.shape[0], eps, _stream()),
           "k3c_rmsnorm")
    return out


def situ_glu(gu, b1=4.0, b2=25.0):
    """k3c_situ_glu: gu [ntok][2n] (gate | up) -> [ntok][n]."""
    import torch
    gu = gu.contiguous()
    n = gu.shape[1] // 2
    out = torch.empty((gu.shape[0], n), dtype=torch.float32, device=gu.device)
    _check(lib().k3c_situ_glu(_ptr(out), _ptr(gu), n, gu.shape[0], b1, b2, _stream()), "k3c_situ_glu")
    return out


class LatentMoeLayer:
    """The K3 latent MoE layer (k3c_moe_latent_decode): full-width routing, trunk down/up and
    shared-expert matrices (fp32 or bf16), routed MXFP4 experts at the latent width in an HBM
    arena of pool-format runs on the tensor-core path."""

    def __init__(self, arena, n_runs, run_of, router_w, router_bias, down, up, sh1, sh3, sh2,
                 latent_norm, wdt, hidden, latent, inter, n_shared, topk, terms=3, renorm=1,
                 routed_scale=1.0, latent_norm_on=1, rms_eps=1e-5, situ_b1=4.0, situ_b2=25.0,
                 cache_only=0):
        import torch
        self._keep = (arena, run_of, router_w, router_bias, down, up, sh1, sh3, sh2, latent_norm)
        ex = MoePoolLayerC(latent, inter, run_of.numel(), topk, renorm, ACT_SITU, routed_scale,
                           router_w.data_ptr(), K3C_F32, None, arena.data_ptr(),
                           pool_run_bytes(latent, inter), n_runs, run_of.data_ptr(), -1, terms)

        def p(t):   # a device tensor's address, or the host address of a k3c_q8_mat (WI8)
            if t is None:
                return None
            return C.addressof(t) if isinstance(t, Q8MatC) else t.data_ptr()
        self.c = MoeLatentLayerC(hidden, ex, p(router_w), p(router_bias), p(down), p(up), p(sh1),
                                 p(sh3), p(sh2), p(latent_norm), wdt, n_shared, latent_norm_on,
                                 rms_eps, situ_b1, situ_b2, int(cache_only))
        self._scratch = torch.empty(0, dtype=torch.uint8, device=arena.device)

    @classmethod
    def from_host(cls, layer: dict, device, terms=3, cache_only=0):
        """Upload a layer given as host numpy arrays in the oracle's form (router_w,
        router_bias, latent_norm, down, up, sh1, sh3, sh2 as fp32 or uint16 bf16 patterns
        per layer["wdt"], and ``experts``: MXFP4 expert dicts at the latent width)."""
        import torch
        dev = torch.device(device)
        t = lambda a, dt=None: None if a is None else torch.from_numpy(   # noqa: E731
            np.ascontiguousarray(a if dt is None else a.astype(dt))).to(dev)
        wdt = int(layer["wdt"])
        Lw, I = int(layer["latent"]), int(layer["inter"])
        keep = []

        def conv(a):
            if a is None:   # the shared expert's matrices of a layer with n_shared = 0
                return None
            if wdt == WBF16:
                return t(a.view(np.int16))
            if wdt == WI8:   # reference rows [f32 scale][int8 * in] -> packed on the device
                out_, row = a.shape
                wq, ws, ldw = q8_pack(t(np.ascontiguousarray(a, np.uint8)), row - 4, out_)
                keep.append((wq, ws))
                return Q8MatC(wq.data_ptr(), ws.data_ptr(), ldw)
            return t(a, np.float32)
        run = pool_run_bytes(Lw, I)
        experts = layer["experts"]
        arena = torch.empty(len(experts) * run, dtype=torch.uint8, device=dev)
        for i, e in enumerate(experts):
            de = DeviceExpert.from_host(e, dev)
            pool_pack(arena[i * run:(i + 1) * run], de.q(), Lw, I)
        torch.cuda.current_stream(dev).synchronize()
        run_of = torch.arange(len(experts), dtype=torch.int32, device=dev)
        obj = cls(arena, len(experts), run_of, t(layer["router_w"], np.float32),
                  t(layer.get("router_bias"), np.float32), conv(layer["down"]), conv(layer["up"]),
                  conv(layer["sh1"]), conv(layer["sh3"]), conv(layer["sh2"]),
                  t(layer["latent_norm"], np.float32), wdt, int(layer["hidden"]), Lw, I,
                  int(layer["n_shared"]), int(layer["topk"]), terms=terms,
                  renorm=int(layer["renorm"]), routed_scale=float(layer["routed_scale"]),
                  latent_norm_on=int(layer["latent_norm_on"]), rms_eps=float(layer["rms_eps"]),
                  situ_b1=float(layer["situ_b1"]), situ_b2=float(layer["situ_b2"]), cache_only=cache_only)
        obj._packed = keep   # the int8 arrays the k3c_q8_mat records point at
        return obj

    def scratch_bytes(self, ntok):
        return lib().k3c_moe_latent_scratch(C.byref(self.c), ntok)

    def decode(self, x, out=None, idx=None, wt=None, drops=None):
        import torch
        x = x.contiguous()
        ntok = x.shape[0]
        need = self.scratch_bytes(ntok)
        if self._scratch.numel() < need:
            self._scratch = torch.empty(need, dtype=torch.uint8, device=x.device)
        K = self.c.experts.topk
        if out is None:
            out = torch.empty((ntok, self.c.hidden), dtype=torch.float32, device=x.device)
        if idx is None:
            idx = torch.empty((ntok, K), dtype=torch.int32, device=x.device)
        if wt is None:
            wt = torch.empty((ntok, K), dtype=torch.float32, device=x.device)
        _check(lib().k3c_moe_latent_decode(_ptr(out), _ptr(x), ntok, C.byref(self.c), _ptr(idx),
                                           _ptr(wt), _ptr(drops), _ptr(self._scratch),
                                           self._scratch.numel(), _stream()),
               "k3c_moe_latent_decode")
        return out, idx, wt

    def decode_routed(self, x, idx, wt, out=None, drops=None):
        """The layer with the routing given (k3c_moe_latent_decode_routed)."""
        import torch
        x = x.contiguous()
        ntok = x.shape[0]
        need = self.scratch_bytes(ntok)
        if self._scratch.numel() < need:
            self._scratch = torch.empty(need, dtype=torch.uint8, device=x.device)
        if out is None:
            out = torch.empty((ntok, self.c.hidden), dtype=torch.float32, device=x.device)
        _check(lib().k3c_moe_latent_decode_routed(_ptr(out), _ptr(x), ntok, C.byref(self.c), _ptr(idx),
                                                  _ptr(wt), _ptr(drops), _ptr(self._scratch),
                                                  self._scratch.numel(), _stream()),
               "k3c_moe_latent_decode_routed")
        return out


# ------------------------------------------------------------------ checkpoint experts
CKPT_ALIGN = 4096


def aligned_host_buffer(nbytes, align=CKPT_ALIGN):
    """A numpy uint8 buffer of nbytes whose address is a multiple of align (for O_DIRECT)."""
    raw = np.empty(nbytes + align, np.uint8)
    off = (-raw.ctypes.data) % align
    return raw[off:off + nbytes]


DT_I8R = 5


class Trunk:
    """A packed trunk directory (k3c_trunk_*): trunk.json + trunk.bin as the reference's
    tools/pack_trunk.py and tools/int8_trunk.py write them; tensors by (layer, name), I8R
    rows (the draft model's int8 trunk) included."""

    def __init__(self, directory):
        self.p = lib().k3c_trunk_open(directory.encode())
        if not self.p:
            raise K3CError(f"k3c_trunk_open: {lib().k3c_last_error().decode()}")

    def close(self):
        if self.p:
            lib().k3c_trunk_close(self.p)
            self.p = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def layers(self):
        return lib().k3c_trunk_layers(self.p)

    def find(self, layer, name):
        t = TensorC()
        _check(lib().k3c_trunk_find(self.p, layer, name.encode(), C.byref(t)), "k3c_trunk_find")
        return t

    def read(self, t):
        """The tensor's bytes (numpy uint8), read with O_DIRECT where the trunk allows it."""
        buf = aligned_host_buffer(int(t.nbytes) + 2 * CKPT_ALIGN)
        off = C.c_int64(0)
        got = lib().k3c_trunk_read(self.p, C.byref(t), buf.ctypes.data, buf.size, C.byref(off))
        if got != t.nbytes:
            raise K3CError(f"k3c_trunk_read: {lib().k3c_last_error().decode()}")
        return buf[off.value:off.value + int(t.nbytes)].copy()

    def q8_mat(self, layer, name, device):
        """An I8R tensor as the draft model's K3C_WI8 trunk matrix: its rows copied to the device
        and packed (k3c_q8_pack). Returns (Q8MatC, the device arrays it points at)."""
        import torch
        t = self.find(layer, name)
        if t.dtype != DT_I8R:
            raise K3CError(f"{name} is dtype {t.dtype}, not I8R")
        rows = torch.from_numpy(self.read(t)).to(device)
        wq, ws, ldw = q8_pack(rows, int(t.shape[1]), int(t.shape[0]))
        return Q8MatC(wq.data_ptr(), ws.data_ptr(), ldw), (wq, ws)


class Checkpoint:
    """The safetensors shards of one checkpoint directory (k3c_ckpt_*): tensor lookup and
    routed-expert runs read from the files (O_DIRECT where the file system allows it) and
    uploaded into pool-format device runs."""

    def __init__(self, directory):
        self.h = lib().k3c_ckpt_open(os.fsencode(directory))
        if not self.h:
            raise K3CError(f"k3c_ckpt_open({directory}): {lib().k3c_last_error().decode()}")

    def close(self):
        if self.h:
            lib().k3c_ckpt_close(self.h)
            self.h = None

    def __del__(self):
        self.close()

    @property
    def shards(self):
        return lib().k3c_ckpt_shards(self.h)

    def direct(self, shard):
        return bool(lib().k3c_ckpt_direct(self.h, shard))

    def find(self, name):
        t = TensorC()
        _check(lib().k3c_ckpt_find(self.h, name.encode(), C.byref(t)), "k3c_ckpt_find")
        return t

    def expert_ref(self, layer, expert):
        r = ExpertRunC()
        _check(lib().k3c_expert_ref(self.h, layer, expert, C.byref(r)), "k3c_expert_ref")
        return r

    def read_expert(self, run, buf=None):
        """The run's bytes (a view into buf, a page-aligned host buffer of at least
        run.nbytes + 8192 bytes; allocated when None)."""
        if buf is None:
            buf = aligned_host_buffer(run.nbytes + 2 * CKPT_ALIGN)
        po = C.c_int64(0)
        n = lib().k3c_expert_read(self.h, C.byref(run), C.c_void_p(buf.ctypes.data), buf.size, C.byref(po))
        if n != run.nbytes:
            raise K3CError(f"k3c_expert_read: {lib().k3c_last_error().decode()}")
        return buf[po.value:po.value + n]

    def upload(self, run, payload, dev_run, dev_staging):
        """Pack a run read by read_expert into the pool-format device run dev_run (a torch
        uint8 view of pool_run_bytes bytes), through dev_staging (run.nbytes device bytes)."""
        ptr = payload.data_ptr() if hasattr(payload, "data_ptr") else payload.ctypes.data
        _check(lib().k3c_expert_upload(_ptr(dev_run), C.byref(run), C.c_void_p(ptr), _ptr(dev_staging),
                                       _stream()), "k3c_expert_upload")
