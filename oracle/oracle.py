"""ctypes binding for the CPU checker libraries. TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm import
this module. It binds

  * ``liboracle.so``      -- the CPU restatement (oracle/k3_oracle.c), and
  * ``_ref/libk3ref.so``  -- the reference's own kernels compiled from its sources plus
                             oracle/ref_harness.c (present when built in the container that
                             has the reference tree; it travels with the snapshot).

Arrays are numpy; every call checks dtypes and contiguity so a wrong buffer cannot be
passed through silently.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libk3ref.so")

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")


class Expert6(C.Structure):
    """Six (packed, scale) host pointers in the K3ExpertQ order p1,s1,p3,s3,p2,s2
    (include/k3/k3.h:323-327 of the reference)."""

    _fields_ = [(n, C.c_void_p) for n in ("p1", "s1", "p3", "s3", "p2", "s2")]


class OraLatent(C.Structure):
    """ora_latent (oracle/k3_oracle.h): one K3 latent MoE layer."""

    _fields_ = ([(n, C.c_void_p) for n in ("router_w", "router_bias", "w1", "w3", "w2",
                                           "experts", "latent_norm", "down", "up", "sh1",
                                           "sh3", "sh2")]
                + [(n, C.c_int) for n in ("wdt", "hidden", "latent", "inter", "n_shared",
                                          "n_experts", "topk", "renorm", "latent_norm_on")]
                + [(n, C.c_float) for n in ("routed_scale", "rms_eps", "situ_b1", "situ_b2")])


def expert6(e: dict) -> Expert6:
    """Build an Expert6 from a dict of numpy uint8 arrays (keys gate_p, gate_s, up_p,
    up_s, down_p, down_s). The caller keeps the arrays alive."""
    return Expert6(*(e[k].ctypes.data for k in ("gate_p", "gate_s", "up_p", "up_s",
                                                 "down_p", "down_s")))


def _build():
    subprocess.run(["make", "-s", "-f", os.path.join(HERE, "Makefile")], check=True)


_lib = None
_ref = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_SO):
            _build()
        L = C.CDLL(ORACLE_SO)
        L.ora_mxfp4_dequant.argtypes = [_f32p, _u8p, _u8p, C.c_int, C.c_int, C.c_int]
        L.ora_matmul_mxfp4.argtypes = [_f32p, _f32p, _u8p, _u8p, C.c_int, C.c_int, C.c_int]
        L.ora_matmul_f32.argtypes = [_f32p, _f32p, _f32p, C.c_int, C.c_int]
        L.ora_matmul_bf16.argtypes = [_f32p, _f32p, _u16p, C.c_int, C.c_int]
        L.ora_rmsnorm.argtypes = [_f32p, _f32p, _f32p, C.c_int, C.c_float]
        L.ora_moe_latent.argtypes = [_f32p, _f32p, C.c_int, C.POINTER(OraLatent), _i32p, _f32p]
        L.ora_matmul_q8.argtypes = [_f32p, _f32p, _u8p, C.c_int, C.c_int]
        L.ora_router.argtypes = [_i32p, _f32p, _f32p, _f32p, C.c_void_p, C.c_int, C.c_int,
                                 C.c_int, C.c_int, C.c_float]
        L.ora_router_select.argtypes = [_i32p, _f32p, _f32p, C.c_void_p, C.c_int, C.c_int,
                                        C.c_int, C.c_float]
        L.ora_router_scores.argtypes = [_f32p, _f32p, _f32p, C.c_int, C.c_int]
        L.ora_swiglu.argtypes = [_f32p, _f32p, C.c_int]
        L.ora_situ_glu.argtypes = [_f32p, _f32p, C.c_int, C.c_float, C.c_float]
        L.ora_expert_ffn.argtypes = [_f32p, _f32p, C.c_int, C.POINTER(Expert6), C.c_int,
                                     C.c_int, C.c_int]
        L.ora_moe_layer.argtypes = [_f32p, _f32p, C.c_int, _f32p, C.c_void_p,
                                    C.POINTER(Expert6), C.c_void_p, C.c_int, C.c_int,
                                    C.c_int, C.c_int, C.c_int, C.c_float, C.c_int,
                                    _i32p, _f32p]
        L.ora_e2m1.restype = C.c_float
        L.ora_e8m0.restype = C.c_float
        _lib = L
    return _lib


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref():
    """The reference's own kernels (k3_matmul_mxfp4, k3_router, k3_matmul_q8, ...) plus the
    BASELINE compositions of oracle/ref_harness.c."""
    global _ref
    if _ref is None:
        if not ref_available():
            raise FileNotFoundError(REF_SO)
        L = C.CDLL(REF_SO)
        L.k3_mxfp4_dequant.argtypes = [_f32p, _u8p, _u8p, C.c_int, C.c_int, C.c_int]
        L.k3_matmul_mxfp4.argtypes = [_f32p, _f32p, _u8p, _u8p, C.c_int, C.c_int, C.c_int]
        L.k3_matmul_q8.argtypes = [_f32p, _f32p, _u8p, C.c_int, C.c_int]
        L.k3_matmul.argtypes = [_f32p, _f32p, _f32p, C.c_int, C.c_int]
        L.k3_matmul_bf16.argtypes = [_f32p, _f32p, _u16p, C.c_int, C.c_int]
        L.refh_moe_latent.argtypes = ([_f32p, _f32p, C.c_int] + [C.c_void_p] * 12
                                      + [C.c_int] * 7 + [C.c_int, C.c_float, C.c_int]
                                      + [C.c_float] * 3 + [_i32p, _f32p])
        L.k3_router.argtypes = [_i32p, _f32p, _f32p, _f32p, C.c_void_p, C.c_int, C.c_int,
                                C.c_int, C.c_int, C.c_float]
        L.refh_expert_ffn.argtypes = [_f32p, _f32p, C.c_int, C.POINTER(Expert6), C.c_int,
                                      C.c_int, C.c_int]
        L.refh_moe_layer.argtypes = [_f32p, _f32p, C.c_int, _f32p, C.c_void_p,
                                     C.POINTER(Expert6), C.c_void_p, C.c_int, C.c_int,
                                     C.c_int, C.c_int, C.c_int, C.c_float, C.c_int,
                                     _i32p, _f32p]
        L.refh_moe_call.argtypes = [C.c_int, _f32p, _f32p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                    C.c_void_p]
        L.refh_moe_call.restype = C.c_long
        L.refh_threads.restype = C.c_int
        L.refh_set_threads.argtypes = [C.c_int]
        L.refh_set_threads.restype = None
        L.refh_expert_read.argtypes = [C.c_char_p, C.c_int, C.c_int, C.c_void_p, C.c_longlong,
                                       C.c_void_p, C.POINTER(C.c_longlong)]
        L.refh_expert_read.restype = C.c_longlong
        L.refh_st_find.argtypes = [C.c_char_p, C.POINTER(C.c_char_p), C.c_int, C.POINTER(C.c_longlong)]
        L.refh_st_find.restype = C.c_int
        L.refh_cache_replay.argtypes = [C.c_char_p, C.c_void_p, C.c_int, C.POINTER(C.c_int), C.c_int, C.c_int,
                                        C.POINTER(C.c_int), C.POINTER(C.c_int), C.POINTER(C.c_ulonglong),
                                        C.POINTER(C.c_int), C.c_longlong, C.POINTER(C.c_longlong),
                                        C.POINTER(C.c_uint)]
        L.refh_cache_replay.restype = C.c_int
        _ref = L
    return _ref


def host_cores() -> int:
    """Host cores this process may run on (its CPU affinity)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


def ref_use_all_cores() -> int:
    """Make the reference's OpenMP loops use every host core of this process and return that
    count. A launcher such as torch.distributed.run exports OMP_NUM_THREADS=1 to every rank;
    the CPU baseline runs on rank 0 alone and may use the whole host."""
    n = host_cores()
    ref().refh_set_threads(n)
    return ref().refh_threads()


def _ptr_or_null(a):
    return None if a is None else a.ctypes.data


# ---------------------------------------------------------------- convenience wrappers


def mxfp4_dequant(packed, scales, group=32, L=None):
    L = L or lib()
    rows, pcols = packed.shape
    out = np.empty((rows, pcols * 2), np.float32)
    fn = L.ora_mxfp4_dequant if hasattr(L, "ora_mxfp4_dequant") else L.k3_mxfp4_dequant
    fn(out, np.ascontiguousarray(packed), np.ascontiguousarray(scales), rows, pcols, group)
    return out


def matmul_mxfp4(x, packed, scales, group=32, use_ref=False):
    L = ref() if use_ref else lib()
    fn = L.k3_matmul_mxfp4 if use_ref else L.ora_matmul_mxfp4
    rows, pcols = packed.shape
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty(rows, np.float32)
    fn(y, x, np.ascontiguousarray(packed), np.ascontiguousarray(scales), pcols * 2, rows,
       group)
    return y


def matmul_q8(x, W_rows, in_, out, use_ref=False):
    L = ref() if use_ref else lib()
    fn = L.k3_matmul_q8 if use_ref else L.ora_matmul_q8
    y = np.empty(out, np.float32)
    fn(y, np.ascontiguousarray(x, np.float32), np.ascontiguousarray(W_rows), in_, out)
    return y


def router(x, W, bias, topk, renorm=1, routed_scale=1.0, use_ref=False):
    L = ref() if use_ref else lib()
    fn = L.k3_router if use_ref else L.ora_router
    E, H = W.shape
    idx = np.empty(topk, np.int32)
    w = np.empty(topk, np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    fn(idx, w, np.ascontiguousarray(x, np.float32), np.ascontiguousarray(W, np.float32),
       _ptr_or_null(b), H, E, topk, renorm, routed_scale)
    return idx, w


def router_select(score, bias, topk, renorm=1, routed_scale=1.0):
    idx = np.empty(topk, np.int32)
    w = np.empty(topk, np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    lib().ora_router_select(idx, w, np.ascontiguousarray(score, np.float32), _ptr_or_null(b),
                            score.shape[0], topk, renorm, routed_scale)
    return idx, w


def router_scores(x, W):
    E, H = W.shape
    s = np.empty(E, np.float32)
    lib().ora_router_scores(s, np.ascontiguousarray(x, np.float32),
                            np.ascontiguousarray(W, np.float32), H, E)
    return s


def expert_ffn(x, e: dict, hidden, inter, act=0, use_ref=False):
    x = np.ascontiguousarray(x, np.float32).reshape(-1, hidden)
    y = np.empty_like(x)
    q = expert6(e)
    if use_ref:
        rc = ref().refh_expert_ffn(y, x, x.shape[0], C.byref(q), hidden, inter, act)
        assert rc == 0
    else:
        lib().ora_expert_ffn(y, x, x.shape[0], C.byref(q), hidden, inter, act)
    return y


def moe_layer(x, router_w, router_bias, experts: list, shared, hidden, inter, topk,
              renorm=1, routed_scale=1.0, act=0, use_ref=False):
    """experts: list indexed by expert id of expert dicts (None for experts that must never
    be selected is not allowed -- every entry must be valid)."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1, hidden)
    T = x.shape[0]
    E = router_w.shape[0]
    arr = (Expert6 * E)(*[expert6(e) for e in experts])
    sh = expert6(shared) if shared is not None else None
    out = np.empty_like(x)
    idx = np.empty((T, topk), np.int32)
    wt = np.empty((T, topk), np.float32)
    b = None if router_bias is None else np.ascontiguousarray(router_bias, np.float32)
    args = (out, x, T, np.ascontiguousarray(router_w, np.float32), _ptr_or_null(b), arr,
            None if sh is None else C.addressof(sh), hidden, inter, E, topk, renorm,
            routed_scale, act, idx, wt)
    if use_ref:
        assert ref().refh_moe_layer(*args) == 0
    else:
        lib().ora_moe_layer(*args)
    return out, idx, wt


def matmul_f32(x, W, use_ref=False):
    """y = W x with fp32 W [out][in] in the reference's k3_matmul order."""
    out_, in_ = W.shape
    y = np.empty(out_, np.float32)
    fn = ref().k3_matmul if use_ref else lib().ora_matmul_f32
    fn(y, np.ascontiguousarray(x, np.float32), np.ascontiguousarray(W, np.float32), in_, out_)
    return y


def matmul_bf16(x, W, use_ref=False):
    """y = W x with bf16 W (uint16 bit patterns [out][in]) in the reference's order."""
    out_, in_ = W.shape
    y = np.empty(out_, np.float32)
    fn = ref().k3_matmul_bf16 if use_ref else lib().ora_matmul_bf16
    fn(y, np.ascontiguousarray(x, np.float32), np.ascontiguousarray(W, np.uint16), in_, out_)
    return y


_LATENT_INTS = ("wdt", "hidden", "latent", "inter", "n_shared", "n_experts", "topk", "renorm",
                "latent_norm_on")
_LATENT_FLOATS = ("routed_scale", "rms_eps", "situ_b1", "situ_b2")


def moe_latent(x, layer: dict, use_ref=False):
    """The K3 latent MoE layer on x [T][hidden]. layer holds numpy arrays (router_w,
    router_bias or None, latent_norm, down, up, sh1, sh3, sh2 -- fp32 or uint16 bf16 per
    layer["wdt"] -- and either the fp32 bank w1/w3/w2 or a list ``experts`` of MXFP4 expert
    dicts at the latent width) plus the integer and float fields of ora_latent. Returns
    (out, idx, wt). use_ref runs the reference's own k3_moe."""
    H, K = layer["hidden"], layer["topk"]
    x = np.ascontiguousarray(x, np.float32).reshape(-1, H)
    T = x.shape[0]
    keep = []

    def ptr(name, dtype=None):
        a = layer.get(name)
        if a is None:
            return None
        a = np.ascontiguousarray(a, dtype) if dtype is not None else np.ascontiguousarray(a)
        keep.append(a)
        return a.ctypes.data

    wdtype = np.uint16 if layer["wdt"] == 1 else (np.uint8 if layer["wdt"] == 2 else np.float32)
    experts = layer.get("experts")
    arr = None
    if experts is not None:
        arr = (Expert6 * len(experts))(*[expert6(e) for e in experts])
    out = np.empty_like(x)
    idx = np.empty((T, K), np.int32)
    wt = np.empty((T, K), np.float32)
    ptrs = dict(router_w=ptr("router_w", np.float32), router_bias=ptr("router_bias", np.float32),
                w1=ptr("w1", np.float32), w3=ptr("w3", np.float32), w2=ptr("w2", np.float32),
                experts=None if arr is None else C.addressof(arr),
                latent_norm=ptr("latent_norm", np.float32),
                down=ptr("down", wdtype), up=ptr("up", wdtype), sh1=ptr("sh1", wdtype),
                sh3=ptr("sh3", wdtype), sh2=ptr("sh2", wdtype))
    if use_ref:
        rc = ref().refh_moe_latent(
            out, x, T, ptrs["router_w"], ptrs["router_bias"], ptrs["experts"], ptrs["w1"],
            ptrs["w3"], ptrs["w2"], ptrs["latent_norm"], ptrs["down"], ptrs["up"],
            ptrs["sh1"], ptrs["sh3"], ptrs["sh2"], layer["wdt"], H, layer["latent"],
            layer["inter"], layer["n_shared"], layer["n_experts"], K, layer["renorm"],
            layer["routed_scale"], layer["latent_norm_on"], layer["rms_eps"],
            layer["situ_b1"], layer["situ_b2"], idx, wt)
        assert rc == 0
    else:
        c = OraLatent(**ptrs, **{k: int(layer[k]) for k in _LATENT_INTS},
                      **{k: float(layer[k]) for k in _LATENT_FLOATS})
        lib().ora_moe_latent(out, x, T, C.byref(c), idx, wt)
    return out, idx, wt


def rmsnorm(x, w, eps=1e-5):
    """k3_rmsnorm row by row (double sum of squares in element order)."""
    x = np.ascontiguousarray(x, np.float32)
    rows = x.reshape(-1, x.shape[-1])
    out = np.empty_like(rows)
    for r in range(rows.shape[0]):
        y = np.empty(rows.shape[1], np.float32)
        lib().ora_rmsnorm(y, np.ascontiguousarray(rows[r]), np.ascontiguousarray(w, np.float32),
                          rows.shape[1], eps)
        out[r] = y
    return out.reshape(x.shape)


def situ_glu(gu, b1=4.0, b2=25.0):
    """k3_situ_glu row by row: gu [..][2n] -> [..][n]."""
    gu = np.ascontiguousarray(gu, np.float32)
    rows = gu.reshape(-1, gu.shape[-1])
    n = rows.shape[1] // 2
    out = np.empty((rows.shape[0], n), np.float32)
    for r in range(rows.shape[0]):
        y = np.empty(n, np.float32)
        lib().ora_situ_glu(y, np.ascontiguousarray(rows[r]), n, b1, b2)
        out[r] = y
    return out


def ref_expert_read(directory, layer, expert, run_struct_type, cap):
    """The reference's own k3_st_open + k3_expert_ref + k3_expert_load_direct. Returns
    (status, run, payload bytes): status -1 when the shards do not open, -2 when the expert is
    rejected, else the bytes read. run_struct_type is a ctypes mirror of K3ExpertRef."""
    import os as _os
    raw = np.empty(cap + 4096, np.uint8)
    off = (-raw.ctypes.data) % 4096
    buf = raw[off:off + cap]
    run = run_struct_type()
    po = C.c_longlong(0)
    n = ref().refh_expert_read(_os.fsencode(directory), layer, expert, buf.ctypes.data, cap,
                               C.addressof(run), C.byref(po))
    if n < 0:
        return int(n), None, None
    return int(n), run, buf[po.value:po.value + n].copy()


def ref_st_find(directory, names):
    """The reference's own k3_st_open + k3_st_find. Returns None when the shards do not open,
    else one tuple per name: (found, shard, dtype, ndim, offset, nbytes, shape0, shape1)."""
    import os as _os
    arr = (C.c_char_p * len(names))(*[n.encode() for n in names])
    info = (C.c_longlong * (8 * len(names)))()
    if ref().refh_st_find(_os.fsencode(directory), arr, len(names), info) != 0:
        return None
    return [tuple(info[8 * i:8 * i + 8]) for i in range(len(names))]


def ref_cache_replay(directory, cfg, nslot, records):
    """The reference's own expert cache (src/cache/k3_cache.c) over the checkpoint in
    `directory`, with exactly nslot slots, replaying records [(kind, layer, ids)]: kind 0 get
    of ids[0], 1 getmany of ids, 2 pin ids[0], 3 unpin ids[0]. cfg: a K3Cfg ctypes structure
    (n_layers, n_experts, topk, first_dense are read). Returns a dict: key_of after each
    record, rc of each call, hits/misses/evictions/prefetch_reads, the (layer, expert) trace
    and the request histogram; None when the checkpoint or the cache does not open."""
    flat = []
    for kind, layer, ids in records:
        flat += [kind, layer, len(ids)] + list(ids)
    nrec = len(records)
    ops = (C.c_int * max(1, len(flat)))(*flat)
    key_of = (C.c_int * (nrec * nslot))()
    rc = (C.c_int * max(1, nrec))()
    stats = (C.c_ulonglong * 4)()
    cap = 2 * nrec + 2
    trace = (C.c_int * cap)()
    ntrace = C.c_longlong(0)
    hist = (C.c_uint * (cfg.n_layers * cfg.n_experts))()
    n = ref().refh_cache_replay(os.fsencode(directory), C.addressof(cfg), nslot, ops, len(flat), nrec, key_of, rc,
                                stats, trace, cap, C.byref(ntrace), hist)
    if n != nrec:
        return None
    return {"key_of": [list(key_of[i * nslot:(i + 1) * nslot]) for i in range(nrec)], "rc": list(rc[:nrec]),
            "hits": stats[0], "misses": stats[1], "evictions": stats[2], "prefetch_reads": stats[3],
            "trace": [(trace[2 * i], trace[2 * i + 1]) for i in range(ntrace.value // 2)],
            "hist": list(hist)}
