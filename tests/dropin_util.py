"""Helpers for the k3_moe / k3_moe_prefill drop-in tests: the reference's K3MoeW / K3Cfg built
from a layer dict (the oracle's form, kimi-k3-in-rust_b200/synth.latent_layer), an expert
source over host numpy experts that logs every call, and the two entry points -- this
library's drop-in and the reference's own k3_moe / k3_moe_prefill (oracle/_ref) -- called on
the same structs and the same source."""
import ctypes as C

import numpy as np


class MoeArgs:
    """K3MoeW + K3Cfg for one layer dict; keeps the arrays they point at alive."""

    def __init__(self, k3, layer, src=None, cache_only=0, layer_id=0):
        self.keep = []
        wdt = int(layer["wdt"])
        wdtype = np.uint16 if wdt == 1 else (np.uint8 if wdt == 2 else np.float32)

        def ptr(name, dtype):
            a = layer.get(name)
            if a is None:
                return None
            a = np.ascontiguousarray(a, dtype)
            self.keep.append(a)
            return a.ctypes.data

        w = k3.K3MoeWC()
        w.gate, w.bias = ptr("router_w", np.float32), ptr("router_bias", np.float32)
        w.w1, w.w3, w.w2 = ptr("w1", np.float32), ptr("w3", np.float32), ptr("w2", np.float32)
        w.latent_norm = ptr("latent_norm", np.float32)
        w.down, w.up = ptr("down", wdtype), ptr("up", wdtype)
        w.sh1, w.sh3, w.sh2 = ptr("sh1", wdtype), ptr("sh3", wdtype), ptr("sh2", wdtype)
        w.wdt = wdt
        if src is not None:
            w.src = C.cast(src, C.POINTER(k3.K3ExpertSrcC)) if isinstance(src, int) else C.pointer(src)
        w.layer = layer_id
        w.cache_only = cache_only
        c = k3.K3CfgC()
        c.hidden, c.latent, c.moe_inter = int(layer["hidden"]), int(layer["latent"]), int(layer["inter"])
        c.n_experts, c.topk, c.n_shared = int(layer["n_experts"]), int(layer["topk"]), int(layer["n_shared"])
        c.routed_scale, c.moe_renorm = float(layer["routed_scale"]), int(layer["renorm"])
        c.latent_norm, c.rms_eps = int(layer["latent_norm_on"]), float(layer["rms_eps"])
        c.situ_b1, c.situ_b2 = float(layer["situ_b1"]), float(layer["situ_b2"])
        c.n_layers = layer_id + 1
        self.w, self.c = w, c


class HostSource:
    """A K3ExpertSrc over host MXFP4 experts (reference layout). get() fails for the ids in
    `fail`; resident() (present when `resident` is a set) reports membership. Every call is
    appended to `log`."""

    def __init__(self, k3, experts, resident=None, fail=(), getmany=True):
        self.experts = experts
        self.resident_set = resident
        self.fail = set(fail)
        self.log = []
        self._get = k3.SRC_GET_FN(self._cb_get)
        self._many = k3.SRC_GETMANY_FN(self._cb_many) if getmany else k3.SRC_GETMANY_FN()
        self._res = k3.SRC_GET_FN(self._cb_res) if resident is not None else k3.SRC_GET_FN()
        self.src = k3.K3ExpertSrcC(self._get, self._many, self._res, None)

    def _fill(self, e, q):
        x = self.experts[e]
        q.contents.p1, q.contents.s1 = x["gate_p"].ctypes.data, x["gate_s"].ctypes.data
        q.contents.p3, q.contents.s3 = x["up_p"].ctypes.data, x["up_s"].ctypes.data
        q.contents.p2, q.contents.s2 = x["down_p"].ctypes.data, x["down_s"].ctypes.data

    def _cb_get(self, selfp, layer, e, q):
        self.log.append(("get", layer, e))
        if e in self.fail or not 0 <= e < len(self.experts):
            return -1
        self._fill(e, q)
        return 0

    def _cb_many(self, selfp, layer, ids, n):
        self.log.append(("getmany", layer, tuple(ids[i] for i in range(n))))
        return n

    def _cb_res(self, selfp, layer, e, q):
        self.log.append(("resident", layer, e, bool(q)))
        r = e in self.resident_set
        if r and q:
            self._fill(e, q)
        return int(r)


def ours(k3, args, x, prefill=False, idx0=None, wt0=None):
    """This library's drop-in. Returns (out, idx, wt, drops counted by the call)."""
    L = k3.lib()
    x = np.ascontiguousarray(x, np.float32)
    T = x.shape[0]
    K = args.c.topk
    out = np.full_like(x, np.nan)
    idx = np.array(idx0 if idx0 is not None else np.full(K, -7), np.int32)
    wt = np.array(wt0 if wt0 is not None else np.full(K, -7.0), np.float32)
    drops = C.c_long.in_dll(L, "k3_expert_drops")
    d0 = drops.value
    fn = L.k3_moe_prefill if prefill else L.k3_moe
    fn(out.ctypes.data, x.ctypes.data, C.byref(args.w), C.byref(args.c), T, idx.ctypes.data, wt.ctypes.data, None)
    return out, idx, wt, drops.value - d0


def reference(ora, args, x, prefill=False, idx0=None, wt0=None):
    """The reference's own k3_moe / k3_moe_prefill on the same structs."""
    x = np.ascontiguousarray(x, np.float32)
    T = x.shape[0]
    K = args.c.topk
    out = np.full_like(x, np.nan)
    idx = np.array(idx0 if idx0 is not None else np.full(K, -7), np.int32)
    wt = np.array(wt0 if wt0 is not None else np.full(K, -7.0), np.float32)
    d = ora.ref().refh_moe_call(int(prefill), out, x, T, C.addressof(args.w), C.addressof(args.c),
                                idx.ctypes.data, wt.ctypes.data)
    assert d >= 0
    return out, idx, wt, d
