"""Expert-parallel MoE prefill across the ranks of a torch.distributed group.

The reference has no multi-GPU path; this is the BASELINE config[3] layer: the routed experts
are sharded over the ranks (each rank owns a set of expert ids), every rank starts with its own
tokens, and a layer is

  1. route     each rank routes its tokens (top-k ids and weights over all experts);
  2. dispatch  each token goes once to every rank that owns at least one of its experts,
               with its whole top-k row (an all-to-all of counts, then of activations, ids
               and weights);
  3. compute   each rank runs its received tokens through its own experts only (the other
               ranks' ids are not resident there and are skipped), giving one weighted
               partial sum per received token;
  4. combine   the partials go back to their source rank (all-to-all), which adds them in
               rank order to its tokens' shared-expert output.

The collectives are torch.distributed all_to_all_single (NCCL over NVLink on GPUs, gloo in
the CPU tests). The three compute steps are callables so the same orchestration runs the
tensor-core kernels on GPUs and the CPU oracle in tests:
  route(x)                  -> idx int32 [T][K], wt fp32 [T][K]
  routed(x, idx, wt)        -> fp32 [T][H], sum over the k with idx resident on this rank
  shared(x)                 -> fp32 [T][H], the shared expert (zeros if there is none)
"""
from __future__ import annotations

import ctypes as C


class ExpertParallel:
    def __init__(self, owner, route, routed, shared, group=None):
        """owner: int tensor [n_experts] -> rank holding that expert (on the compute device)."""
        import torch.distributed as dist
        self.owner = owner
        self.route, self.routed, self.shared = route, routed, shared
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.last = {}

    def _a2a(self, out, inp, out_splits=None, in_splits=None):
        """all_to_all_single; on a one-rank group the exchange is the identity (a copy), which
        keeps device tensors off a host-staged backend."""
        import torch.distributed as dist
        if self.world == 1:
            out.copy_(inp)
        else:
            dist.all_to_all_single(out, inp, output_split_sizes=out_splits, input_split_sizes=in_splits,
                                   group=self.group)

    def forward(self, x):
        import torch
        T, H = x.shape
        N = self.world
        idx, wt = self.route(x)
        # 2. dispatch: (rank, token) pairs, rank-major, tokens ascending within a rank
        dest = self.owner[idx.long()]                                  # [T, K]
        member = torch.zeros((T, N), dtype=torch.bool, device=x.device)
        member.scatter_(1, dest, True)
        pairs = member.t().nonzero()                                   # [S, 2]: (rank, token)
        send_tok = pairs[:, 1]
        send_counts = member.sum(0).to(torch.int64)                    # tokens to each rank
        recv_counts = torch.empty_like(send_counts)
        self._a2a(recv_counts, send_counts)
        ss = send_counts.cpu().tolist()
        rs = recv_counts.cpu().tolist()
        R = sum(rs)
        recv_x = x.new_empty((R, H))
        self._a2a(recv_x, x[send_tok].contiguous(), rs, ss)
        K = idx.shape[1]
        recv_idx = idx.new_empty((R, K))
        self._a2a(recv_idx, idx[send_tok].contiguous(), rs, ss)
        recv_wt = wt.new_empty((R, K))
        self._a2a(recv_wt, wt[send_tok].contiguous(), rs, ss)
        # 3. compute over this rank's experts
        part = self.routed(recv_x, recv_idx, recv_wt)                  # [R, H] fp32
        # 4. combine: partials back in the order they were sent
        back = part.new_empty((len(send_tok), H))
        self._a2a(back, part.contiguous(), ss, rs)
        y = self.shared(x)
        off = 0
        for r in range(N):                 # fixed rank order; one row per token per rank
            n = ss[r]
            if n:
                y.index_add_(0, send_tok[off:off + n], back[off:off + n])
            off += n
        self.last = {"sent_tokens": len(send_tok), "recv_tokens": R,
                     "dispatch_bytes": int(len(send_tok) * H * x.element_size()),
                     "combine_bytes": int(len(send_tok) * H * 4)}
        return y


def gpu_layer_fns(k3, layer_routed, layer_shared, router_w, router_bias, topk, renorm=1,
                  routed_scale=1.0):
    """The three compute steps on the tensor-core kernels: the router (k3c_router), the
    rank's experts with routing given (k3c_moe_prefill_tc_routed on a layer whose run table
    marks other ranks' experts -1 and which has no shared expert), and the shared expert
    alone (the same entry on a layer with only its shared run)."""
    import torch

    def route(x):
        idx, wt, _ = k3.router(x, router_w, router_bias, topk, renorm, routed_scale)
        return idx, wt

    def routed(x, idx, wt):
        return layer_routed.prefill_routed(x, idx, wt)

    def shared(x):
        T = x.shape[0]
        idx = torch.full((T, topk), -1, dtype=torch.int32, device=x.device)
        wt = torch.zeros((T, topk), dtype=torch.float32, device=x.device)
        return layer_shared.prefill_routed(x, idx, wt)

    return route, routed, shared


class FusedExpertParallel:
    """Expert-parallel MoE prefill with the exchange done by this library's kernels over peer
    memory (k3c_moe_prefill_ep_experts, k3c_moe_ep_combine): no all-to-all.

    Per layer: (1) this rank copies its tokens into its shared x buffer and routes them into
    its shared idx / wt buffers; (2) after a barrier, every rank runs its own experts over the
    pairs of ALL ranks (its quantisation kernel reads the peers' token rows over NVLink) and
    its down-projection epilogue stores each pair's output as a bf16 row into the token
    owner's receive buffer (stores over NVLink, overlapping the following tiles' MMAs);
    (3) after a second barrier, each rank adds its tokens' rows in top-k order with its own
    weights, then the shared expert's row -- the single-GPU combine, so the result equals the
    single-GPU layer bit for bit.

    The barriers are one-element NCCL all-reduces on the current stream: a rank's step-2
    kernels start only after every rank's step-1 writes are complete, and its combine only
    after every rank has stored its pair rows.

    layer: a PoolMoeLayer whose run table marks the other ranks' experts -1 and whose shared
    run is the shared expert (each rank computes its own tokens' shared expert). An expert in
    every rank's run table is a replicated hot expert: each rank runs only its own tokens'
    pairs of it (k3c_ep_peers.local_only).

    gather_x (more than one rank): every rank's token rows are gathered into a local buffer
    by an NCCL all-gather on a side stream while the router runs (over NVSwitch each row
    leaves its owner once), so the token quantisation of step 2 reads them from local memory
    instead of pulling them from the owners over NVLink after the barrier. The all-gather has
    a communicator of its own, so it runs beside the first barrier, and step 2 waits for it
    (k3c_ep_peers.x_ready) only after its planning, right before the quantisation.
    """

    def __init__(self, k3, layer, t_max, x_dtype=None, group=None, gather_x=True):
        import torch
        import torch.distributed as dist
        self.k3, self.layer, self.group = k3, layer, group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > k3.EP_MAX:
            raise ValueError(f"expert parallelism over at most {k3.EP_MAX} ranks")
        c = layer.c
        self.H, self.K, self.E = c.hidden, c.topk, c.n_experts
        self.t_max = int(t_max)
        self.x_dtype = x_dtype or torch.bfloat16
        L = k3.lib()
        esize = torch.empty(0, dtype=self.x_dtype).element_size()
        W_, T_ = self.world, self.t_max
        sizes = {"x": T_ * self.H * esize, "idx": T_ * self.K * 4, "wt": T_ * self.K * 4,
                 "recv": T_ * (self.K + 1) * self.H * 2}
        self._own, handles = {}, {}
        for name, nb in sizes.items():
            ptr, h = C.c_void_p(), k3.IpcHandleC()
            k3._check(L.k3c_ep_alloc(C.byref(ptr), nb, C.byref(h)), "k3c_ep_alloc")
            self._own[name] = ptr.value
            handles[name] = bytes(h.bytes)
        dev = torch.device("cuda", torch.cuda.current_device())
        self.x_buf = k3.device_view(self._own["x"], (T_, self.H), self.x_dtype)
        self.idx_buf = k3.device_view(self._own["idx"], (T_, self.K), torch.int32)
        self.wt_buf = k3.device_view(self._own["wt"], (T_, self.K), torch.float32)
        # the rank holding each expert (every rank's run table marks its own experts)
        mine = (layer.run_of >= 0).to(torch.int32)
        every = [torch.empty_like(mine) for _ in range(W_)] if W_ > 1 else [mine]
        if W_ > 1:
            dist.all_gather(every, mine, group=group)
        rank_of = torch.full((self.E,), -1, dtype=torch.int32, device=dev)
        for q in reversed(range(W_)):
            rank_of[every[q].bool()] = q
        self.expert_rank = rank_of
        # experts every rank holds (hot experts replicated to spread their load): each rank
        # runs only its own tokens' pairs of them, so their pair rows stay local
        held = torch.stack([v.bool() for v in every]).all(0) if W_ > 1 else torch.zeros_like(mine, dtype=torch.bool)
        self.local_only = held.to(torch.uint8) if bool(held.any()) else None
        torch.cuda.synchronize()
        everyone = [None] * W_
        dist.all_gather_object(everyone, handles, group=group)
        self._opened = []
        self.peers = k3.EpPeersC()
        self.peers.world, self.peers.rank, self.peers.t_max = W_, self.rank, T_
        self.peers.x_dtype = k3._dtype_code(torch.empty(0, dtype=self.x_dtype))
        self.peers.local_only = self.local_only.data_ptr() if self.local_only is not None else None
        for q in range(W_):
            for name in sizes:
                if q == self.rank:
                    p = self._own[name]
                else:
                    h = k3.IpcHandleC()
                    C.memmove(h.bytes, everyone[q][name], 64)
                    ptr = C.c_void_p()
                    k3._check(L.k3c_ep_open(C.byref(ptr), C.byref(h)), "k3c_ep_open")
                    p = ptr.value
                    self._opened.append(p)
                getattr(self.peers, name)[q] = p
        # every rank's token rows, ranks after one another: the quantisation reads the other
        # ranks' tokens from here (this rank's own from x_buf)
        self.gx = None
        if gather_x and W_ > 1:
            self.gx = torch.empty((W_ * T_, self.H), dtype=self.x_dtype, device=dev)
            for q in range(W_):
                if q != self.rank:
                    self.peers.x[q] = self.gx[q * T_:(q + 1) * T_].data_ptr()
            self._side = torch.cuda.Stream(device=dev)
            self._gx_group = dist.new_group(dist.get_process_group_ranks(group) if group is not None
                                            else list(range(W_)))
            self._gx_ready = torch.cuda.Event()
        self._flag = torch.zeros(1, dtype=torch.float32, device=dev)
        self._ntok = torch.zeros(W_, dtype=torch.int32, device=dev)
        self._scratch = torch.empty(0, dtype=torch.uint8, device=dev)
        self._rscratch = torch.empty(0, dtype=torch.uint8, device=dev)
        self._counts = None
        self._ph = None
        self.last = {}

    PHASES = ("route", "barrier1", "experts_call", "barrier2", "combine")

    def phase_timing(self, on=True):
        """Record CUDA events between the layer's phases on the current stream (route: token copy
        and router; barrier1; experts_call: planning, dispatch, the grouped GEMMs and the pair
        rows; barrier2; combine); phase_read() returns their mean milliseconds."""
        self._ph = [] if on else None

    def phase_read(self):
        import torch
        if not self._ph:
            return None
        torch.cuda.synchronize()
        tot = [0.0] * len(self.PHASES)
        for ev in self._ph:
            for i in range(len(self.PHASES)):
                tot[i] += ev[i].elapsed_time(ev[i + 1])
        n = len(self._ph)
        self._ph = []
        return {name: tot[i] / n for i, name in enumerate(self.PHASES)}

    def _mark(self, ev, i):
        if ev is not None:
            ev[i].record()

    def _barrier(self):
        import torch.distributed as dist
        if self.world > 1:
            dist.all_reduce(self._flag, group=self.group)

    def forward(self, x, counts=None):
        """counts: every rank's token count when the caller knows it (e.g. equal splits);
        otherwise it is gathered, which costs a host synchronisation per layer."""
        import torch
        import torch.distributed as dist
        k3, L, c = self.k3, self.k3.lib(), self.layer.c
        T = x.shape[0]
        if T > self.t_max:
            raise ValueError(f"{T} tokens > t_max {self.t_max}")
        # every rank's token count (the plan is sized on the host)
        if counts is not None:
            counts = [int(v) for v in counts]
            if len(counts) != self.world or counts[self.rank] != T:
                raise ValueError(f"counts {counts} do not match this rank's {T} tokens")
        elif self.world > 1:
            mine = torch.full((1,), T, dtype=torch.int32, device=x.device)
            dist.all_gather_into_tensor(self._ntok, mine, group=self.group)
            counts = self._ntok.cpu().tolist()
        else:
            counts = [T]
        for q in range(self.world):
            self.peers.ntok[q] = int(counts[q])
        ev = None
        if self._ph is not None:
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(len(self.PHASES) + 1)]
            self._ph.append(ev)
        self._mark(ev, 0)
        # 1. this rank's tokens and their routing into the shared buffers; with gather_x the
        # token rows of every rank are gathered on a side stream meanwhile
        self.x_buf[:T].copy_(x)
        main = torch.cuda.current_stream()
        if self.gx is not None:
            self._side.wait_stream(main)
            with torch.cuda.stream(self._side):
                dist.all_gather_into_tensor(self.gx, self.x_buf, group=self._gx_group)
                self._gx_ready.record(self._side)
            self.peers.x_ready = self._gx_ready.cuda_event
        if T:
            rneed = L.k3c_router_scratch(self.H, self.E, T)
            if self._rscratch.numel() < rneed:
                self._rscratch = torch.empty(rneed, dtype=torch.uint8, device=x.device)
            k3._check(L.k3c_router_ws(k3._ptr(self.idx_buf), k3._ptr(self.wt_buf), None, k3._ptr(self.x_buf),
                                      k3._dtype_code(self.x_buf), C.c_void_p(c.router_w), c.router_dtype,
                                      C.c_void_p(c.router_bias), self.H, self.E, self.K, c.renorm,
                                      c.routed_scale, T, k3._ptr(self._rscratch), self._rscratch.numel(),
                                      k3._stream()), "k3c_router_ws")
        self._mark(ev, 1)
        self._barrier()
        self._mark(ev, 2)
        # 2. every rank's pairs through this rank's experts; pair rows to the tokens' owners
        need = L.k3c_moe_prefill_ep_scratch(C.byref(c), C.byref(self.peers))
        if need == 0:
            raise k3.K3CError(f"k3c_moe_prefill_ep_scratch: {L.k3c_last_error().decode()}")
        if self._scratch.numel() < need:
            self._scratch = torch.empty(need, dtype=torch.uint8, device=x.device)
        k3._check(L.k3c_moe_prefill_ep_experts(C.byref(c), C.byref(self.peers), k3._ptr(self._scratch),
                                               self._scratch.numel(), k3._stream()),
                  "k3c_moe_prefill_ep_experts")
        if self.gx is not None:
            main.wait_stream(self._side)   # ordered through x_ready already; joins the streams
        self._mark(ev, 3)
        self._barrier()
        self._mark(ev, 4)
        # 3. this rank's tokens: their pair rows in top-k order, then the shared row
        out = torch.empty((T, self.H), dtype=torch.float32, device=x.device)
        k3._check(L.k3c_moe_ep_combine(k3._ptr(out), C.byref(self.peers), self.H, self.K,
                                       k3._ptr(self.expert_rank), self.E, 1 if c.shared_run >= 0 else 0,
                                       k3._stream()), "k3c_moe_ep_combine")
        self._mark(ev, 5)
        self.last = {"tokens": counts, "remote_rows_read": sum(counts) - T}
        return out

    def close(self):
        """Unmaps the peers' buffers and frees this rank's (between barriers, so no peer is
        still using them)."""
        import torch
        if not self._own:
            return
        torch.cuda.synchronize()
        self._barrier()
        torch.cuda.synchronize()
        L = self.k3.lib()
        for p in self._opened:
            L.k3c_ep_close(C.c_void_p(p))
        self._opened = []
        self._barrier()
        torch.cuda.synchronize()
        for p in self._own.values():
            L.k3c_ep_free(C.c_void_p(p))
        self._own = {}


def balanced_placement(load, world):
    """Expert -> rank placement with every rank holding len(load) / world experts and the
    ranks' summed loads as even as a greedy pass makes them: experts in decreasing load, each
    to the least-loaded rank that still has room (longest-processing-time first). `load` is a
    per-expert pair count from a routing sample. Returns (owner [E] list, per-rank id lists,
    each ascending)."""
    E = len(load)
    if E % world:
        raise ValueError(f"{E} experts do not split over {world} ranks")
    cap = E // world
    order = sorted(range(E), key=lambda e: (-float(load[e]), e))
    sums = [0.0] * world
    lists = [[] for _ in range(world)]
    owner = [0] * E
    for e in order:
        r = min((q for q in range(world) if len(lists[q]) < cap), key=lambda q: (sums[q], q))
        lists[r].append(e)
        sums[r] += float(load[e])
        owner[e] = r
    return owner, [sorted(v) for v in lists]
