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
