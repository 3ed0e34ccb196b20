"""bench.py -- BASELINE metric "MXFP4 MoE-layer tokens/s" on B200.

Workload: one MoE layer decode on one GPU -- hidden 7168, 384 routed
MXFP4 experts (gate/up 2048x7168, down 7168x2048, E8M0 bytes uniform in [118,124]) plus
one shared expert, all HBM-resident; bf16 router W ~ N(0,0.02), sigmoid top-8 with
renormalised weights; and the INT8 trunk projection 7168x7168 (int8 uniform [-127,127],
fp32 row scales ~ U(1e-3,1e-2)) on the same bf16 input. A step is one batch of B=16 tokens
x ~ N(0,1) in bf16 through the INT8 projection and the MoE layer; B=1 and B=4 are reported
in "batches". Each step uses a different token batch from a rotating pool, so each step
touches ~110 different experts (~2.6 GB): inputs larger than L2.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
  python bench.py --workload prefill [--steps K] [--warmup W]   (config[2], one line)
  python bench.py --workload streamed [--steps K] [--warmup W]  (config[4], one line)
  torchrun ... bench.py --workload ep --gpus N                   (config[3], one line)
  python bench.py --workload expert [--steps K] [--warmup W]    (config[0], one line)
  python bench.py --workload latent [--steps K] [--warmup W]    (K3 latent MoE layer, one line)

N > 1 (torchrun) runs N independent replicas (decode does not shard; scaling "weak").
The same line carries, under "ep", BASELINE config[3] on the same N GPUs: the expert-parallel
MoE prefill of 16384 tokens with the 384 experts sharded 384/N per GPU (scaling "strong"),
timed as the max over ranks, with its NVLink bytes, per-stage times and a parity check after
the timed region (64 tokens per rank against the single-GPU layer over the same weights, and
8 tokens on rank 0 against the reference's own CPU path). --no-ep leaves it out.
--impl reference times the reference's own CPU kernels (oracle/_ref, built from its
sources) on the same workload with every host core (also under torchrun, which exports
OMP_NUM_THREADS=1).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

H, I, E, K = 7168, 2048, 384, 8
METRIC = "MXFP4 MoE-layer tokens/s"
UNIT = "tokens/s"
WORKLOAD = "config[1] MoE layer decode: B=16 bf16 tokens, 384 HBM-resident MXFP4 experts " \
           "(7168->2048->7168) + 1 shared, bf16 sigmoid top-8 router, INT8 7168x7168 trunk"


class CopyPipe:
    """The end-to-end loop of a serving process: every step's inputs go host -> device on an
    upload stream and its outputs device -> host on a download stream, with two sets of
    device buffers, so step i's copies overlap the compute of steps i-1 and i+1. All copies
    of the timed steps are inside the timed region (finish() joins the download stream).
    compute(i, dev_in, dev_out) enqueues step i's work on the current stream."""

    def __init__(self, host_in, dev_in, dev_out, host_out):
        import torch
        self.host_in, self.dev_in, self.dev_out, self.host_out = host_in, dev_in, dev_out, host_out
        self.up, self.down = torch.cuda.Stream(), torch.cuda.Stream()
        self.ev_in = [torch.cuda.Event() for _ in range(2)]
        self.ev_done = [torch.cuda.Event() for _ in range(2)]
        self.ev_out = [torch.cuda.Event() for _ in range(2)]

    def step(self, i, compute):
        import torch
        main = torch.cuda.current_stream()
        b = i % 2
        self.up.wait_event(self.ev_done[b])          # step i-2 has read this input buffer
        with torch.cuda.stream(self.up):
            for h, d in zip(self.host_in(i), self.dev_in[b]):
                d.copy_(h, non_blocking=True)
            self.ev_in[b].record(self.up)
        main.wait_event(self.ev_in[b])
        main.wait_event(self.ev_out[b])              # step i-2's outputs have left this buffer
        compute(i, self.dev_in[b], self.dev_out[b])
        self.ev_done[b].record(main)
        self.down.wait_event(self.ev_done[b])
        with torch.cuda.stream(self.down):
            for d, h in zip(self.dev_out[b], self.host_out[b]):
                h.copy_(d, non_blocking=True)
            self.ev_out[b].record(self.down)

    def finish(self):
        import torch
        torch.cuda.current_stream().wait_stream(self.down)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d.get("bf16_tflops"), "measured"
    return 6650.0, 1590.0, "fallback"


class Clocks:
    """SM clock and clock-event (throttle) reasons sampled through NVML every 5 ms in a
    background thread while the timed region runs (read-only queries)."""

    HW_SLOWDOWN, SW_POWER_CAP, SW_THERMAL, HW_THERMAL, HW_POWER_BRAKE = 0x8, 0x4, 0x20, 0x40, 0x80

    def __init__(self, cuda_index):
        import threading
        self.samples, self.reasons, self.max_mhz, self.err = [], 0, None, None
        self._stop = threading.Event()
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            self.nv = pynvml
            p = torch.cuda.get_device_properties(cuda_index)
            bus = f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0"
            try:
                self.h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:
                self.h = pynvml.nvmlDeviceGetHandleByIndex(cuda_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            get = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
            self._reasons_fn = get
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        except Exception as e:  # no NVML: report it rather than inventing clocks
            self.err = f"nvml unavailable: {e}"
            self.t = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                self.reasons |= int(self._reasons_fn(self.h))
            except Exception as e:
                self.err = str(e)
            self._stop.wait(0.005)

    def stop(self):
        if self.t is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [self.err]}
        self._stop.set()
        self.t.join(2)
        names = {self.HW_SLOWDOWN: "hw_slowdown", self.HW_THERMAL: "hw_thermal_slowdown",
                 self.SW_THERMAL: "sw_thermal_slowdown", self.SW_POWER_CAP: "sw_power_cap",
                 self.HW_POWER_BRAKE: "hw_power_brake_slowdown"}
        reasons = sorted(n for bit, n in names.items() if self.reasons & bit)
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": reasons + ["no samples"]}
        return {"sm_mhz": float(np.median(self.samples)), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(self.samples)}


def dist_setup(args):
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


# ------------------------------------------------------------------ reference arm
def host_workload(seed, ndistinct=48):
    """Host copy of the config[1] workload for the CPU runs: ndistinct random experts tiled
    over the 384 expert ids, shared expert, fp32 router W (bf16 values), INT8 trunk rows."""
    import __graft_entry__ as ge
    synth = ge.load_package().synth
    g = synth.rng(seed)
    distinct = [synth.expert(g) for _ in range(ndistinct)]
    shared = synth.expert(g)
    wf, _ = synth.router_weights(g, E, H)
    _, _, q8rows = synth.q8_matrix(g, H, H)
    batches = [synth.activations(g, 16, H)[0] for _ in range(4)]
    return distinct, shared, wf, q8rows, batches


def cpu_moe_tokens_per_s(budget_s, steps=None, warmup=0, seed=7):
    """Time the reference's kernels (oracle/_ref) on the config[1] step; returns
    (tokens/s, threads, steps run, seconds)."""
    import ctypes as C
    from oracle import oracle as ora
    R = ora.ref()
    ora.ref_use_all_cores()
    distinct, shared, wf, q8rows, batches = host_workload(seed)
    experts = [distinct[i % len(distinct)] for i in range(E)]
    arr = (ora.Expert6 * E)(*[ora.expert6(e) for e in experts])
    sh = ora.expert6(shared)
    out = np.empty((16, H), np.float32)
    y8 = np.empty(H, np.float32)
    idx = np.empty((16, K), np.int32)
    wt = np.empty((16, K), np.float32)

    def step(b):
        x = batches[b % len(batches)]
        for t in range(16):
            R.k3_matmul_q8(y8, x[t], q8rows, H, H)
        R.refh_moe_layer(out, x, 16, wf, None, arr, C.addressof(sh), H, I, E, K, 1, 1.0, 0,
                         idx, wt)

    for w in range(warmup):
        step(w)
    n, t0 = 0, time.perf_counter()
    while True:
        step(n)
        n += 1
        el = time.perf_counter() - t0
        if (steps is not None and n >= steps) or (steps is None and el >= budget_s):
            break
    return 16 * n / el, R.refh_threads(), n, el


def run_reference(args, ws, rank):
    if rank != 0:
        return
    from oracle import oracle as ora
    if not ora.ref_available():
        print(json.dumps({"impl": "reference", "unavailable":
                          "oracle/_ref/libk3ref.so not built (needs the reference tree)"}))
        return
    tps, threads, n, el = cpu_moe_tokens_per_s(None, steps=args.steps, warmup=args.warmup)
    sample = f"{n} steps of 16 tokens, 48 distinct experts tiled over 384 ids"
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": tps, "unit": UNIT, "n_gpus": args.gpus,
        "steps": n, "warmup": args.warmup, "ms_per_step": 1e3 * el / n, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp64 accumulate (reference CPU)",
        "data": "synthetic", "config": decode_config(args.gpus),
        "cpu_baseline": {"value": tps, "unit": UNIT, "cores": threads, "kind": "reference",
                         "sample": sample},
        "e2e": {"value": tps, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))


# ------------------------------------------------------------------------ our arm
def build_device_workload(k3, dev, seed, distinct=E, path="tc", terms=3):
    """distinct < 384 tiles that many random experts over the 384 ids (profiling runs with
    a smaller device footprint); the default gives every expert id its own weights.
    path "tc": experts generated directly in the pool format of the tensor-core path
    (random nibbles and scale bytes have the same distribution in any byte order);
    path "cuda": the reference's expert run layout for the CUDA-core kernels."""
    import torch
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    if path == "tc":
        lay, run = k3.pool_layout(H, I)
    else:
        lay, run = k3.expert_run_layout(H, I)
    blob = torch.empty((distinct + 1) * run, dtype=torch.uint8, device=dev)
    b2 = blob.view(distinct + 1, run)
    for name, (off, nb) in lay.items():
        seg = b2[:, off:off + nb]
        if name.endswith("_p"):
            seg.copy_(torch.randint(0, 256, seg.shape, generator=g, device=dev, dtype=torch.uint8))
        else:
            seg.copy_(torch.randint(118, 125, seg.shape, generator=g, device=dev, dtype=torch.uint8))
    W = (torch.randn((E, H), generator=g, device=dev) * 0.02).to(torch.bfloat16)
    if path == "tc":
        run_of = torch.tensor([i % distinct for i in range(E)], dtype=torch.int32, device=dev)
        layer = k3.PoolMoeLayer(blob, distinct + 1, run_of, distinct, W, None, H, I, K,
                                terms=terms)
    else:
        qs = k3.experts_from_blob(blob, distinct + 1, H, I)
        layer = k3.MoeLayer([qs[i % distinct] for i in range(E)], qs[distinct], W, None, H, I,
                            K, device=dev)
    wq = torch.randint(-127, 128, (H, H), generator=g, device=dev, dtype=torch.int8)
    ws = torch.rand(H, generator=g, device=dev) * 9e-3 + 1e-3
    return blob, layer, wq, ws


def decode_config(ws):
    """The config of the headline line (both arms print the same dict)."""
    return {"workload": WORKLOAD, "batch": 16, "hidden": H, "inter": I, "experts": E, "topk": K,
            "parallelism": f"replicas x{ws}" if ws > 1 else "single GPU",
            "l2": "inputs larger than L2: each step reads ~110 different experts (~2.6 GB) "
                  "from a rotating pool of 32 token batches"}


def run_ours(args, ws, rank, local):
    """The headline line: config[1] decode (replicas at N > 1) and, under "ep", the config[3]
    expert-parallel layer across the same N GPUs."""
    import gc
    import torch
    import torch.distributed as dist
    import __graft_entry__ as ge
    line = decode_line(args, ws, rank, local)
    gc.collect()
    torch.cuda.empty_cache()
    if not args.no_ep and args.path == "tc":
        k3 = ge.load_package()
        dev = torch.device("cuda", local)
        ep = ep_layer(args, k3, k3.lib(), dev, ws, rank, local, args.ep_steps, 3, parity=not args.no_parity)
        if line is not None:
            line["ep"] = ep
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line))


def decode_line(args, ws, rank, local):
    """config[1]: returns the line on rank 0 (None on the others); leaves the process group
    open."""
    import torch
    import __graft_entry__ as ge
    k3 = ge.load_package()
    L = k3.lib()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    blob, layer, wq, wsc, = build_device_workload(k3, dev, 1234 + rank, args.distinct, args.path,
                                                  args.terms)
    g = torch.Generator(device=dev)
    g.manual_seed(99 + rank)
    B = 16
    NB = 32
    xs = [torch.randn((B, H), generator=g, device=dev).to(torch.bfloat16) for _ in range(NB)]
    host_x = [x.cpu().pin_memory() for x in xs]
    out = torch.empty((B, H), dtype=torch.float32, device=dev)
    y8 = torch.empty((B, H), dtype=torch.float32, device=dev)
    idx_log = [torch.empty((B, K), dtype=torch.int32, device=dev) for _ in range(args.steps)]
    wt = torch.empty((B, K), dtype=torch.float32, device=dev)
    import ctypes as C

    # The trunk projection and the MoE layer read the same tokens and nothing of each other:
    # the trunk runs on a side stream, overlapping the layer's latency-bound router.
    main = torch.cuda.current_stream()
    side = torch.cuda.Stream()
    side_h = C.c_void_p(side.cuda_stream)

    q8_ws = torch.empty(k3.q8_gemv_scratch(B, H, H), dtype=torch.uint8, device=dev)   # caller-owned scratch

    def compute(x, o, y, idx):
        side.wait_stream(main)
        rc = L.k3c_q8_gemv_ws(C.c_void_p(y.data_ptr()), H, C.c_void_p(x.data_ptr()), k3.K3C_BF16, H,
                              B, C.c_void_p(wq.data_ptr()), C.c_void_p(wsc.data_ptr()), H, H, H,
                              C.c_void_p(q8_ws.data_ptr()), q8_ws.numel(), side_h)
        assert rc == 0, L.k3c_last_error()
        layer.decode(x, out=o, idx=idx, wt=wt)
        main.wait_stream(side)

    def step(i, idx=None):
        compute(xs[i % NB], out, y8, idx if idx is not None else idx_log[0])

    pipe = CopyPipe(lambda i: [host_x[i % NB]],
                    [[torch.empty((B, H), dtype=torch.bfloat16, device=dev)] for _ in range(2)],
                    [[torch.empty((B, H), dtype=torch.float32, device=dev) for _ in range(2)] for _ in range(2)],
                    [[torch.empty((B, H), dtype=torch.float32).pin_memory() for _ in range(2)] for _ in range(2)])

    def e2e_compute(i, din, dout):
        compute(din[0], dout[0], dout[1], idx_log[0])

    def barrier():
        torch.cuda.synchronize()
        if ws > 1:
            import torch.distributed as dist
            dist.barrier()
        torch.cuda.synchronize()

    def maxed(v):
        if ws == 1:
            return v
        import torch.distributed as dist
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    for i in range(args.warmup):
        step(i)
    # --- device-resident timed region
    barrier()
    clk = Clocks(local)
    L.k3c_timing_enable(1)
    ms_buf = (C.c_double * 4)()
    n_buf = (C.c_longlong * 4)()
    L.k3c_timing_read(ms_buf, n_buf, 4)          # discard warm-up records
    launches0 = L.k3c_launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        step(args.warmup + i, idx=idx_log[i])
    e1.record()
    torch.cuda.synchronize()
    launches = L.k3c_launch_count() - launches0
    L.k3c_timing_enable(0)
    L.k3c_timing_read(ms_buf, n_buf, 4)
    clocks = clk.stop()
    dt = maxed(e0.elapsed_time(e1) / 1e3)
    barrier()
    # unique experts per step (the algorithmic bytes of the expert stage)
    uniq = [int(torch.unique(t).numel()) for t in idx_log]
    run_bytes = k3.expert_run_layout(H, I)[1]
    expert_bytes = sum((u + 1) * run_bytes for u in uniq)
    exp_ms = ms_buf[0]
    achieved = expert_bytes / (exp_ms / 1e3) / 1e9 if exp_ms > 0 else None
    hbm_peak, _, peak_kind = peaks()
    router_bytes = E * H * 2
    layer_bytes = expert_bytes + args.steps * (router_bytes + H * H + 4 * H)
    # --- end-to-end timed region: pinned host x in, host results out, every step (copies on
    # their own streams, overlapping the neighbouring steps' compute)
    for i in range(3):
        pipe.step(i, e2e_compute)
    pipe.finish()
    barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for i in range(args.steps):
        pipe.step(args.warmup + i, e2e_compute)
    pipe.finish()
    f1.record()
    torch.cuda.synchronize()
    dte = maxed(f0.elapsed_time(f1) / 1e3)
    # --- B = 1 and B = 4 (same layer, device-resident)
    batches = {}
    for b in (1, 4):
        xb = [x[:b].contiguous() for x in xs]
        ob = torch.empty((b, H), dtype=torch.float32, device=dev)
        ib = torch.empty((b, K), dtype=torch.int32, device=dev)
        wb = torch.empty((b, K), dtype=torch.float32, device=dev)
        for i in range(args.warmup):
            layer.decode(xb[i % NB], out=ob, idx=ib, wt=wb)
        barrier()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record()
        for i in range(args.steps):
            layer.decode(xb[(args.warmup + i) % NB], out=ob, idx=ib, wt=wb)
        c1.record()
        torch.cuda.synchronize()
        t_launch = maxed(c0.elapsed_time(c1) / 1e3)
        # A serving loop replays a captured step: one CUDA graph per input batch holds the
        # layer's launches, so a ~0.1 ms step is not bounded by the host's per-launch cost.
        graphs = []
        cap = torch.cuda.Stream()
        cap.wait_stream(torch.cuda.current_stream())
        for i in range(NB):
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=cap):
                layer.decode(xb[i], out=ob, idx=ib, wt=wb)
            graphs.append(gr)
        for i in range(3):
            graphs[i].replay()
        barrier()
        c0.record()
        for i in range(args.steps):
            graphs[(args.warmup + i) % NB].replay()
        c1.record()
        torch.cuda.synchronize()
        tb = maxed(c0.elapsed_time(c1) / 1e3)
        del graphs
        # the distinct experts each of these steps streams (its routed ids + the shared expert)
        nu = []
        for i in range(args.steps):
            layer.decode(xb[(args.warmup + i) % NB], out=ob, idx=ib, wt=wb)
            nu.append(len(set(ib.cpu().numpy().ravel().tolist())) + 1)
        step_bytes = float(np.mean(nu)) * run_bytes
        batches[f"B{b}"] = {"tokens_per_s": ws * b * args.steps / tb, "ms_per_step": 1e3 * tb / args.steps,
                            "ms_per_step_stream_launches": 1e3 * t_launch / args.steps,
                            "distinct_experts_per_step": float(np.mean(nu)),
                            "step_hbm_frac": step_bytes / (tb / args.steps) / 1e9 / hbm_peak,
                            "how": "distinct experts' bytes / whole-step time / measured HBM peak; steps replayed "
                                   "from CUDA graphs of the layer call (one per input batch); "
                                   "ms_per_step_stream_launches: the same steps launched from the host"}
    batches["config0_expert"] = expert_ffn_probe(k3, L, dev, rank, hbm_peak)
    batches["q8_alone"] = q8_probe(k3, L, dev, wq, wsc, q8_ws, hbm_peak)
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()
    if rank != 0:
        return None
    cpu = None
    if ws == 1 and not args.no_cpu:
        from oracle import oracle as ora
        if ora.ref_available():
            tps, threads, n, el = cpu_moe_tokens_per_s(args.cpu_seconds)
            cpu = {"value": tps, "unit": UNIT, "cores": threads, "kind": "reference",
                   "sample": f"{n} steps of 16 tokens ({el:.1f} s), 48 distinct experts tiled over 384 ids"}
    line = {
        "metric": METRIC, "value": ws * B * args.steps / dt, "unit": UNIT, "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * dt / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": (f"mxfp4 x e4m3 (activations as {args.terms} E4M3 terms), fp32 accumulate "
                  "(tcgen05 kind::mxf8f6f4)") if args.path == "tc" else
                 "fp32 (MXFP4 weights, bf16 inputs widened exactly, fp32 accumulate)",
        "data": "synthetic",
        "config": decode_config(ws),
        "impl": {"path": args.path, "terms": args.terms if args.path == "tc" else None},
        "decode_hbm_gbs": layer_bytes / dt / 1e9,
        "unique_experts_per_step": float(np.mean(uniq)),
        "batches": batches,
        "stages_ms_per_step": {name: ms_buf[j] / args.steps
                               for j, name in enumerate(("experts", "router", "combine", "q8"))},
        "q8_hbm_gbs": (H * H + 4 * H) * args.steps / (ms_buf[3] / 1e3) / 1e9 if ms_buf[3] > 0 else None,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                     "frac": (achieved / hbm_peak) if achieved else None,
                     "traffic": (DEC_TRAFFIC_RATIO * expert_bytes / args.steps) if args.path == "tc" else None,
                     "traffic_unit": "bytes per step (both expert kernels)",
                     "algorithmic_bytes_per_step": expert_bytes / args.steps,
                     "traffic_source": f"ncu dram__bytes_read.sum + dram__bytes_write.sum of the k_tc_moe launches of "
                                       f"3 full-size steps = {DEC_TRAFFIC_RATIO:.3f} x their algorithmic bytes",
                     "kernel": "expert stage (tcgen05 gate/up+act and down kernels, k_tc_moe)",
                     "peak_kind": peak_kind},
        "cpu_baseline": cpu,
        "e2e": {"value": ws * B * args.steps / dte, "unit": UNIT,
                "h2d_bytes_per_step": B * H * 2, "d2h_bytes_per_step": 2 * B * H * 4,
                "copies": "pinned host buffers; uploads and downloads on their own streams, two device buffer sets"},
        "gpu_launches": int(launches),
        "clocks": clocks,
    }
    return line


# DRAM bytes the two k_tc_moe launches of a config[1] step move, over the step's algorithmic
# bytes ((unique routed experts + shared) x 23,396,352): measured with ncu (dram__bytes_read.sum +
# dram__bytes_write.sum, one pass, full-size workload, 3 steps: 8.197 GB for 7.885 GB). The extra
# 4% are the activation terms, scale atoms and requantised intermediate rows.
DEC_TRAFFIC_RATIO = 1.040

# ------------------------------------------------------------------ prefill (config[2])
PF_T = 4096
PF_WORKLOAD = "config[2] MoE layer prefill: 4096 bf16 tokens, 384 HBM-resident MXFP4 experts " \
              "(7168->2048->7168) + 1 shared, bf16 sigmoid top-8 router with a Zipf(1.1) selection bias"


def run_prefill(args, ws, rank, local):
    """One step = the whole layer over 4096 tokens through k3c_moe_prefill_tc (router,
    expert-sorted grouped tcgen05 GEMMs, combine). Routing popularity follows Zipf(1.1) over
    the expert ids by a selection bias fitted on a separate sample of tokens."""
    import ctypes as C
    import torch
    import __graft_entry__ as ge
    k3 = ge.load_package()
    L = k3.lib()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    D = args.distinct                                    # < 384 only for small profiling runs
    blob, layer0, _, _ = build_device_workload(k3, dev, 1234 + rank, D, "tc", 2)
    W = layer0.router_w
    g = torch.Generator(device=dev)
    g.manual_seed(77 + rank)
    sample = torch.randn((2048, H), generator=g, device=dev).to(torch.bfloat16)
    scores = torch.sigmoid(sample.float() @ W.float().T)
    bias = k3.synth.zipf_fit_bias(scores, s=1.1, topk=K, iters=600)
    layer = k3.PoolMoeLayer(blob, D + 1, layer0.run_of, D, W, bias, H, I, K, terms=2)
    NB = 2
    xs = [torch.randn((PF_T, H), generator=g, device=dev).to(torch.bfloat16) for _ in range(NB)]
    host_x = xs[0].cpu().pin_memory()
    out = torch.empty((PF_T, H), dtype=torch.float32, device=dev)
    idx = torch.empty((PF_T, K), dtype=torch.int32, device=dev)
    wt = torch.empty((PF_T, K), dtype=torch.float32, device=dev)
    h_out = torch.empty((PF_T, H), dtype=torch.float32).pin_memory()
    x_dev = torch.empty((PF_T, H), dtype=torch.bfloat16, device=dev)
    for i in range(args.warmup):
        layer.prefill(xs[i % NB], out=out, idx=idx, wt=wt)
    torch.cuda.synchronize()
    # routing statistics of the measured batches
    uniq, counts = [], torch.zeros(E, dtype=torch.int64, device=dev)
    for b in range(NB):
        layer.prefill(xs[b], out=out, idx=idx, wt=wt)
        uniq.append(int(torch.unique(idx).numel()))
        counts += torch.bincount(idx.reshape(-1).long(), minlength=E)
    pop = (counts.double() / counts.sum()).sort(descending=True).values
    target = k3.synth.zipf_topk_marginal(E, 1.1, K, device=dev)
    clk = Clocks(local)
    L.k3c_timing_enable(1)
    ms_buf = (C.c_double * 4)()
    n_buf = (C.c_longlong * 4)()
    L.k3c_timing_read(ms_buf, n_buf, 4)
    launches0 = L.k3c_launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for i in range(args.steps):
        layer.prefill(xs[i % NB], out=out, idx=idx, wt=wt)
    e1.record()
    torch.cuda.synchronize()
    launches = L.k3c_launch_count() - launches0
    L.k3c_timing_enable(0)
    L.k3c_timing_read(ms_buf, n_buf, 4)
    clocks = clk.stop()
    dt = e0.elapsed_time(e1) / 1e3
    # end to end: pinned host tokens in, host outputs back, every step (copies on their own
    # streams, overlapping the neighbouring steps' compute)
    pipe = CopyPipe(lambda i: [host_x],
                    [[x_dev], [torch.empty_like(x_dev)]],
                    [[out], [torch.empty_like(out)]],
                    [[h_out], [torch.empty_like(h_out).pin_memory()]])

    def e2e_compute(i, din, dout):
        layer.prefill(din[0], out=dout[0], idx=idx, wt=wt)

    for i in range(2):
        pipe.step(i, e2e_compute)
    pipe.finish()
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for i in range(args.steps):
        pipe.step(i, e2e_compute)
    pipe.finish()
    f1.record()
    torch.cuda.synchronize()
    dte = f0.elapsed_time(f1) / 1e3
    if rank != 0:
        return
    run_bytes = k3.pool_run_bytes(H, I)
    flop = (PF_T * K + PF_T) * 2 * 3 * I * H          # routed pairs + shared expert
    exp_s = ms_buf[0] / 1e3 / args.steps
    wbytes = (np.mean(uniq) + 1) * run_bytes
    hbm, bf16, kind = peaks()
    fp4_nominal, fp8_nominal = 9000.0, 4500.0       # dense TFLOP/s, B200 datasheet
    tflops = flop / exp_s / 1e12 if exp_s > 0 else None
    bound_s = max(flop / (fp8_nominal * 1e12), wbytes / (hbm * 1e9))
    print(json.dumps({
        "metric": METRIC, "value": PF_T * args.steps / dt, "unit": UNIT, "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * dt / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "mxfp4 x e4m3 (activations as 2 E4M3 terms), fp32 accumulate (tcgen05 kind::mxf8f6f4)",
        "data": "synthetic",
        "config": {"workload": PF_WORKLOAD, "tokens": PF_T, "hidden": H, "inter": I, "experts": E,
                   "topk": K, "parallelism": "single GPU",
                   "l2": "inputs larger than L2: ~9 GB of expert weights per step",
                   "distinct_expert_weights": D},
        "routing": {"unique_experts": float(np.mean(uniq)), "top1_share": float(pop[0]),
                    "top10_share": float(pop[:10].sum()),
                    "zipf_topk_target": {"top1": float(target[0]), "top10": float(target[:10].sum())},
                    "l1_to_target": float((pop - target).abs().sum())},
        "stages_ms_per_step": {name: ms_buf[j] / args.steps
                               for j, name in enumerate(("experts", "router", "combine", "q8"))},
        "roofline": {"bound": "tensor", "kernel": "expert stage (GU + D grouped tcgen05 kernels)",
                     "achieved": tflops, "unit": "TFLOP/s",
                     "useful_flop_per_step": flop, "weight_bytes_per_step": wbytes,
                     "frac_of_fp4_dense_nominal": tflops / fp4_nominal if tflops else None,
                     "frac_of_fp8_dense_nominal": tflops / fp8_nominal if tflops else None,
                     "frac_of_bf16_measured": tflops / bf16 if (tflops and bf16) else None,
                     "hbm_gbs": wbytes / exp_s / 1e9 if exp_s > 0 else None,
                     "expert_stage_vs_bound": bound_s / exp_s if exp_s > 0 else None,
                     "note": "activations run as 2 E4M3 terms at the FP8 MMA rate: the issued "
                             "MMA work is 2x the useful FLOP"},
        "e2e": {"value": PF_T * args.steps / dte, "unit": UNIT,
                "copies": "pinned host buffers; uploads and downloads on their own streams, two device buffer sets",
                "h2d_bytes_per_step": PF_T * H * 2,
                "d2h_bytes_per_step": PF_T * H * 4},
        "gpu_launches": int(launches),
        "clocks": clocks,
    }))


# ------------------------------------------------------------------ streamed (config[4])
ST_LAYERS = 16
ST_WORKLOAD = "config[4] streamed-expert decode: 16-layer stack of config[1] MoE layers, 1 token per " \
              "step, seeded top-8 routing reusing 4 of the previous step's experts per layer, HBM " \
              "expert pool = 25% of the 143.7 GB of expert bytes, the rest in pinned host memory"


def streamed_routing(seed, steps, layers=ST_LAYERS, n_experts=E, topk=K, reuse=4):
    """Per (step, layer): topk distinct experts, `reuse` of them drawn from the previous
    step's set of that layer, the rest new; weights positive and normalised."""
    g = np.random.default_rng(seed)
    prev = [g.choice(n_experts, topk, replace=False) for _ in range(layers)]
    idx = np.empty((steps, layers, topk), np.int32)
    wt = np.empty((steps, layers, topk), np.float32)
    for s in range(steps):
        for l in range(layers):
            keep = g.choice(prev[l], reuse, replace=False)
            pool_ids = np.setdiff1d(np.arange(n_experts), keep)
            new = g.choice(pool_ids, topk - reuse, replace=False)
            ids = np.concatenate([keep, new])
            g.shuffle(ids)
            idx[s, l] = ids
            w = g.random(topk).astype(np.float32) + 0.05
            wt[s, l] = w / w.sum()
            prev[l] = ids
    return idx, wt


def run_streamed(args, ws, rank, local):
    """One step = one token through 16 MoE layers whose experts come from an HBM pool of
    25% of the stack's expert bytes; misses are copied from pinned host memory on the pool's
    copy stream (k3c_pool_*), then the layer runs on the tensor-core decode path."""
    import ctypes as C
    import torch
    import __graft_entry__ as ge
    k3 = ge.load_package()
    L = k3.lib()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    run_bytes = k3.pool_run_bytes(H, I)
    n_keys = ST_LAYERS * (E + 1)                            # expert E of a layer: its shared expert
    total_bytes = ST_LAYERS * E * run_bytes
    n_slots = int(0.25 * total_bytes // run_bytes) + ST_LAYERS
    # pinned host images: 32 distinct pool-format runs tiled over the keys (every miss still
    # moves a whole run over PCIe)
    D = 32
    g = torch.Generator(device=dev)
    g.manual_seed(4321)
    lay, _ = k3.pool_layout(H, I)
    images = []
    tmp = torch.empty(run_bytes, dtype=torch.uint8, device=dev)
    for d in range(D):
        for name, (off, nb) in lay.items():
            seg = tmp[off:off + nb]
            if name.endswith("_p"):
                seg.copy_(torch.randint(0, 256, (nb,), generator=g, device=dev, dtype=torch.uint8))
            else:
                seg.copy_(torch.randint(118, 125, (nb,), generator=g, device=dev, dtype=torch.uint8))
        images.append(tmp.cpu().pin_memory())

    def src(layer, expert):
        return images[(layer * (E + 1) + expert) % D]

    pool = k3.ExpertPool(H, I, ST_LAYERS, E + 1, n_slots, src)
    W = (torch.randn((E, H), generator=g, device=dev) * 0.02).to(torch.bfloat16)
    shared_slots = [pool.pin(l, E) for l in range(ST_LAYERS)]
    tables = [pool.run_table() for _ in range(ST_LAYERS)]
    layers = [pool.layer(W, H, I, K, E, tables[l], shared_slot=shared_slots[l], terms=3)
              for l in range(ST_LAYERS)]
    total_steps = args.warmup + args.steps
    idx_h, wt_h = streamed_routing(2024 + rank, total_steps)
    idx_d = torch.from_numpy(idx_h).to(dev)
    wt_d = torch.from_numpy(wt_h).to(dev)
    x0 = torch.randn((1, H), generator=g, device=dev).to(torch.bfloat16)
    torch.cuda.synchronize()

    def step(s):
        x = x0
        for l in range(ST_LAYERS):
            ids = idx_h[s, l]
            pool.acquire(l, ids, run_of=tables[l])
            out = layers[l].decode_routed(x, idx_d[s, l:l + 1], wt_d[s, l:l + 1])
            pool.release(l, ids)
            x = out.to(torch.bfloat16)
        return out

    for s in range(args.warmup):
        step(s)
    torch.cuda.synchronize()
    st0 = pool.stats()
    clk = Clocks(local)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = L.k3c_launch_count()
    t0 = time.perf_counter()
    e0.record()
    for s in range(args.warmup, total_steps):
        out = step(s)
    h_out = out.cpu()                                      # the step's result read back
    e1.record()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    clocks = clk.stop()
    dt = e0.elapsed_time(e1) / 1e3
    launches = L.k3c_launch_count() - launches0
    st1 = pool.stats()
    req = (st1["hits"] - st0["hits"]) + (st1["misses"] - st0["misses"])
    hits = st1["hits"] - st0["hits"]
    h2d = st1["bytes_h2d"] - st0["bytes_h2d"]
    hbm_bytes = args.steps * ST_LAYERS * (K + 1) * run_bytes
    hbm, _, kind = peaks()
    pool.close()
    # the link's own ceiling: one large pinned host -> device copy
    big = torch.empty(1 << 30, dtype=torch.uint8).pin_memory()
    dbig = torch.empty(1 << 30, dtype=torch.uint8, device=dev)
    dbig.copy_(big, non_blocking=True)
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c0.record()
    for _ in range(4):
        dbig.copy_(big, non_blocking=True)
    c1.record()
    torch.cuda.synchronize()
    pcie_peak = 4 * (1 << 30) / (c0.elapsed_time(c1) / 1e3) / 1e9
    del big, dbig
    if rank != 0:
        return
    print(json.dumps({
        "metric": METRIC, "value": args.steps / dt, "unit": UNIT, "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * dt / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": "mxfp4 x e4m3 (activations as 3 E4M3 terms), fp32 accumulate (tcgen05 kind::mxf8f6f4)",
        "data": "synthetic",
        "config": {"workload": ST_WORKLOAD, "layers": ST_LAYERS, "hidden": H, "inter": I, "experts": E,
                   "topk": K, "pool_slots": n_slots, "pool_gb": n_slots * run_bytes / 1e9,
                   "expert_bytes_gb": total_bytes / 1e9, "host_images": D},
        "cache": {"requests": req, "hit_rate": hits / req if req else None,
                  "misses_per_step": (req - hits) / args.steps,
                  "evictions": st1["evictions"] - st0["evictions"]},
        "pcie_h2d_gbs": h2d / dt / 1e9, "h2d_bytes_per_step": h2d / args.steps,
        "roofline": {"bound": "pcie", "achieved": h2d / dt / 1e9, "peak": pcie_peak, "unit": "GB/s",
                     "frac": h2d / dt / 1e9 / pcie_peak, "peak_kind": "measured in this run: 1 GiB pinned copies"},
        "hbm_expert_gbs": hbm_bytes / dt / 1e9, "hbm_peak_gbs": hbm, "peak_kind": kind,
        "e2e": {"value": args.steps / wall, "unit": UNIT, "h2d_bytes_per_step": h2d / args.steps,
                "d2h_bytes_per_step": H * 4 / args.steps},
        "gpu_launches": int(launches),
        "clocks": clocks,
    }))


# ------------------------------------------------------------------ single expert (config[0])
EX_WORKLOAD = "config[0] single MXFP4 expert SwiGLU FFN, 1 fp32 token per step (7168->2048->7168, " \
              "E2M1 codes uniform, E8M0 uniform in [118,124]), fp32 accumulate"


def expert_ffn_setup(k3, L, dev, seed, NX=16):
    """NX random experts in the reference's run layout (NX x 23.4 MB, more than L2 for NX=16),
    NX fp32 tokens and a step function: one token through expert i % NX (k3c_expert_ffn)."""
    import ctypes as C
    import torch
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    lay, run = k3.expert_run_layout(H, I)
    blob = torch.empty(NX * run, dtype=torch.uint8, device=dev)
    b2 = blob.view(NX, run)
    for name, (off, nb) in lay.items():
        seg = b2[:, off:off + nb]
        if name.endswith("_p"):
            seg.copy_(torch.randint(0, 256, seg.shape, generator=g, device=dev, dtype=torch.uint8))
        else:
            seg.copy_(torch.randint(118, 125, seg.shape, generator=g, device=dev, dtype=torch.uint8))
    qs = k3.experts_from_blob(blob, NX, H, I)
    xs = torch.randn((NX, H), generator=g, device=dev)
    y = torch.empty((1, H), dtype=torch.float32, device=dev)
    nbytes = L.k3c_expert_ffn_scratch(1, H, I)
    scratch = torch.empty(nbytes, dtype=torch.uint8, device=dev)

    def step(i, x=None):
        q = qs[i % NX]
        xx = xs[i % NX:i % NX + 1] if x is None else x
        rc = L.k3c_expert_ffn(C.c_void_p(y.data_ptr()), C.c_void_p(xx.data_ptr()), 1, C.byref(q), H, I, 0,
                              C.c_void_p(scratch.data_ptr()), nbytes, k3._stream())
        assert rc == 0, L.k3c_last_error()

    return step, run, xs, y, (blob, qs, scratch)


def q8_probe(k3, L, dev, wq, wsc, ws_buf, hbm_peak, copies=16, reps=20):
    """The INT8 trunk projection timed alone (in the step it shares the GPU with the layer's
    router and experts): 16 bf16 tokens through 7168 x 7168, rotated over `copies` weight
    matrices (822 MB, more than L2), calls replayed from a CUDA graph."""
    import ctypes as C
    import torch
    B = 16
    ws_ = [wq] + [wq.clone() for _ in range(copies - 1)]
    x = torch.randn((B, H), device=dev).to(torch.bfloat16)
    y = torch.empty((B, H), dtype=torch.float32, device=dev)

    def call(w):
        rc = L.k3c_q8_gemv_ws(C.c_void_p(y.data_ptr()), H, C.c_void_p(x.data_ptr()), k3.K3C_BF16, H, B,
                              C.c_void_p(w.data_ptr()), C.c_void_p(wsc.data_ptr()), H, H, H,
                              C.c_void_p(ws_buf.data_ptr()), ws_buf.numel(), k3._stream())
        assert rc == 0, L.k3c_last_error()

    for w in ws_:
        call(w)
    torch.cuda.synchronize()
    gr = torch.cuda.CUDAGraph()
    cap = torch.cuda.Stream()
    cap.wait_stream(torch.cuda.current_stream())
    with torch.cuda.graph(gr, stream=cap):
        for w in ws_:
            call(w)
    for _ in range(3):
        gr.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        gr.replay()
    e1.record()
    torch.cuda.synchronize()
    dt = e0.elapsed_time(e1) / 1e3 / (reps * copies)
    del gr, ws_
    nbytes = H * H + 4 * H
    return {"us_per_call": 1e6 * dt, "hbm_gbs": nbytes / dt / 1e9, "hbm_frac": nbytes / dt / 1e9 / hbm_peak,
            "how": "k3c_q8_gemv_ws alone, 16 bf16 tokens x 7168x7168 int8, 16 weight copies rotated (> L2), "
                   "graph replay"}


def expert_ffn_probe(k3, L, dev, rank, hbm_peak, steps=160):
    """config[0] beside the headline: one fp32 token through one expert, 16 experts rotated,
    the calls replayed from a CUDA graph (the --workload expert measurement, shorter)."""
    import torch
    step, run, _, _, keep = expert_ffn_setup(k3, L, dev, 4242 + rank)
    for i in range(16):
        step(i)
    torch.cuda.synchronize()
    gr = torch.cuda.CUDAGraph()
    cap = torch.cuda.Stream()
    with torch.cuda.graph(gr, stream=cap):
        for i in range(16):
            step(i)
    for _ in range(3):
        gr.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps // 16):
        gr.replay()
    e1.record()
    torch.cuda.synchronize()
    dt = e0.elapsed_time(e1) / 1e3 / (16 * (steps // 16))
    del gr, keep
    return {"us_per_token": 1e6 * dt, "hbm_frac": run / dt / 1e9 / hbm_peak,
            "how": "k3c_expert_ffn, one fp32 token, 23.4 MB per token, graph replay (as --workload expert)"}


def run_expert(args, ws, rank, local):
    """One step = one fp32 token through one expert (k3c_expert_ffn, the fp32-activation
    CUDA-core path the 1e-5 tolerance calls for), rotating over 16 experts (374 MB, more than
    L2) so every step streams its 23.4 MB from HBM."""
    import ctypes as C
    import torch
    import __graft_entry__ as ge
    k3 = ge.load_package()
    L = k3.lib()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    NX = 16
    step, run, xs, y, _keep = expert_ffn_setup(k3, L, dev, 4242 + rank, NX)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    # Device throughput: the K steps replayed from CUDA graphs (one per rotation of the 16
    # experts, plus one for the K mod 16 remainder), so the host's per-call cost does not
    # starve a ~4 us step. The end-to-end figure below calls the API directly.
    reps, rem = divmod(args.steps, NX)
    graphs, per = [], []
    cap = torch.cuda.Stream()
    for n in ([NX] if reps else []) + ([rem] if rem else []):
        gr = torch.cuda.CUDAGraph()
        l0 = L.k3c_launch_count()
        with torch.cuda.graph(gr, stream=cap):
            for i in range(n):
                step(i)
        graphs.append(gr)
        per.append(L.k3c_launch_count() - l0)
    for _ in range(3):
        graphs[0].replay()
    torch.cuda.synchronize()
    clk = Clocks(local)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        graphs[0].replay()
    if rem:
        graphs[-1].replay()
    e1.record()
    torch.cuda.synchronize()
    clocks = clk.stop()
    launches = per[0] * reps + (per[-1] if rem else 0)
    dt = e0.elapsed_time(e1) / 1e3
    # end to end: the token from pinned host memory, the output back, every step
    hx = xs.cpu().pin_memory()
    hy = torch.empty((1, H), dtype=torch.float32).pin_memory()
    xd = torch.empty((1, H), dtype=torch.float32, device=dev)
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for i in range(args.steps):
        xd.copy_(hx[i % NX:i % NX + 1], non_blocking=True)
        step(i, xd)
        hy.copy_(y, non_blocking=True)
    f1.record()
    torch.cuda.synchronize()
    dte = f0.elapsed_time(f1) / 1e3
    if rank != 0:
        return
    hbm, _, kind = peaks()
    achieved = args.steps * run / dt / 1e9
    print(json.dumps({
        "metric": "MXFP4 expert tokens/s", "value": args.steps / dt, "unit": UNIT, "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * dt / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp32 (MXFP4 weights, fp32 activations, fp32 accumulate)", "data": "synthetic",
        "config": {"workload": EX_WORKLOAD, "hidden": H, "inter": I,
                   "l2": "16 experts rotated (374 MB) > L2",
                   "timing": "K steps replayed from CUDA graphs of the k3c_expert_ffn calls; e2e calls the API directly"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": achieved / hbm, "kernel": "gate/up + down CUDA-core GEMVs (k3c_expert_ffn)",
                     "bytes_per_token": run, "peak_kind": kind},
        "e2e": {"value": args.steps / dte, "unit": UNIT, "h2d_bytes_per_step": H * 4, "d2h_bytes_per_step": H * 4},
        "gpu_launches": int(launches),
        "clocks": clocks,
    }))


# ------------------------------------------------------------------ K3 latent MoE layer
LH, LL, LI, LE, LK, LS = 7168, 3584, 3072, 896, 16, 2
LAT_WORKLOAD = ("K3 latent MoE layer decode: B=16 fp32 tokens, full-width fp32 sigmoid top-16 router over "
                "896 HBM-resident MXFP4 experts at the latent width (3584->3072->3584, SiTU), bf16 trunk "
                "down 7168->3584 / up 3584->7168, aggregate RMSNorm, full-width shared expert "
                "(7168->6144->7168, bf16), the K3 model's shapes")


def host_latent_workload(seed, ndistinct=8):
    """Host copy of the latent workload for the CPU runs: ndistinct random experts tiled over
    the 896 ids, bf16 trunk, fp32 router."""
    import __graft_entry__ as ge
    synth = ge.load_package().synth
    g = synth.rng(seed)
    distinct = [synth.expert(g, LL, LI) for _ in range(ndistinct)]
    SI = LI * LS

    def trunk(o, i):
        return synth.bf16_bits(g.standard_normal((o, i), dtype=np.float32) * np.float32(1 / np.sqrt(i)))

    layer = dict(router_w=synth.bf16_to_f32(synth.bf16_bits(
                     g.standard_normal((LE, LH), dtype=np.float32) * np.float32(0.02))),
                 router_bias=None, experts=[distinct[i % ndistinct] for i in range(LE)],
                 latent_norm=np.ones(LL, np.float32), down=trunk(LL, LH), up=trunk(LH, LL),
                 sh1=trunk(SI, LH), sh3=trunk(SI, LH), sh2=trunk(LH, SI), wdt=1, hidden=LH, latent=LL,
                 inter=LI, n_shared=LS, n_experts=LE, topk=LK, renorm=1, latent_norm_on=1,
                 routed_scale=1.0, rms_eps=1e-5, situ_b1=4.0, situ_b2=25.0)
    xs = [g.standard_normal((16, LH), dtype=np.float32) for _ in range(2)]
    return layer, xs


def cpu_latent_tokens_per_s(budget_s, steps=None, warmup=0, seed=8):
    """The reference's own k3_moe (oracle/_ref) on the latent workload, one token at a time as
    it runs; returns (tokens/s, threads, tokens run, seconds)."""
    from oracle import oracle as ora
    layer, xs = host_latent_workload(seed)
    for w in range(warmup):
        ora.moe_latent(xs[0][w % 16:w % 16 + 1], layer, use_ref=True)
    n, t0 = 0, time.perf_counter()
    while True:
        ora.moe_latent(xs[(n // 16) % 2][n % 16:n % 16 + 1], layer, use_ref=True)
        n += 1
        el = time.perf_counter() - t0
        if (steps is not None and n >= steps) or (steps is None and el >= budget_s):
            break
    return n / el, ora.ref().refh_threads(), n, el


def run_latent(args, ws, rank, local):
    """One step = 16 fp32 tokens through k3c_moe_latent_decode (router, trunk down, routed
    experts at the latent width on the tensor-core path, aggregate RMSNorm, trunk up, shared
    expert), rotating over 32 token batches: each step reads ~230 distinct experts (~4 GB)."""
    import ctypes as C
    import torch
    import __graft_entry__ as ge
    k3 = ge.load_package()
    L = k3.lib()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    g = torch.Generator(device=dev)
    g.manual_seed(5151 + rank)
    # --distinct D < 384 (profiling only): D distinct expert runs tiled over the 896 ids
    ND = args.distinct if args.distinct < E else LE
    lay, run = k3.pool_layout(LL, LI)
    arena = torch.empty(ND * run, dtype=torch.uint8, device=dev)
    a2 = arena.view(ND, run)
    for name, (off, nb) in lay.items():
        seg = a2[:, off:off + nb]
        if name.endswith("_p"):
            seg.copy_(torch.randint(0, 256, seg.shape, generator=g, device=dev, dtype=torch.uint8))
        else:
            seg.copy_(torch.randint(118, 125, seg.shape, generator=g, device=dev, dtype=torch.uint8))
    SI = LI * LS

    def trunk(o, i):
        return (torch.randn((o, i), generator=g, device=dev) / float(np.sqrt(i))).to(torch.bfloat16)

    router = (torch.randn((LE, LH), generator=g, device=dev) * 0.02).to(torch.bfloat16).float()
    down, up, sh1, sh3, sh2 = trunk(LL, LH), trunk(LH, LL), trunk(SI, LH), trunk(SI, LH), trunk(LH, SI)
    norm = torch.ones(LL, dtype=torch.float32, device=dev)
    run_of = torch.arange(LE, dtype=torch.int32, device=dev) % ND
    lat = k3.LatentMoeLayer(arena, ND, run_of, router, None, down, up, sh1, sh3, sh2, norm, k3.WBF16,
                            LH, LL, LI, LS, LK, terms=args.terms)
    B = args.batch
    NB = 32 if B <= 32 else 4          # rotating token batches (each larger than L2 above 32)
    xs = [torch.randn((B, LH), generator=g, device=dev) for _ in range(NB)]
    out = torch.empty((B, LH), dtype=torch.float32, device=dev)
    idx_log = [torch.empty((B, LK), dtype=torch.int32, device=dev) for _ in range(args.steps)]
    wt = torch.empty((B, LK), dtype=torch.float32, device=dev)
    for i in range(args.warmup):
        lat.decode(xs[i % NB], out=out, idx=idx_log[0], wt=wt)
    torch.cuda.synchronize()
    clk = Clocks(local)
    L.k3c_timing_enable(1)
    ms_buf, n_buf = (C.c_double * 4)(), (C.c_longlong * 4)()
    L.k3c_timing_read(ms_buf, n_buf, 4)
    l0 = L.k3c_launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        lat.decode(xs[(args.warmup + i) % NB], out=out, idx=idx_log[i], wt=wt)
    e1.record()
    torch.cuda.synchronize()
    launches = L.k3c_launch_count() - l0
    L.k3c_timing_enable(0)
    L.k3c_timing_read(ms_buf, n_buf, 4)
    clocks = clk.stop()
    dt = e0.elapsed_time(e1) / 1e3
    # end to end: pinned host tokens in, outputs back, every step (copies on their own streams)
    hx = [x.cpu().pin_memory() for x in xs]
    pipe = CopyPipe(lambda i: [hx[i % NB]],
                    [[torch.empty((B, LH), dtype=torch.float32, device=dev)] for _ in range(2)],
                    [[torch.empty((B, LH), dtype=torch.float32, device=dev)] for _ in range(2)],
                    [[torch.empty((B, LH), dtype=torch.float32).pin_memory()] for _ in range(2)])

    def e2e_compute(i, din, dout):
        lat.decode(din[0], out=dout[0], idx=idx_log[0], wt=wt)

    for i in range(3):
        pipe.step(i, e2e_compute)
    pipe.finish()
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for i in range(args.steps):
        pipe.step(args.warmup + i, e2e_compute)
    pipe.finish()
    f1.record()
    torch.cuda.synchronize()
    dte = f0.elapsed_time(f1) / 1e3
    if rank != 0:
        return
    uniq = [int(torch.unique(t).numel()) for t in idx_log]
    run_bytes = k3.expert_run_layout(LL, LI)[1]
    expert_bytes = sum(u * run_bytes for u in uniq)
    trunk_bytes = 2 * (2 * LL * LH + 3 * SI * LH)
    hbm, _, kind = peaks()
    exp_ms, trunk_ms = ms_buf[0], ms_buf[3]
    achieved = expert_bytes / (exp_ms / 1e3) / 1e9 if exp_ms > 0 else None
    cpu = None
    if not args.no_cpu:
        from oracle import oracle as ora
        if ora.ref_available():
            tps, threads, n, el = cpu_latent_tokens_per_s(args.cpu_seconds)
            cpu = {"value": tps, "unit": UNIT, "cores": threads, "kind": "reference",
                   "sample": f"{n} tokens through the reference's k3_moe ({el:.1f} s), 8 distinct experts tiled over 896 ids"}
    print(json.dumps({
        "metric": "K3 latent MoE-layer tokens/s", "value": B * args.steps / dt, "unit": UNIT, "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * dt / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": (f"experts mxfp4 x e4m3 ({args.terms} terms, tcgen05 kind::mxf8f6f4); " +
                  ("trunk bf16 weights x fp32 activations, fp64 accumulate in the reference's order (bit-exact)"
                   if B <= 32 else
                   "trunk bf16 weights x fp32 activations as two bf16 terms, fp32 accumulate (tcgen05 kind::f16)")),
        "data": "synthetic",
        "config": {"workload": LAT_WORKLOAD.replace("decode: B=16", f"{'decode' if B <= 32 else 'prefill'}: B={B}"),
                   "batch": B, "hidden": LH, "latent": LL, "inter": LI, "experts": LE,
                   "topk": LK, "n_shared": LS, "l2": "inputs larger than L2: each step reads its distinct experts (unique_experts_per_step x 17.5 MB) "
                         "and a rotating token batch"},
        "unique_experts_per_step": float(np.mean(uniq)),
        "stages_ms_per_step": {"experts": exp_ms / args.steps, "router": ms_buf[1] / args.steps,
                               "trunk": trunk_ms / args.steps},
        "trunk_gbs": trunk_bytes * args.steps / (trunk_ms / 1e3) / 1e9 if trunk_ms > 0 else None,
        "trunk_tflops": (2.0 * B * trunk_bytes / 2 * args.steps / (trunk_ms / 1e3) / 1e12
                         if trunk_ms > 0 and B > 32 else None),
        "layer_hbm_gbs": (expert_bytes + args.steps * (trunk_bytes + LE * LH * 4)) / dt / 1e9,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": achieved / hbm if achieved else None,
                     "kernel": "expert stage (tcgen05 gate/up+SiTU and down kernels at the latent width)",
                     "algorithmic_bytes_per_step": expert_bytes / args.steps, "peak_kind": kind},
        "cpu_baseline": cpu,
        "e2e": {"value": B * args.steps / dte, "unit": UNIT, "h2d_bytes_per_step": B * LH * 4,
                "d2h_bytes_per_step": B * LH * 4},
        "gpu_launches": int(launches),
        "clocks": clocks,
    }))


# ------------------------------------------------------------------ expert parallel (config[3])
EP_T = 16384
EP_WORKLOAD = "config[3] expert-parallel MoE prefill: 16384 bf16 tokens sharded over the GPUs, 384 " \
              "MXFP4 experts (7168->2048->7168) sharded over the GPUs (the 16 hottest on every GPU, each running its " \
              "own tokens' pairs of them; the rest (384-16)/N per GPU, placed by a balance of a calibration batch's " \
              "slot counts) + a shared expert on each, top-8 under a Zipf(1.1) selection bias (popularity over a " \
              "random permutation of the ids); token rows all-gathered during the router, pair rows stored at the " \
              "tokens' owners over NVLink from the expert kernels (--ep-impl a2a: NCCL all-to-all)"


def ep_init_group(ws, dev):
    """The process group of the expert-parallel layer: NCCL across ranks, or a one-rank gloo
    group in memory (no network) when this process is alone."""
    import datetime
    import torch.distributed as dist
    if dist.is_initialized():
        return
    if ws > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    else:
        dist.init_process_group("gloo", store=dist.HashStore(), rank=0, world_size=1)


def ep_cpu_leg(k3, ref_runs, W, bias, x, out_ep, idx_ep, ntok=8):
    """The reference's own CPU path (oracle/_ref: k3_router + k3_matmul_mxfp4 experts, SwiGLU,
    the top-k-order combine; every host core) on `ntok` of this rank's tokens: times it as the
    layer's CPU baseline and, as the checker, compares its routing and outputs with the
    expert-parallel layer's. Rank 0 only, after the timed region."""
    from oracle import oracle as ora
    if not ora.ref_available():
        return None, {"unavailable": "oracle/_ref/libk3ref.so not built"}
    import torch
    threads = ora.ref_use_all_cores()
    ids = sorted(set(int(v) for v in idx_ep[:ntok].reshape(-1).tolist()))
    host = {e: k3.synth.host_expert(ref_runs, e, H, I) for e in ids}
    shared = k3.synth.host_expert(ref_runs, E, H, I)
    experts = [host.get(e, host[ids[0]]) for e in range(E)]   # the others are never selected
    xf = x[:ntok].float().cpu().numpy()
    wf = W.float().cpu().numpy()
    t0 = time.perf_counter()
    ro, ri, _ = ora.moe_layer(xf, wf, bias.cpu().numpy(), experts, shared, H, I, K, use_ref=True)
    el = time.perf_counter() - t0
    got = out_ep[:ntok].cpu().numpy().astype(np.float64)
    err = float(np.abs(got - ro).max() / np.abs(ro).max())
    cpu = {"value": ntok / el, "unit": UNIT, "cores": threads, "kind": "reference",
           "sample": f"{ntok} config[3] tokens through the reference's k3_router and k3_matmul_mxfp4 "
                     f"experts ({el:.2f} s)"}
    return cpu, {"tokens": ntok, "indices_equal": bool(np.array_equal(ri, idx_ep[:ntok].cpu().numpy())),
                 "maxrel": err, "checker": "the reference's own kernels (oracle/_ref)"}


def ep_layer(args, k3, L, dev, ws, rank, local, steps, warmup, place="balanced", impl="fused",
             parity=True):
    """BASELINE config[3] on this process group: 16384 tokens in total, EP_T / ws per rank, the
    384 routed experts sharded 384 / ws per rank, top-8 under the Zipf(1.1) selection bias.
    Every rank generates the same 384 + 1 experts (same seed) and keeps its share in its
    arena; the full bank stays resident only for the parity check after the timed region,
    which runs 64 of each rank's tokens through the single-GPU layer built from the same
    weights (and, on rank 0, 8 of them through the reference's own CPU path).
    Returns the result dict on rank 0 (None elsewhere)."""
    import ctypes as C
    import torch
    import torch.distributed as dist
    ep_init_group(ws, dev)
    assert E % ws == 0
    per = E // ws
    ref_runs, arena_all = k3.synth.device_bank(k3, E + 1, H, I, dev, seed=4242)   # index E: shared
    stride = k3.pool_run_bytes(H, I)
    W, bias, sample = k3.synth.zipf_router(dev, E, H, K)
    if ws > 1:
        dist.broadcast(bias, 0)
    if place == "balanced" and ws > 1:
        # expert placement from routing statistics: a calibration batch of EP_T tokens drawn
        # apart from the benchmark's tokens (the way a deployment places experts from past
        # traffic), routed with the fitted bias. An expert's GEMM time goes with its 128-row
        # slots, so its load is its slot count at the full batch; greedy, heaviest expert to
        # the least-loaded rank.
        gc = torch.Generator(device=dev)
        gc.manual_seed(31337)
        calib = torch.randn((EP_T, H), generator=gc, device=dev).to(torch.bfloat16)
        sidx, _, _ = k3.router(calib, W, bias, K)
        del calib
        pairs = torch.bincount(sidx.reshape(-1).long(), minlength=E).double()
        dist.broadcast(pairs, 0)
        pl = pairs.cpu().tolist()
        # the R hottest experts are held by every rank, each running its own tokens' pairs of
        # them (their load splits evenly and their pair rows stay local); the rest are placed
        nrep = max(0, getattr(args, "ep_replicate", 0) if impl == "fused" else 0)
        while nrep and (E - nrep) % ws:
            nrep -= 1
        hot = sorted(sorted(range(E), key=lambda e: (-pl[e], e))[:nrep])
        rest = [e for e in range(E) if e not in set(hot)]
        own_r, lists_r = k3.ep.balanced_placement([float(np.ceil(pl[e] / 128.0)) for e in rest], ws)
        owner_l = [0] * E
        for i, e in enumerate(rest):
            owner_l[e] = own_r[i]
        lists = [sorted([rest[i] for i in lst] + hot) for lst in lists_r]
    else:
        hot = []
        owner_l = [e // per for e in range(E)]
        lists = [list(range(q * per, (q + 1) * per)) for q in range(ws)]
    owner = torch.tensor(owner_l, dtype=torch.int64, device=dev)
    hot_mask = torch.zeros(E, dtype=torch.bool, device=dev)
    hot_mask[hot] = True
    mine = torch.tensor(lists[rank] + [E], dtype=torch.int64, device=dev)
    per = len(lists[rank])
    if ws == 1:
        arena = arena_all
    else:
        arena = arena_all.view(E + 1, stride).index_select(0, mine).reshape(-1)
    run_of = torch.full((E,), -1, dtype=torch.int32, device=dev)
    run_of[mine[:-1]] = torch.arange(per, dtype=torch.int32, device=dev)
    none = torch.full((E,), -1, dtype=torch.int32, device=dev)
    T = EP_T // ws
    if impl == "fused":
        layer = k3.PoolMoeLayer(arena, per + 1, run_of, per, W, bias, H, I, K, terms=2)
        epl = k3.ep.FusedExpertParallel(k3, layer, t_max=T, gather_x=not getattr(args, "ep_no_gather", False))
    else:
        lr = k3.PoolMoeLayer(arena, per + 1, run_of, -1, W, bias, H, I, K, terms=2)
        lsh = k3.PoolMoeLayer(arena, per + 1, none, per, W, bias, H, I, K, terms=2)
        route, routed, shared = k3.ep.gpu_layer_fns(k3, lr, lsh, W, bias, K)
        epl = k3.ep.ExpertParallel(owner, route, routed, shared)
    gx = torch.Generator(device=dev)
    gx.manual_seed(99 + rank)
    xs = [torch.randn((T, H), generator=gx, device=dev).to(torch.bfloat16) for _ in range(2)]
    fwd_kw = {"counts": [T] * ws} if impl == "fused" else {}   # equal splits: no count exchange
    for i in range(warmup):
        epl.forward(xs[i % 2], **fwd_kw)
    torch.cuda.synchronize()
    graphs = None
    if impl == "fused" and getattr(args, "ep_graph", False):
        # the layer's launches (and its two barriers) captured once per input buffer and
        # replayed: no host work between the kernels of a step
        graphs = []
        per_graph = 0
        for i in range(2):
            gr = torch.cuda.CUDAGraph()
            l0 = L.k3c_launch_count()
            with torch.cuda.graph(gr):
                epl.forward(xs[i], **fwd_kw)
            per_graph = L.k3c_launch_count() - l0
            graphs.append(gr)
        for i in range(2):
            graphs[i].replay()
        torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    clk = Clocks(local)
    L.k3c_timing_enable(1)
    ms_buf = (C.c_double * 5)()
    n_buf = (C.c_longlong * 5)()
    L.k3c_timing_read(ms_buf, n_buf, 5)          # discard warm-up records
    launches0 = L.k3c_launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(steps):
        if graphs:
            graphs[i % 2].replay()
        else:
            epl.forward(xs[i % 2], **fwd_kw)
    e1.record()
    torch.cuda.synchronize()
    launches = L.k3c_launch_count() - launches0 if not graphs else per_graph * steps
    L.k3c_timing_enable(0)
    L.k3c_timing_read(ms_buf, n_buf, 5)
    stages = {name: ms_buf[j] / steps for j, name in enumerate(("experts", "router", "combine", "q8", "dispatch")) if name != "q8"}
    # the layer's phases, timed in separate steps after the timed region (events between them)
    phases = None
    if impl == "fused":
        epl.phase_timing(True)
        if graphs:   # replayed steps record no stage events: take the stages from these steps
            L.k3c_timing_enable(1)
            L.k3c_timing_read(ms_buf, n_buf, 5)
        for i in range(3):
            epl.forward(xs[i % 2], **fwd_kw)
        phases = epl.phase_read()
        epl.phase_timing(False)
        if graphs:
            L.k3c_timing_enable(0)
            L.k3c_timing_read(ms_buf, n_buf, 5)
            stages = {name: ms_buf[j] / 3 for j, name in enumerate(("experts", "router", "combine", "q8", "dispatch")) if name != "q8"}
        ph = torch.tensor([phases[k] for k in epl.PHASES], dtype=torch.float64, device=dev)
        if ws > 1:
            dist.all_reduce(ph, op=dist.ReduceOp.MAX)
        phases = {"rank0": phases, "max_over_ranks": dict(zip(epl.PHASES, ph.tolist())),
                  "experts_call_parts_rank0": {"grouped_gemms": stages["experts"],
                                               "dispatch": stages["dispatch"],
                                               "plan_other": phases["experts_call"] - stages["experts"]
                                               - stages["dispatch"]}}
    dist.barrier()
    torch.cuda.synchronize()
    clocks = clk.stop()
    dt_local = e0.elapsed_time(e1) / 1e3
    # NVLink traffic of one layer, from this rank's tokens' routing: a token is read once by
    # every other rank that owns one of its experts, and each of its pairs computed elsewhere
    # comes back as one bf16 row
    out_ep = epl.forward(xs[0], **fwd_kw)
    idx_ep = (epl.idx_buf[:T].clone() if impl == "fused" else k3.router(xs[0], W, bias, K)[0])
    dest = owner[idx_ep.long()]
    dest[hot_mask[idx_ep.long()]] = rank          # replicated experts run at the token's owner
    member = torch.zeros((T, ws), dtype=torch.bool, device=dev)
    member.scatter_(1, dest, True)
    member[:, rank] = False
    remote_rows = float(member.sum().item())
    gathered = impl == "fused" and getattr(epl, "gx", None) is not None
    if gathered:   # every other rank's rows arrive through the all-gather
        remote_rows = float((ws - 1) * T)
    remote_pairs = float((dest != rank).sum().item())
    # parity: 64 of this rank's tokens against the single-GPU layer over the full bank
    maxrel, idx_ok = 0.0, 1.0
    sel = None
    if parity:
        full = k3.PoolMoeLayer(arena_all, E + 1, torch.arange(E, dtype=torch.int32, device=dev), E, W, bias,
                               H, I, K, terms=2)
        pick = np.random.default_rng(rank).choice(np.arange(1, T - 1), 62, replace=False)
        sel = torch.from_numpy(np.sort(np.concatenate([[0, T - 1], pick]))).to(dev)
        ref_o, ref_i, _ = full.prefill(xs[0][sel])
        got = out_ep[sel].double()
        maxrel = float(((got - ref_o.double()).abs().max() / ref_o.double().abs().max()).item())
        idx_ok = float(torch.equal(ref_i, idx_ep[sel]))
        del full
    t = torch.tensor([dt_local, remote_rows, maxrel, -idx_ok, remote_pairs, stages["experts"]], dtype=torch.float64,
                     device=dev)
    if ws > 1:
        mx = t.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        sm = t.clone()
        dist.all_reduce(sm, op=dist.ReduceOp.SUM)
        dt, rows_all, maxrel_all, idx_all = float(mx[0]), float(sm[1]), float(mx[2]), -float(mx[3])
        pairs_all, exp_max, exp_mean = float(sm[4]), float(mx[5]), float(sm[5]) / ws
    else:
        dt, rows_all, maxrel_all, idx_all = dt_local, remote_rows, maxrel, idx_ok
        pairs_all, exp_max, exp_mean = remote_pairs, stages["experts"], stages["experts"]
    graphs = None   # graphs holding NCCL calls go before the process group does
    if impl == "fused":
        epl.close()
    if rank != 0:
        return None
    cpu, ora_par = (None, None)
    if parity and not args.no_cpu:
        cpu, ora_par = ep_cpu_leg(k3, ref_runs, W, bias, xs[0][sel], out_ep[sel], idx_ep[sel])
        if ws > 1:
            cpu = None   # a CPU baseline is reported at N = 1 only; the check above still ran
    flop = (EP_T * K + EP_T) * 2 * 3 * I * H
    return {
        "workload": EP_WORKLOAD, "tokens": EP_T, "n_gpus": ws, "steps": steps, "warmup": warmup,
        "tokens_per_s": EP_T * steps / dt, "unit": UNIT, "ms_per_step": 1e3 * dt / steps,
        "scaling": "strong", "parallelism": f"ep{ws}",
        "placement": (place + (f", the {len(hot)} hottest experts on every rank" if hot else "")) if ws > 1
                     else "all experts", "impl": impl,
        "dtype": "mxfp4 x e4m3 (activations as 2 E4M3 terms), fp32 accumulate (tcgen05 kind::mxf8f6f4)",
        "useful_tflops": flop * steps / dt / 1e12,
        "stages_ms_per_step_rank0": stages,
        "phases_ms": phases,
        "expert_stage_ms_max_over_ranks": exp_max, "expert_stage_ms_mean_over_ranks": exp_mean,
        "nvlink_per_step": {"remote_token_rows_received": rows_all, "bytes_received": rows_all * H * 2,
                            "pair_rows_written": pairs_all, "bytes_written": pairs_all * H * 2,
                            "how": ("every rank's bf16 token rows all-gathered to every rank (NCCL, side stream, "
                                    "during the router)" if gathered else
                                    "bf16 token rows read by each rank that owns one of the token's experts")
                                   + "; one bf16 pair row stored at the token's owner per pair computed elsewhere"}
        if impl == "fused" else None,
        "parity": {"tokens_per_rank": 64 if parity else 0, "maxrel_vs_single_gpu": maxrel_all if parity else None,
                   "indices_equal_single_gpu": bool(idx_all == 1.0) if parity else None,
                   "single_gpu_layer": "k3c_moe_prefill_tc over all 384 experts, same weights",
                   "tolerance": 2e-2, "oracle": ora_par},
        "cpu_baseline": cpu,
        "gpu_launches": int(launches),
        "clocks": clocks,
    }


def run_ep(args, ws, rank, local):
    """--workload ep: config[3] as its own line (the same section the default line carries
    under "ep")."""
    import torch
    import torch.distributed as dist
    import __graft_entry__ as ge
    k3 = ge.load_package()
    L = k3.lib()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    r = ep_layer(args, k3, L, dev, ws, rank, local, args.steps, args.warmup, args.ep_place, args.ep_impl,
                 parity=not args.no_parity)
    dist.destroy_process_group()
    if rank != 0:
        return
    print(json.dumps({
        "metric": METRIC, "value": r["tokens_per_s"], "unit": UNIT, "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": r["dtype"], "data": "synthetic",
        "config": {"workload": EP_WORKLOAD, "tokens": EP_T, "hidden": H, "inter": I, "experts": E, "topk": K,
                   "parallelism": f"ep{ws}", "placement": r["placement"]},
        **{k: r[k] for k in ("useful_tflops", "stages_ms_per_step_rank0", "phases_ms", "expert_stage_ms_max_over_ranks",
                             "expert_stage_ms_mean_over_ranks", "nvlink_per_step", "parity", "cpu_baseline",
                             "gpu_launches", "clocks")}}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--distinct", type=int, default=E,
                    help="distinct expert weights tiled over the 384 ids (profiling only)")
    ap.add_argument("--path", default="tc", choices=["tc", "cuda"],
                    help="tc: tcgen05 block-scaled MMA path; cuda: CUDA-core GEMV path")
    ap.add_argument("--terms", type=int, default=3, help="E4M3 activation terms (tc path)")
    ap.add_argument("--batch", type=int, default=16,
                    help="latent workload: tokens per step (above 32 the many-token path)")
    ap.add_argument("--ep-place", default="balanced", choices=["balanced", "contiguous"],
                    help="ep workload: expert placement balanced on a routing sample's pair counts, or "
                         "contiguous id ranges")
    ap.add_argument("--ep-impl", default="fused", choices=["fused", "a2a"],
                    help="ep workload: fused peer-memory exchange in the expert kernels, or NCCL all-to-all")
    ap.add_argument("--ep-graph", action="store_true",
                    help="ep: replay each step from a CUDA graph of the layer's launches (barriers included)")
    ap.add_argument("--ep-steps", type=int, default=10,
                    help="default line: timed steps of the config[3] expert-parallel layer (its 'ep' object)")
    ap.add_argument("--ep-replicate", type=int, default=16,
                    help="ep workload, balanced placement: the R hottest experts (calibration batch) held by every rank, "
                         "each rank running its own tokens' pairs of them")
    ap.add_argument("--ep-no-gather", action="store_true",
                    help="ep workload: the quantisation pulls the other ranks' token rows after the barrier "
                         "instead of an all-gather during the router")
    ap.add_argument("--no-ep", action="store_true", help="default line without the 'ep' object")
    ap.add_argument("--no-parity", action="store_true", help="ep: skip the parity check after the timed region")
    ap.add_argument("--workload", default="decode",
                    choices=["decode", "prefill", "streamed", "ep", "expert", "latent"],
                    help="decode: config[1] (the headline line); prefill: config[2]; streamed: config[4]; "
                         "ep: config[3] (expert-parallel prefill; torchrun for N > 1)")
    args = ap.parse_args()
    ws, rank, local = dist_setup(args)
    if args.workload == "prefill" and args.impl != "reference":
        run_prefill(args, ws, rank, local)
    elif args.workload == "streamed" and args.impl != "reference":
        run_streamed(args, ws, rank, local)
    elif args.workload == "ep" and args.impl != "reference":
        run_ep(args, ws, rank, local)
    elif args.workload == "expert" and args.impl != "reference":
        run_expert(args, ws, rank, local)
    elif args.workload == "latent" and args.impl != "reference":
        run_latent(args, ws, rank, local)
    elif args.impl == "reference":
        run_reference(args, ws, rank)
    else:
        run_ours(args, ws, rank, local)


if __name__ == "__main__":
    main()
