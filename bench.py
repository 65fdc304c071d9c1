"""Benchmark of the ReSS/HeSS sparse global-attention layer on B200.

Workload: one VGGT global-attention layer at 32
frames x (5 special + 37*37 patch) tokens = 43,968 tokens, 16 heads x 64,
bf16, synthetic clustered Q/K/V; apply_ress(sparse_ratio=0.5, n_iters=5)
with a HeSS budget from a log-normal (3, 24, 16) Fisher table mixed at
lambda = 0.5.  One step = the whole layer after the Q/K/V projection:
scoring + quantisation, budget, restore-swap selection, tcgen05 sparse
attention, dense special-token queries, output in the full token layout.

Metric: views of the global layer processed per second (32 views per step;
the layer ms is reported beside it).  With --gpus N (torchrun) the 16 heads
are split across the N GPUs (strong scaling); HeSS needs the baseline counts
of all heads per q-block, which are all-gathered with NCCL.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ress|reference]
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

N_FRAMES = 32
# DRAM bytes (read + write) of one attention launch on the 32-frame layer:
# 237.4 MB measured by ncu (dram__bytes_read.sum + dram__bytes_write.sum) on
# the 24-frame layer, scaled by the token count 43,968 / 32,976.
ATTN_DRAM_BYTES_PER_LAUNCH = 237.4e6 * 43968 / 32976
SPARSE_RATIO = 0.5
CDF = 0.97
METRIC = "global-attn layer throughput, VGGT cfg2 (32 views, 43,968 tokens, 16x64 heads, apply_ress sr=0.5)"
UNIT = "views/s"


def _args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ress", choices=["ress", "reference"])
    ap.add_argument("--frames", type=int, default=N_FRAMES)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-attn", action="store_true", help="one small layer, for ncu")
    ap.add_argument("--profile-score", action="store_true",
                    help="the scoring passes (pooling, quantisation, key mean) on the cfg2 layer, for ncu")
    ap.add_argument("--profile-rs", action="store_true",
                    help="restore-swap on the cfg2 layer with 0/1/5 rounds and track-best off/on, for ncu")
    ap.add_argument("--profile-select", action="store_true",
                    help="top-m and round-step kernels at the reference's quoted Triton shapes")
    ap.add_argument("--profile-dense", action="store_true",
                    help="the dense bf16 attention kernel on frame-attention and special-query shapes")
    ap.add_argument("--eager", action="store_true", help="time eager calls instead of CUDA-graph replays")
    ap.add_argument("--shard", default="heads", choices=["heads", "views"],
                    help="views: frames split over the ranks, K/V all-gathered (whole-model sharding)")
    ap.add_argument("--sparse-ratio", type=float, default=None)
    ap.add_argument("--model", default=None, choices=["vggt"],
                    help="whole VGGT-1B-shaped aggregator (configs 3/4) instead of one global layer")
    ap.add_argument("--sweep", action="store_true",
                    help="standalone block-sparse attention: token counts x densities with random per-head maps")
    return ap.parse_args()


def _dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("bf16_tflops", 1590.0), d.get("hbm_gbs", 6650.0), "measured"
    return 1590.0, 6650.0, "fallback"


class Clocks:
    """nvidia-smi sampling during the timed region.  The sampler is started
    and its first sample awaited before the region begins (starting
    nvidia-smi takes longer than a short region); samples arrive every 25 ms
    and are timestamped on arrival, and only those that arrive between the
    start and the end of the region (plus one sampling interval) count."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    INTERVAL_MS = int(os.environ.get("RESS_BENCH_CLOCK_MS", "25"))

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.stamped = []  # (arrival time, line)
        self.t0 = self.t1 = None

    def _reader(self):
        for ln in self.proc.stdout:
            if ln.strip():
                self.stamped.append((time.monotonic(), ln))

    def __enter__(self):
        import threading

        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", str(self.INTERVAL_MS)],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        if self.proc is not None:
            self.thread = threading.Thread(target=self._reader, daemon=True)
            self.thread.start()
            deadline = time.monotonic() + 5.0
            while not self.stamped and time.monotonic() < deadline and self.proc.poll() is None:
                time.sleep(0.005)
        self.t0 = time.monotonic()
        return self

    def __exit__(self, *exc):
        self.t1 = time.monotonic()
        if self.proc is not None:
            time.sleep(self.INTERVAL_MS * 2 / 1000.0)  # the sample taken at the region's end
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.proc.wait()
            self.thread.join(timeout=5)
        grace = self.INTERVAL_MS * 1.5 / 1000.0
        self.lines = [ln for t, ln in self.stamped if self.t0 <= t <= self.t1 + grace]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        region_ms = round((self.t1 - self.t0) * 1e3, 1) if self.t0 is not None and self.t1 is not None else None
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": [], "samples": 0, "region_ms": region_ms}
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm),
                "region_ms": region_ms}


def _setup(frames, world, rank, device):
    from ress_b200 import kernels as K
    from ress_b200 import layer as LY
    from ress_b200 import synth

    shape = synth.LayerShape(n_frames=frames)
    q, k, v = synth.layer_qkv(shape, seed=0, dtype=torch.bfloat16, device=device)
    H = shape.n_heads
    if world > H:
        raise SystemExit(f"{H} heads do not split over {world} GPUs")
    # HessBudget tables: row 0 (W_Q) of two log-normal (3, 24, 16) tables, lambda = 0.5, layer 0
    cam, pcd = synth.fisher_table(seed=1)[0], synth.fisher_table(seed=3)[0]
    cam = cam / cam.sum(-1, keepdim=True)
    pcd = pcd / pcd.sum(-1, keepdim=True)
    comb = 0.5 * cam + 0.5 * pcd
    head_scores = (comb / comb.sum(-1, keepdim=True))[0]
    sn = K.scores_norm(head_scores).to(device)
    shard = None
    heads = list(range(H))
    if world > 1:
        from ress_b200 import shard as SH

        # heads balanced over the GPUs by their expected work (HeSS budgets grow with the
        # score); ranks may hold different numbers of heads
        shard = SH.make_head_shard(H, world, rank, scores=head_scores, cap=1.0 / (1.0 - SPARSE_RATIO),
                                   equal_size=False)
        heads = list(shard.heads)
    hl = len(heads)
    hidx = torch.as_tensor(heads, dtype=torch.long, device=device)
    q, k, v = (t.index_select(1, hidx).contiguous() for t in (q, k, v))
    L = K.Layout(1, hl, shape.n_frames, shape.n_special, shape.hw)
    M = synth.metric_from_weight(synth.out_proj_weight(), H)[hidx.cpu()].to(device)
    h0 = heads[0]
    budget = LY.BudgetSpec("hess", sparse_ratio=SPARSE_RATIO, cdf_threshold=None, scores_norm=sn)
    budget_hess = LY.BudgetSpec("hess", sparse_ratio=SPARSE_RATIO, cdf_threshold=CDF, scores_norm=sn)
    order = LY.OrderSpec("restore_swap", M=M, n_iters=5, track_best=True)
    order_prob = LY.OrderSpec("probability")
    return dict(shape=shape, q=q, k=k, v=v, L=L, budget=budget, budget_hess=budget_hess, order=order,
                order_prob=order_prob, shard=shard, h0=h0, hl=hl, heads=heads)


def _int8_peak(device):
    """Dense int8 tensor-core throughput (TOP/s) of this GPU: cuBLASLt int8 x
    int8 -> int32 GEMM at 8192^3 through torch._int_mm, best of 10 CUDA-event
    timed calls after 3 warm-ups (the int8 counterpart of the driver's bf16
    burst figure)."""
    n = 8192
    g = torch.Generator(device=device).manual_seed(0)
    a = torch.randint(-128, 128, (n, n), dtype=torch.int8, device=device, generator=g)
    b = torch.randint(-128, 128, (n, n), dtype=torch.int8, device=device, generator=g)
    for _ in range(3):
        torch._int_mm(a, b)
    best = None
    for _ in range(10):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        torch._int_mm(a, b)
        e1.record()
        e1.synchronize()
        ms = e0.elapsed_time(e1)
        best = ms if best is None else min(best, ms)
    del a, b
    return 2.0 * n ** 3 / (best / 1e3) / 1e12


def _attn_flops(lists, counts, L):
    """Kept-block FLOPs: 4 * q_rows * k_rows * 64 per (row, kept block)."""
    rows = counts.numel()
    nq = L.nq
    qb = torch.arange(rows, device=counts.device) % nq
    q_rows = (L.Tp - qb * 128).clamp(max=128).to(torch.float64)
    ar = torch.arange(lists.shape[1], device=lists.device)
    valid = ar.unsqueeze(0) < counts.unsqueeze(1)
    k_rows = (L.Tk - lists.to(torch.int64) * 64).clamp(min=0, max=64).to(torch.float64)
    k_sum = torch.where(valid, k_rows, torch.zeros_like(k_rows)).sum(1)
    return float((4.0 * 64.0 * q_rows * k_sum).sum().item())


def _time_region(fn, steps, stream):
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(steps):
        fn()
    end.record(stream)
    end.synchronize()
    return start.elapsed_time(end)


def _cpu_layer_once(S, t):
    """One cfg2 layer on the host cores: the oracle's scoring + HeSS +
    restore-swap selection (C, OpenMP) and fp32 block-gathered attention over
    every (head, q-block) row.  Fills t["select"], t["attn"] (seconds)."""
    import oracle

    q, k, v, qp, key, val, M, hs = S["_cpu"]
    t0 = time.perf_counter()
    o = oracle.layer_select(qp, key[..., : qp.shape[-2], :], val[..., : qp.shape[-2], :], key.shape[-2] - qp.shape[-2],
                            M, head_scores=hs, mode="ress", sparse_ratio=SPARSE_RATIO)
    t1 = time.perf_counter()
    oracle.gathered_attention_fp32(qp, key, val, o["lists"], o["counts"])
    t2 = time.perf_counter()
    t["select"], t["attn"] = t1 - t0, t2 - t1
    return o


def _cpu_prepare(S):
    from ress_b200 import synth

    if "_cpu" not in S:
        shape = S["shape"]
        q, k, v = (t.cpu() for t in (S["q"], S["k"], S["v"]))
        qp, _ = synth.split_tokens(q, shape)
        kp, ks = synth.split_tokens(k, shape)
        vp, vs = synth.split_tokens(v, shape)
        S["_cpu"] = (q, k, v, qp, torch.cat([kp, ks], -2), torch.cat([vp, vs], -2), S["order"].M.cpu(),
                     S["budget"].scores_norm.cpu())
    return S["_cpu"]


def _cpu_baseline(S, reps=3):
    """The path on the host cores over one whole cfg2 layer (no extrapolation):
    selection by the oracle, attention as fp32 block-gathered torch matmuls
    over every (head, q-block) row and its kept blocks.  One warm-up layer,
    then the median of `reps` timed layers; the two legs are reported
    separately."""
    import oracle

    _cpu_prepare(S)
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    runs = []
    for i in range(reps + 1):
        t = {}
        _cpu_layer_once(S, t)
        if i > 0:
            runs.append(t)
    runs.sort(key=lambda t: t["select"] + t["attn"])
    med = runs[len(runs) // 2]
    per_layer = med["select"] + med["attn"]
    return {"value": S["shape"].n_frames / per_layer, "unit": UNIT, "cores": threads, "kind": "port",
            "select_s": round(med["select"], 4), "attn_s": round(med["attn"], 4),
            "cpu": _cpu_model(), "oracle_threads": oracle.num_threads(), "torch_threads": torch.get_num_threads(),
            "sample": (f"one whole cfg2 layer per run, median of {reps} after one warm-up: oracle scoring + "
                       f"HeSS + restore-swap ({med['select']:.2f} s) and fp32 block-gathered torch attention "
                       f"over all {S['L'].H * S['L'].nq} (head, q-block) rows ({med['attn']:.2f} s)")}


def _cpu_model():
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


def run_reference(args):
    """--impl reference: the path on the host cores (the oracle's selection
    and fp32 block-gathered attention, see _cpu_baseline), one whole cfg2
    layer per step; rank 0 only."""
    ws, rank, local = _dist()
    if rank != 0:
        return
    device = "cuda" if torch.cuda.is_available() else "cpu"
    S = _setup(args.frames, 1, 0, device)
    steps = max(1, min(args.steps, 5))
    warm = min(1, max(0, args.warmup))
    _cpu_prepare(S)
    torch.set_num_threads(os.cpu_count() or 1)
    runs = []
    for i in range(warm + steps):
        t = {}
        _cpu_layer_once(S, t)
        if i >= warm:
            runs.append(t)
    runs.sort(key=lambda t: t["select"] + t["attn"])
    med = runs[len(runs) // 2]
    per_layer = med["select"] + med["attn"]
    value = args.frames / per_layer
    import oracle

    cb = {"value": value, "unit": UNIT, "cores": os.cpu_count(), "kind": "port", "cpu": _cpu_model(),
          "oracle_threads": oracle.num_threads(), "torch_threads": torch.get_num_threads(),
          "select_s": round(med["select"], 4), "attn_s": round(med["attn"], 4),
          "sample": (f"one whole cfg2 layer per step, median of {steps} steps after {warm} warm-up: oracle "
                     f"scoring + HeSS + restore-swap and fp32 block-gathered torch attention over all "
                     f"{S['L'].H * S['L'].nq} (head, q-block) rows")}
    line = {"metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
            "steps": steps, "warmup": warm, "ms_per_step": per_layer * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"cfg2 single global layer, {args.frames} views", "sparse_ratio": SPARSE_RATIO,
                       "n_iters": 5, "note": "the reference's path on the host cores: its selection as restated by "
                                             "the oracle, its attention as fp32 block-gathered torch attention "
                                             "(SpargeAttn has no CPU implementation); steps capped at 5"},
            "cpu_baseline": cb,
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_ress(args):
    from ress_b200 import kernels as K
    from ress_b200 import layer as LY

    ws, rank, local = _dist()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if ws > 1:
        import torch.distributed as dist
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    S = _setup(args.frames, ws, rank, device)
    L = S["L"]
    stream = torch.cuda.current_stream(device)
    out = torch.empty(1, L.H, L.frames * (L.special + L.hw), 64, dtype=torch.float32, device=device)

    def eager_step():
        # attn_split=None: with the heads split over many GPUs a rank's launch has few
        # rows, and rows that keep nearly every block run as two halves
        return LY.global_layer(S["q"], S["k"], S["v"], L, S["budget"], S["order"], out=out, shard=S["shard"],
                               attn_split=None)

    def barrier():
        if ws > 1:
            torch.distributed.barrier()

    res = eager_step()
    torch.cuda.synchronize()
    K.check_status(device)
    graph = None
    if args.eager:
        step = eager_step
    else:
        graph = LY.CapturedLayer(eager_step)
        step = graph.replay
        res = graph.result
    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    K.check_status(device)
    # kept blocks and list slots over all ranks (head groups may differ in size)
    kept = torch.stack([res.counts.sum().to(torch.float64),
                        torch.tensor(float(res.counts.numel() * res.width), dtype=torch.float64, device=device)])
    if ws > 1:
        torch.distributed.all_reduce(kept)
    sparsity = 1.0 - float(kept[0].item()) / float(kept[1].item())
    attn_flops = _attn_flops(res.lists, res.counts, L)

    barrier()
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        ms = _time_region(step, args.steps, stream)
    torch.cuda.synchronize()
    barrier()
    K.check_status(device)
    t = torch.tensor([ms], device=device)
    if ws > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms = float(t.item())
    ms_step = ms / args.steps
    value = args.frames * args.steps / (ms / 1000.0)

    # dominant kernel: the sparse attention, timed alone on the same lists
    qbar, q8, qs = K.pool_quant_q(S["q"], L)
    _, _, k8, ks, v16, _ = K.pool_quant_kv(S["k"], S["v"], L, pool=False)
    lists, counts = res.lists, res.counts

    def attn():
        K.sparse_attn(q8, qs, k8, ks, v16, lists, counts, out=out, out_layout=L, split=None)

    for _ in range(3):
        attn()
    reps = max(5, min(50, args.steps))
    attn_ms = _time_region(attn, reps, stream) / reps
    K.check_status(device)
    bf16_peak, hbm_peak, peak_src = _peaks()
    int8_peak = _int8_peak(device)
    mixed_peak = 2.0 / (1.0 / bf16_peak + 1.0 / int8_peak)
    achieved = attn_flops / (attn_ms / 1000.0) / 1e12

    # stage breakdown (eager calls, the second of two instrumented steps).  A
    # device-side sleep is queued first so that the host has enqueued the
    # whole step before it starts: the events then bracket device time only,
    # not the gaps of eager launches.
    stages = {}
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
    for _ in range(2):
        torch.cuda._sleep(40_000_000)
        ev[0].record(stream)
        qbar, q8, qs = K.pool_quant_q(S["q"], L)
        kbar, vbar, k8, ks, v16, km = K.pool_quant_kv(S["k"], S["v"], L)
        ev[1].record(stream)
        af, ac = K.predict(qbar, kbar, L.n_cand)
        base = K.baseline(ac, SPARSE_RATIO).view(1, L.H, L.nq)
        if S["shard"] is not None:
            base = S["shard"].gather(base)
        nts = K.hess_adjust(base, S["budget"].scores_norm, L.n_cand, min_clamp=2)
        if S["shard"] is not None:
            nts = S["shard"].select(nts, L.H)
        ev[2].record(stream)
        r = K.restore_swap(af, vbar, S["order"].M, nts.view(-1), L.n_cand, sink_blocks=L.sink_blocks)
        ev[3].record(stream)
        K.sparse_attn(q8, qs, k8, ks, v16, r["lists"], r["counts"], out=out, out_layout=L, split=None)
        ev[4].record(stream)
        ev[4].synchronize()
    for i, name in enumerate(["score_quant", "predict_budget", "restore_swap", "sparse_attn"]):
        stages[name] = round(ev[i].elapsed_time(ev[i + 1]), 4)
    hess_ms = None
    if ws == 1:
        def step_hess():
            LY.global_layer(S["q"], S["k"], S["v"], L, S["budget_hess"], S["order_prob"], out=out)
        step_hess()
        torch.cuda.synchronize()
        hess_ms = _time_region(step_hess, max(10, args.steps // 4), stream) / max(10, args.steps // 4)

    # e2e: host buffers in and out through the public layer call.  Steps are
    # pipelined the way a serving loop would run them: step i+1's inputs go
    # host->device on a copy stream while step i computes and step i-1's
    # output goes device->host on another, with two device slots of inputs
    # and outputs.  Every step copies its own inputs in and its result out
    # inside the timed region.
    qh, kh, vh = (x.cpu().pin_memory() for x in (S["q"], S["k"], S["v"]))
    ohs = [torch.empty(out.shape, dtype=out.dtype, pin_memory=True) for _ in range(2)]
    s_in = torch.cuda.Stream(device)
    s_out = torch.cuda.Stream(device)
    slots = [dict(q=torch.empty_like(S["q"]), k=torch.empty_like(S["k"]), v=torch.empty_like(S["v"]),
                  o=torch.empty_like(out), in_ready=torch.cuda.Event(), used=torch.cuda.Event(),
                  done=torch.cuda.Event(), drained=torch.cuda.Event()) for _ in range(2)]
    for sl in slots:
        sl["used"].record(stream)
        sl["drained"].record(stream)

    def e2e_step(i):
        sl = slots[i % 2]
        with torch.cuda.stream(s_in):
            s_in.wait_event(sl["used"])
            sl["q"].copy_(qh, non_blocking=True)
            sl["k"].copy_(kh, non_blocking=True)
            sl["v"].copy_(vh, non_blocking=True)
            sl["in_ready"].record(s_in)
        stream.wait_event(sl["in_ready"])
        stream.wait_event(sl["drained"])
        LY.global_layer(sl["q"], sl["k"], sl["v"], L, S["budget"], S["order"], out=sl["o"], shard=S["shard"],
                        attn_split=None)
        sl["used"].record(stream)
        sl["done"].record(stream)
        with torch.cuda.stream(s_out):
            s_out.wait_event(sl["done"])
            ohs[i % 2].copy_(sl["o"], non_blocking=True)
            sl["drained"].record(s_out)

    for i in range(2):
        e2e_step(i)
    torch.cuda.synchronize()
    barrier()
    e_steps = max(3, args.steps)  # as many as the device-timed region: the pipeline's fill and drain amortise
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    s_in.wait_stream(stream)
    s_out.wait_stream(stream)
    for i in range(e_steps):
        e2e_step(i)
    stream.wait_stream(s_out)
    e1.record(stream)
    e1.synchronize()
    e_ms = e0.elapsed_time(e1)
    te = torch.tensor([e_ms], device=device)
    if ws > 1:
        torch.distributed.all_reduce(te, op=torch.distributed.ReduceOp.MAX)
    e_ms = float(te.item())
    # bytes of the whole layer: every rank copies its own heads' share, summed over ranks
    nb = torch.tensor([float(sum(x.numel() * x.element_size() for x in (qh, kh, vh))),
                       float(ohs[0].numel() * ohs[0].element_size())], dtype=torch.float64, device=device)
    if ws > 1:
        torch.distributed.all_reduce(nb)
    h2d, d2h = int(nb[0].item()), int(nb[1].item())

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        try:
            cpu = _cpu_baseline(S)
        except Exception as exc:  # the baseline is reported, never required
            cpu = {"value": None, "unit": UNIT, "cores": None, "kind": "port", "sample": f"failed: {exc}"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": args.steps,
            "warmup": max(3, args.warmup), "ms_per_step": ms_step, "layer_ms": ms_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": f"cfg2: one VGGT global-attention layer, {args.frames} views x 1374 tokens, "
                                   f"16 heads x 64, bf16, apply_ress(sparse_ratio={SPARSE_RATIO}, n_iters=5), "
                                   "HeSS budget lambda=0.5",
                       "parallelism": f"heads split over {ws} GPU(s)" + (
                           f" by expected work ({L.H} heads on rank 0), NCCL all-gather of HeSS baselines"
                           if ws > 1 else ""),
                       "launch": "eager calls" if args.eager else "one CUDA graph replay per step (layer captured once)",
                       "l2": "inputs larger than L2 (Q/K/V bf16 270 MB)", "sparsity": round(sparsity, 4)},
            "stages_ms": stages,
            "apply_hess_layer_ms": hess_ms,
            # per step: pool_q, pool_kv1<K>, key_mean, kquant, pool_kv1<V>, predict,
            # baseline, hess, vbar_terms, restore_swap, row_order, sparse_attn
            # (this library's kernels)
            "gpu_launches": 12 * args.steps,
            "roofline": {"bound": "tensor", "kernel": "sparse_attn_kernel", "achieved": achieved,
                         "peak": mixed_peak, "unit": "TFLOP/s", "frac": achieved / mixed_peak,
                         "traffic": ATTN_DRAM_BYTES_PER_LAUNCH * args.frames / N_FRAMES * L.H / S["shape"].n_heads,
                         "traffic_note": "dram read+write bytes per launch on this rank (its share of the heads), "
                                         "ncu on the 24-frame layer scaled by tokens",
                         "attn_ms": attn_ms, "attn_tflop_per_launch": attn_flops / 1e12,
                         "peak_note": f"harmonic mix of the bf16 burst peak {bf16_peak:.0f} TF/s ({peak_src}, "
                                      f"P.V half) and the int8 peak {int8_peak:.0f} TOP/s measured in this run "
                                      "(torch._int_mm 8192^3, best of 10; Q.K^T half)"},
            "clocks": clk.summary(),
            "e2e": {"value": args.frames * e_steps / (e_ms / 1000.0), "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "steps": e_steps,
                    "note": "pinned host Q/K/V in, fp32 output out, every step; copies of neighbouring steps "
                            "overlap the layer on separate streams (two device slots)"},
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    del graph, step
    torch.cuda.synchronize()
    if ws > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def run_views(args):
    """One global layer with the frames split over the ranks (the whole-model
    sharding of many-view runs): each rank owns frames/N frames, all-gathers
    K and V with NCCL and runs its q-blocks.  Weak in queries, fixed layer."""
    from ress_b200 import kernels as K
    from ress_b200 import shard as SH

    ws, rank, local = _dist()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if ws > 1:
        import torch.distributed as dist
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    S = _setup(args.frames, 1, 0, device)
    L = S["L"]
    geom = SH.ViewGeom(args.frames, L.special, L.hw, ws, rank)
    per = geom.frames_local * (L.special + L.hw)
    q, k, v = (t[:, :, rank * per:(rank + 1) * per].contiguous() for t in (S["q"], S["k"], S["v"]))
    del S["q"], S["k"], S["v"]
    if ws > 1:
        gather = SH.make_view_gather(ws)
    else:
        def gather(name, t):
            return [t]
    stream = torch.cuda.current_stream(device)

    def step():
        return SH.view_sharded_layer(q, k, v, geom, S["budget"], S["order"], gather)

    for _ in range(max(3, args.warmup)):
        res = step()
    torch.cuda.synchronize()
    K.check_status(device)
    if ws > 1:
        torch.distributed.barrier()
    ms = _time_region(step, args.steps, stream)
    torch.cuda.synchronize()
    K.check_status(device)
    t = torch.tensor([ms], device=device)
    if ws > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms = float(t.item())
    kept = res.counts.sum().to(torch.float64)
    rows = torch.tensor([float(res.counts.numel())], dtype=torch.float64, device=device)
    if ws > 1:
        torch.distributed.all_reduce(kept)
        torch.distributed.all_reduce(rows)
    width = L.n_cand + L.sink_blocks
    if rank == 0:
        line = {"metric": "global-attn layer throughput, view-sharded", "value": args.frames * args.steps / (ms / 1e3),
                "unit": UNIT, "n_gpus": ws, "steps": args.steps, "warmup": max(3, args.warmup),
                "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "bf16", "data": "synthetic",
                "config": {"workload": f"one VGGT global layer, {args.frames} views, frames split over {ws} GPU(s), "
                                       f"apply_ress(sparse_ratio={SPARSE_RATIO}), NCCL all-gather of K and V",
                           "parallelism": f"views over {ws}", "sparsity": round(1 - float(kept.item()) /
                                                                                 (float(rows.item()) * width), 4)}}
        print(json.dumps(line), flush=True)
    if ws > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def run_sweep(args):
    """The block-sparse attention op alone (config 5): Tp queries = Tk keys in
    8K..300K, random per-(head, q-block) keep maps at densities 0.1..0.9,
    16 heads x 64, bf16 inputs quantised like the layer.  One JSON line per
    point; kernel time by CUDA events over `--steps` launches.  Under
    torchrun the heads are split over the GPUs (16 / N each, no exchange:
    every (head, q-block) row is independent) and the time is the maximum
    over ranks; TFLOP/s count the kept blocks of all ranks."""
    from ress_b200 import kernels as K

    ws, rank, local = _dist()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if ws > 1:
        import torch.distributed as dist
        from datetime import timedelta

        if 16 % ws:
            raise SystemExit(f"16 heads do not split over {ws} GPUs")
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    H = 16
    hl = H // ws
    h0 = rank * hl
    stream = torch.cuda.current_stream(device)
    bf16_peak, _, peak_src = _peaks()
    int8_peak = _int8_peak(device)
    mixed = 2.0 / (1.0 / bf16_peak + 1.0 / int8_peak)
    g = torch.Generator(device=device).manual_seed(0)  # every rank draws the full op, then keeps its heads
    for T in (8192, 32768, 131072, 300032):
        q, k, v = (torch.randn(1, H, T, 64, device=device, generator=g, dtype=torch.float32).to(torch.bfloat16)
                   for _ in range(3))
        q, k, v = (t[:, h0:h0 + hl].contiguous() for t in (q, k, v))
        L = K.Layout.plain(q)
        _, q8, qs = K.pool_quant_q(q, L, pool=False)
        _, _, k8, ks, v16, _ = K.pool_quant_kv(k, v, L, pool=False)
        del q, k, v
        nq, nkb = L.nq, L.nkb
        for dens in (0.1, 0.5, 0.9):
            m = torch.rand(H * nq, nkb, device=device, generator=g) < dens
            m = m[h0 * nq:(h0 + hl) * nq].contiguous()
            lists, counts = K.map_to_lists(m)
            out = torch.empty(hl, T, 64, dtype=torch.float32, device=device)

            def call():
                K.sparse_attn(q8, qs, k8, ks, v16, lists, counts, out=out)

            for _ in range(3):
                call()
            steps = max(3, min(args.steps, 20))
            torch.cuda.synchronize()
            if ws > 1:
                torch.distributed.barrier()
            ms = _time_region(call, steps, stream) / steps
            K.check_status(device)
            t = torch.tensor([ms, float(counts.sum().item())], dtype=torch.float64, device=device)
            if ws > 1:
                mx = t[:1].clone()
                torch.distributed.all_reduce(mx, op=torch.distributed.ReduceOp.MAX)
                torch.distributed.all_reduce(t)
                t[0] = mx[0]
            ms, kept = float(t[0].item()), float(t[1].item())
            flops = 4.0 * 128 * 64 * 64 * kept
            tf = flops / (ms / 1e3) / 1e12
            if rank == 0:
                print(json.dumps({"metric": "block-sparse attention op (config 5)", "Tp": T, "density": dens,
                                  "n_gpus": ws, "heads_per_gpu": hl, "kept_blocks": int(kept), "ms": round(ms, 4),
                                  "tflops": round(tf, 1), "frac": round(tf / (mixed * ws), 4),
                                  "peak_note": f"mixed peak {mixed:.0f} TF/s per GPU: bf16 {bf16_peak:.0f} "
                                               f"({peak_src}), int8 {int8_peak:.0f} (measured); frac against "
                                               f"{ws} x that"}), flush=True)
            del lists, counts, m, out
        del q8, qs, k8, ks, v16
        torch.cuda.empty_cache()
    if ws > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def run_model(args):
    """The whole VGGT-1B-shaped aggregator (random init, bf16): patch encoder,
    24 frame + 24 global blocks, intermediates at 4/11/17/23, on uniform
    [0, 1) images of 518 x 518.  Global attention through the package's
    apply_ress (HeSS budget from synthetic log-normal tables, lambda 0.5,
    restore-swap 5 rounds).  Under torchrun the views are sharded: frame
    blocks stay local and each global block all-gathers K/V with NCCL."""
    import tempfile

    from ress_b200 import api, shard as SH, synth, vggt, wiring

    ws, rank, local = _dist()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if ws > 1:
        import torch.distributed as dist
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
    N = args.frames
    if N % ws:
        raise SystemExit(f"{N} views do not split over {ws} GPUs")
    nl = N // ws
    torch.manual_seed(0)
    model = vggt.VGGTAggregatorModel().to(device=device, dtype=torch.bfloat16).eval()
    g = torch.Generator(device=device).manual_seed(1)
    images = torch.rand(1, N, 3, 518, 518, device=device, generator=g)[:, rank * nl:(rank + 1) * nl].contiguous()
    stream = torch.cuda.current_stream(device)

    def barrier():
        if ws > 1:
            torch.distributed.barrier()

    dense_ms = None
    if ws == 1:
        with torch.inference_mode():
            def dense_step():
                model(images)
            for _ in range(2):
                dense_step()
            torch.cuda.synchronize()
            dense_ms = _time_region(dense_step, max(2, min(args.steps, 5)), stream) / max(2, min(args.steps, 5))

    tables = tempfile.mkdtemp(prefix="ress_tables_")
    torch.save(synth.fisher_table(24, 16, seed=1), os.path.join(tables, "fisher_scores_vggt_cam_pos.pt"))
    torch.save(synth.fisher_table(24, 16, seed=3), os.path.join(tables, "fisher_scores_vggt_pcd.pt"))
    os.environ["RESS_CALIBRATION_DIR"] = tables
    wiring.wire_ress_attention(model, model.aggregator.global_blocks, num_special_tokens=5)
    model._ress_backbone = "vggt"
    api.apply_ress(model, sparse_ratio=SPARSE_RATIO, n_iters=5)
    for blk in model.aggregator.global_blocks:
        blk.attn.ress_shape = {"H": 37, "W": 37, "N": nl}  # token split without a host read of pos
    if ws > 1:
        geom = SH.ViewGeom(N, 5, 1369, ws, rank)
        gather = SH.make_view_gather(ws)
        for blk in model.aggregator.global_blocks:
            blk.attn.ress_view = (geom, gather)

    with torch.inference_mode():
        def step():
            model(images, first_frame=(rank == 0))
        for _ in range(max(2, min(args.warmup, 3))):
            step()
        torch.cuda.synchronize()
        barrier()
        steps = max(2, min(args.steps, 10))
        with Clocks(local) as clk:
            ms = _time_region(step, steps, stream)
        torch.cuda.synchronize()
    t = torch.tensor([ms], device=device)
    if ws > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms = float(t.item()) / steps
    split = _model_op_split(model, images, rank, stream) if ws == 1 else None
    if rank == 0:
        line = {"metric": "VGGT aggregator views/s", "value": N / (ms / 1e3), "unit": UNIT, "n_gpus": ws,
                "steps": steps, "warmup": max(2, min(args.warmup, 3)), "ms_per_step": ms,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (uniform [0,1) images, random-init weights)",
                "config": {"workload": f"VGGT-1B-shaped aggregator, {N} views of 518x518, apply_ress("
                                       f"sparse_ratio={SPARSE_RATIO}, n_iters=5), HeSS lambda 0.5",
                           "parallelism": f"views over {ws} GPU(s)" + (", NCCL all-gather of K/V per global block"
                                                                        if ws > 1 else "")},
                "dense_global_ms_per_step": dense_ms,
                "dense_global_note": "the same model with exact dense attention (torch SDPA) in the 24 global "
                                     "blocks instead of apply_ress",
                "op_split_ms": split,
                "clocks": clk.summary()}
        print(json.dumps(line), flush=True)
    if ws > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def _model_op_split(model, images, rank, stream):
    """Device time of one aggregator forward by part: CUDA events around the
    patch encoder and around each block's attention, MLP and the rest of the
    block (norms, layer scales, residuals), summed per block kind."""
    agg = model.aggregator
    spans = []

    def wrap(mod, name):
        def pre(_m, _a):
            e = torch.cuda.Event(enable_timing=True)
            e.record(stream)
            spans.append([name, e, None])

        def post(_m, _a, _o):
            for sp in reversed(spans):
                if sp[0] == name and sp[2] is None:
                    e = torch.cuda.Event(enable_timing=True)
                    e.record(stream)
                    sp[2] = e
                    break
        return [mod.register_forward_pre_hook(pre), mod.register_forward_hook(post)]

    hooks = wrap(agg.patch_embed, "patch_encoder")
    for kind, blocks in (("frame", agg.frame_blocks), ("global", agg.global_blocks)):
        for blk in blocks:
            hooks += wrap(blk, f"{kind}_block")
            hooks += wrap(blk.attn, f"{kind}_attention")
            hooks += wrap(blk.mlp, f"{kind}_mlp")
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.inference_mode():
        e0.record(stream)
        model(images, first_frame=(rank == 0))
        e1.record(stream)
    torch.cuda.synchronize()
    for h in hooks:
        h.remove()
    tot = {}
    for name, a, b in spans:
        tot[name] = tot.get(name, 0.0) + a.elapsed_time(b)
    out = {"total": round(e0.elapsed_time(e1), 2), "patch_encoder": round(tot.get("patch_encoder", 0.0), 2)}
    for kind in ("frame", "global"):
        blk, att, mlp = (tot.get(f"{kind}_{x}", 0.0) for x in ("block", "attention", "mlp"))
        out[f"{kind}_attention"] = round(att, 2)
        out[f"{kind}_mlp"] = round(mlp, 2)
        out[f"{kind}_norms_residuals"] = round(blk - att - mlp, 2)
    out["other"] = round(out["total"] - out["patch_encoder"] - sum(out[f"{k}_{x}"] for k in ("frame", "global")
                                                                    for x in ("attention", "mlp", "norms_residuals")), 2)
    out["note"] = "one extra forward with CUDA events around each part (eager; events add small gaps)"
    return out


def profile_select():
    """The selection kernels at the shapes the reference's Triton kernels are
    timed on in its sources: top-m masks over 16 x 810 rows of 1,619
    candidates (src/ress/scoring/fused_topm.py:127-131: 0.344 ms) and one
    restore-swap round over 16 x 128 rows of 4,096 / 6,476 / 8,192
    candidates (src/ress/scoring/fused_round.py:55-62: 0.398 / 2.481 / 1.707
    ms).  Those Triton kernels are not run here: the reference tree is not on
    the GPU box.  CUDA-event time per call, median of 20 after 3 warm-ups;
    one JSON line per shape."""
    from ress_b200 import kernels as K

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)

    def timed(fn):
        for _ in range(3):
            fn()
        ts = []
        for _ in range(20):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            e1.synchronize()
            ts.append(e0.elapsed_time(e1))
        return sorted(ts)[len(ts) // 2]

    rows, n = 16 * 810, 1619
    q = torch.rand(rows, n, device=dev, generator=g)
    cnt = torch.randint(0, n + 1, (rows,), device=dev, generator=g, dtype=torch.int32)
    ms = timed(lambda: K.top_m_mask(q, cnt))
    print(json.dumps({"kernel": "ress_top_m_mask", "rows": rows, "n": n, "dtype": "f32", "ms": round(ms, 4),
                      "reference_triton_ms_quoted": 0.344,
                      "bytes_GBs": round((rows * n * 5) / (ms / 1e3) / 1e9, 1)}), flush=True)
    for n, quoted in ((4096, 0.398), (6476, 2.481), (8192, 1.707)):
        rows = 16 * 128
        P = torch.rand(rows, n, device=dev, generator=g).bfloat16()
        tk = torch.rand(rows, n, device=dev, generator=g).bfloat16()
        ssq = (torch.rand(rows, n, device=dev, generator=g) * 0.01).bfloat16()
        tq = torch.rand(rows, device=dev, generator=g)
        drop = torch.rand(rows, n, device=dev, generator=g) < 0.5
        pic = torch.randint(1, 64, (rows,), device=dev, generator=g, dtype=torch.int32)
        gn = torch.rand(rows, device=dev, generator=g)
        km = torch.rand(rows, device=dev, generator=g) + 1.0
        ms = timed(lambda: K.round_step(P, tk, ssq, tq, drop, pic, True, True, g_norm_sq=gn, kept_mass=km))
        print(json.dumps({"kernel": "ress_round_step", "rows": rows, "n": n, "dtype": "bf16", "ms": round(ms, 4),
                          "reference_triton_ms_quoted": quoted,
                          "bytes_GBs": round((rows * n * 8) / (ms / 1e3) / 1e9, 1)}), flush=True)


def profile_dense():
    """The dense bf16 attention kernel on one frame-attention layer of the
    32-view aggregator (32 frames x 16 heads = 512 sequences of 1,374 tokens)
    and on the global layer's special-token queries (16 heads x 160 queries
    over 43,968 keys); TFLOP/s (4 * Tq * Tk * 64 per sequence) by CUDA
    events, beside torch's SDPA on the same inputs."""
    from ress_b200 import kernels as K

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    bf16_peak, _, peak_src = _peaks()
    for name, S, Tq, Tk in (("frame", 512, 1374, 1374), ("special", 16, 160, 43968)):
        q = torch.randn(S, Tq, 64, device=dev, generator=g).bfloat16()
        k = torch.randn(S, Tk, 64, device=dev, generator=g).bfloat16()
        v = torch.randn(S, Tk, 64, device=dev, generator=g).bfloat16()
        out = torch.empty(S, Tq, 64, device=dev, dtype=torch.bfloat16)
        flops = 4.0 * Tq * Tk * 64 * S

        def ours():
            K.dense_attn(q, k, v, out=out)

        def torch_sdpa():
            torch.nn.functional.scaled_dot_product_attention(q.unsqueeze(0), k.unsqueeze(0), v.unsqueeze(0))

        res = {"case": name, "sequences": S, "Tq": Tq, "Tk": Tk}
        for tag, fn in (("ress_dense_attn", ours), ("torch_sdpa", torch_sdpa)):
            for _ in range(3):
                fn()
            ms = _time_region(fn, 20, torch.cuda.current_stream(dev)) / 20
            res[f"{tag}_ms"] = round(ms, 4)
            res[f"{tag}_tflops"] = round(flops / (ms / 1e3) / 1e12, 1)
        K.check_status(dev)
        res["frac_of_bf16_peak"] = round(res["ress_dense_attn_tflops"] / bf16_peak, 3)
        res["peak_note"] = f"bf16 burst {bf16_peak:.0f} TF/s ({peak_src})"
        print(json.dumps(res), flush=True)


def profile_attn():
    """Small case for ncu: a 24-frame layer (int8 Q/K + fp16 V = 135 MB,
    above the 126 MB L2; under 1 GB on the device), two layers."""
    from ress_b200 import layer as LY

    S = _setup(24, 1, 0, torch.device("cuda", 0))
    for _ in range(2):
        LY.global_layer(S["q"], S["k"], S["v"], S["L"], S["budget"], S["order"])
    torch.cuda.synchronize()


def profile_score():
    """Scoring passes for ncu: the cfg2 layer's Q pass and K/V passes (pooled
    means, int8 Q and K, fp16 V, key mean), three times each; CUDA-event
    times of the third printed."""
    from ress_b200 import kernels as K

    dev = torch.device("cuda", 0)
    S = _setup(N_FRAMES, 1, 0, dev)
    L = S["L"]
    ws = K.workspace(dev, L.B * L.H, L.Tp, L.Tk, L.n_cand)
    for i in range(3):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        torch.cuda._sleep(20_000_000)
        ev[0].record()
        K.pool_quant_q(S["q"], L)
        ev[1].record()
        K.pool_quant_kv(S["k"], S["v"], L, ws=ws)
        ev[2].record()
        ev[2].synchronize()
    q_ms, kv_ms = ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2])
    mb = 1e6
    print(f"Q pass {q_ms * 1e3:.1f} us, K/V passes {kv_ms * 1e3:.1f} us; algorithmic bytes "
          f"(Q, K, V read once + int8 Q, K written) {SCORE_BYTES(L) / mb:.0f} MB -> "
          f"{SCORE_BYTES(L) / ((q_ms + kv_ms) * 1e-3) / 1e9:.0f} GB/s", flush=True)


def SCORE_BYTES(L):
    """Algorithmic bytes of the scoring passes: Q, K, V (bf16) read once and
    int8 Q and K written (pooled means and scales are < 2 %)."""
    n = L.B * L.H * 64
    return n * (L.Tp * 2 + L.Tk * 2 * 2) + n * (L.Tp + L.Tk)


def profile_rs(frames=N_FRAMES):
    """Restore-swap phase split for ncu: the layer's restore-swap (cfg2 by
    default, --frames for others) run as (rounds, track-best) = (0, off),
    (0, on), (5, on), (1, off), one launch each after a warm-up pass, with
    CUDA-event times printed."""
    from ress_b200 import kernels as K

    dev = torch.device("cuda", 0)
    S = _setup(frames, 1, 0, dev)
    L = S["L"]
    qbar, _, _ = K.pool_quant_q(S["q"], L)
    kbar, vbar, _, _, _, _ = K.pool_quant_kv(S["k"], S["v"], L)
    af, ac = K.predict(qbar, kbar, L.n_cand)
    base = K.baseline(ac, SPARSE_RATIO).view(1, L.H, L.nq)
    nts = K.hess_adjust(base, S["budget"].scores_norm, L.n_cand, min_clamp=2).view(-1)
    M = S["order"].M
    runs = [(0, False), (0, True), (5, True), (1, False)]

    def rs(n, tb):
        K.restore_swap(af, vbar, M, nts, L.n_cand, n_iters=n, track_best=tb, sink_blocks=L.sink_blocks)

    for n, tb in runs:
        rs(n, tb)
    torch.cuda.synchronize()
    for n, tb in runs:
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        ev[0].record()
        rs(n, tb)
        ev[1].record()
        ev[1].synchronize()
        print(f"restore_swap rounds={n} track_best={int(tb)}: {ev[0].elapsed_time(ev[1]):.4f} ms", flush=True)


def main():
    args = _args()
    global SPARSE_RATIO
    if args.sparse_ratio is not None:
        SPARSE_RATIO = args.sparse_ratio
    if args.profile_attn:
        profile_attn()
        return
    if args.profile_rs:
        profile_rs(args.frames)
        return
    if args.profile_select:
        profile_select()
        return
    if args.profile_dense:
        profile_dense()
        return
    if args.profile_score:
        profile_score()
        return
    if args.sweep:
        run_sweep(args)
        return
    if args.model == "vggt" and args.impl == "ress":
        run_model(args)
        return
    if args.shard == "views" and args.impl == "ress":
        run_views(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ress(args)


if __name__ == "__main__":
    main()
