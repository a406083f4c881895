"""Decode benchmark of the B200 expert-slice backend (one JSON line on rank 0).

Workload: a full decode pass of 48 MoE layers for one
token, hidden 2048, 512 experts with seeded top-10 routing per layer (fresh
every step), Q4_K gate/up and MXFP4 down (the reference's routed layout), all
20 neuron slices split over the N GPUs the way the reference planner splits
them over nodes, and a sum of the partials after every layer (NCCL all-reduce
over NVLink; none at N=1).  Layer l+1 depends on layer l: its input is the
pre-normed residual stream h_{l+1} = h_l + y_l, so layers serialize as in
real decode.  A step = one token through all 48 layers; value = tokens/s of
the whole job (every GPU works on the same token: strong scaling).

--tokens T (BASELINE configs[3] with T=16): T concurrent tokens per step, each
with its own seeded top-10 routing per layer; one launch per layer serves the
union of their experts.  value = T x steps/s.

--prefill: one MoE layer for 512 tokens with Zipf(1.1)
expert popularity, MXFP4 gate/up/down, on the tensor-core prefill path
(tcgen05 kind::i8 grouped GEMMs); value = prefill tokens/s.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--tokens T | --prefill] [--impl ours|reference]
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "MoE decode tokens/s at 1/2/4/8 B200; expert-weight GB/s vs HBM peak"
HIDDEN, LAYERS, SLICES, TOPK = 2048, 48, 20, 10
SEED = 0x5EED
POOL = 64
SLICE_BYTES = 2 * 32 * (HIDDEN // 256) * 144 + HIDDEN * 17     # 108,544 (Q4_K gate/up + MXFP4 down)
# --formats: the routed block formats of the pass.  q4k-mxfp4 is the
# reference's own layout (configs[0], [2], [3]); mxfp4-q80 is configs[1]'s
# (MXFP4 gate/up, Q8_0 down: 139,264 B a slice).
FORMATS = {"q4k-mxfp4": (12, 39, "Q4_K gate/up, MXFP4 down"),
           "mxfp4-q80": (39, 8, "MXFP4 gate/up, Q8_0 down")}
FMT = "q4k-mxfp4"


def set_formats(name):
    global FMT, SLICE_BYTES
    FMT = name
    gt, dt, _ = FORMATS[name]
    row = {12: HIDDEN // 256 * 144, 39: HIDDEN // 32 * 17, 8: HIDDEN // 32 * 34}
    SLICE_BYTES = 2 * 32 * row[gt] + HIDDEN * (17 if dt == 39 else 34)


def workload(tokens):
    fmt = FORMATS[FMT][2]
    if tokens == 1:
        if FMT != "q4k-mxfp4":
            return ("decode48 in BASELINE configs[1]'s formats: 48 MoE layers, 1 token, d=2048, 512 experts top-10, "
                    "%s, 20 slices split over the GPUs (1/2/4/8), partial sum after every layer" % fmt)
        return ("decode48 (BASELINE configs[2]): 48 MoE layers, 1 token, d=2048, 512 experts top-10, "
                "%s, 20 slices split over the GPUs, partial sum after every layer" % fmt)
    return ("decode48x%d (BASELINE configs[3]): 48 MoE layers, %d concurrent tokens with independent top-10 "
            "routing (one launch per layer over the union of their experts), d=2048, 512 experts, %s, "
            "20 slices split over the GPUs, partial sum after every layer" % (tokens, tokens, fmt))


_out = sys.stdout


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def emit(line):
    # numpy scalars print as plain numbers
    print(json.dumps(line, default=lambda o: o.item() if hasattr(o, "item") else str(o)), file=_out, flush=True)


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback 6.65 TB/s (MEASURED_PEAKS.json absent)"


def step_routing(steps, tokens=1):
    """Routing and gates for every (step, layer, token) and the tokens' x0 per
    step: the same seeds the CPU baseline harness uses (oracle/ref_bench.c).
    Shapes [steps][48][T][10], [steps][48][T][11], [steps][T][2048]."""
    import fronk_b200 as fb
    ex = np.zeros((steps, LAYERS, tokens, TOPK), np.uint16)
    gt = np.zeros((steps, LAYERS, tokens, 11), np.float32)
    x0 = np.zeros((steps, tokens, HIDDEN), np.float32)
    for s in range(steps):
        for l in range(LAYERS):
            e, g, x = fb.synth_request(HIDDEN, tokens, fb.rand64(SEED, 1000003 * s + l))
            ex[s, l], gt[s, l] = e, g
            if l == 0:
                x0[s] = x
    return ex, gt, x0


# ---------------------------------------------------------------- clocks

class ClockSampler:
    """SM clock, power and clock-event (throttle) reasons of one GPU, queried
    in-process through NVML every millisecond from a thread started before
    set-up (queries only; nothing is set).  mark_start / mark_end bracket the
    timed region; the summary uses the samples inside it (at least the last
    few before mark_end when the region is shorter than a sampling period).
    Falls back to nvidia-smi (200 ms) when NVML cannot be loaded."""

    NAMES = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
             ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
             ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
             ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"),
             ("hw_power_brake", "nvmlClocksEventReasonHwPowerBrakeSlowdown"))

    def __init__(self, device):
        self.device, self.rows, self.stop_flag, self.t = device, [], False, None
        self.t_start = self.t_end = None
        self.source = "nvml"

    def start(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.hnd = pynvml.nvmlDeviceGetHandleByIndex(self.device)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.hnd, pynvml.NVML_CLOCK_SM)
            self.bits = {n: getattr(pynvml, c, 0) for n, c in self.NAMES}
        except Exception:  # noqa: BLE001
            self.nv = None
            self.source = "unavailable"
            return
        self.t = threading.Thread(target=self._poll, daemon=True)
        self.t.start()

    def _poll(self):
        nv, h = self.nv, self.hnd
        while not self.stop_flag:
            try:
                self.rows.append((time.perf_counter(), nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM),
                                  nv.nvmlDeviceGetCurrentClocksEventReasons(h),
                                  nv.nvmlDeviceGetPowerUsage(h) / 1000.0))
            except Exception:  # noqa: BLE001
                pass
            time.sleep(0.001)

    def mark_start(self):
        self.t_start = time.perf_counter()

    def mark_end(self):
        self.t_end = time.perf_counter()

    def stop(self):
        self.stop_flag = True
        if self.t:
            self.t.join(timeout=2)
        if self.nv is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "source": self.source}
        lo, hi = self.t_start or 0.0, self.t_end or float("inf")
        rows = [r for r in self.rows if lo <= r[0] <= hi]
        if len(rows) < 3:  # a region shorter than a few polls: the polls closest before its end
            before = [r for r in self.rows if r[0] <= hi]
            rows = before[-3:]
        reasons = sorted({n for r in rows for n, b in self.bits.items() if b and r[2] & b})
        sms = [r[1] for r in rows]
        try:
            self.nv.nvmlShutdown()
        except Exception:  # noqa: BLE001
            pass
        return {"sm_mhz": statistics.median(sms) if sms else None, "sm_max_mhz": self.max_mhz,
                "sm_mhz_min": min(sms) if sms else None, "power_w_max": max((r[3] for r in rows), default=None),
                "reasons": reasons, "samples": len(rows), "source": "nvml in-process, 1 ms polls in the timed region"}


# ------------------------------------------------------------ CPU baseline

def cpu_baseline(steps, warmup, tokens=1):
    """The reference's own AVX2 backend (compiled from its sources into
    oracle/_ref) on the same seeded workload, all host threads it tunes to
    (bursts of at most 8 tokens per call, the reference's FR_MAX_BURST)."""
    exe = os.path.join(ROOT, "oracle", "_ref", "ref_bench_2048")
    if not os.path.exists(exe):
        return {"unavailable": "reference not compiled (oracle/_ref/ref_bench_2048 missing)"}
    t0 = time.time()
    out = subprocess.run([exe, "avx2", str(SLICES), str(POOL), str(steps), str(warmup), str(SEED), str(tokens)],
                         capture_output=True, text=True, timeout=1800)
    if out.returncode:
        return {"unavailable": "ref_bench failed: " + out.stderr.strip()[-200:]}
    r = json.loads(out.stdout.strip().splitlines()[-1])
    tok_s = tokens * 1e9 / r["ns_per_pass_mean"]
    return {"value": tok_s, "unit": "tokens/s", "cores": r["workers"], "kind": "reference",
            "sample": "reference backends/avx2.c (fr_avx2.run), full workload: all 20 slices resident in sparse "
                      "host units, %d timed 48-layer passes of %d token(s) after %d warm-up, d=2048 build"
                      % (steps, tokens, warmup) + (
                          "; the reference's unit layout fixes routed gate/up rows to Q4_K and down rows to MXFP4, "
                          "so its pass runs the same routing over that layout" if FMT != "q4k-mxfp4" else ""),
            "host": {"cpu": r["cpu"], "cores": r["cores"], "logical_cores": r["logical_cores"]},
            "ms_per_pass": r["ns_per_pass_mean"] / 1e6, "wall_s": round(time.time() - t0, 1)}


def run_reference(args, rank):
    set_formats(args.formats)
    if rank != 0:
        return
    if args.prefill:
        steps, warm = max(1, min(args.steps, 5)), max(3, min(args.warmup, 5))
        cb = prefill_cpu_baseline(steps, warm)
        if "unavailable" in cb:
            emit({"impl": "reference", "unavailable": cb["unavailable"]})
            return
        emit({"impl": "reference", "metric": PF_METRIC, "value": cb["value"], "unit": "tokens/s",
              "n_gpus": args.gpus, "steps": steps, "warmup": warm, "ms_per_step": cb["ms_per_pass"],
              "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8",
              "data": "synthetic", "config": prefill_config(args.gpus), "cpu_baseline": cb,
              "e2e": {"value": cb["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})
        return
    # the same warm-up as this build's arm (which runs at least 3); steps capped
    # so the CPU arm ends within minutes
    steps = max(1, min(args.steps, 50 if args.tokens == 1 else 3))
    warm = max(3, min(args.warmup, 10))
    cb = cpu_baseline(steps, warm, args.tokens)
    if "unavailable" in cb:
        emit({"impl": "reference", "unavailable": cb["unavailable"]})
        return
    line = {"impl": "reference", "metric": METRIC, "value": cb["value"], "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": steps, "warmup": warm, "ms_per_step": cb["ms_per_pass"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic", "config": config(args.gpus, tokens=args.tokens),
            "cpu_baseline": cb, "e2e": {"value": cb["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                                        "d2h_bytes_per_step": 0}}
    emit(line)


def config(n, reduce="peer", tokens=1, unique_per_layer=TOPK):
    from fronk_b200.planner import equal_shares
    step_bytes = LAYERS * unique_per_layer * SLICES * SLICE_BYTES
    return {"workload": workload(tokens), "hidden": HIDDEN, "layers": LAYERS, "tokens_per_step": tokens,
            "experts": 512, "top_k": TOPK, "slices": SLICES, "shares": equal_shares(n),
            "formats": FORMATS[FMT][2], "activations": "Q8 per 64 (src/q4.c scheme), exact block terms "
                                                        "summed in double (gate/up), fp32 down terms",
            "unique_experts_per_layer": unique_per_layer, "weight_bytes_per_step": int(step_bytes),
            "l2": "inputs larger than L2: %.2f GB of expert weights per step, fresh routing every step"
                  % (step_bytes / 1e9),
            "parallelism": ("slice-split x%d, per-layer sum of the partials %s" %
                            (n, "in the layer kernel over NVLink peer memory" if reduce == "peer" else "by NCCL all-reduce"))
                           if n > 1 else "1 GPU, all slices"}


# ------------------------------------------------------------------- ours

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--tokens", type=int, default=1, choices=range(1, 17), metavar="T",
                    help="concurrent tokens per step (1: configs[2], the headline; 16: configs[3])")
    ap.add_argument("--prefill", action="store_true",
                    help="configs[4]: one layer, 512 tokens, Zipf(1.1) routing, MXFP4, tensor-core prefill path")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--reduce", default="peer", choices=["peer", "nccl"],
                    help="per-layer sum of the GPUs' partials: in-kernel over NVLink peer memory, or NCCL all-reduce")
    ap.add_argument("--formats", default="q4k-mxfp4", choices=sorted(FORMATS),
                    help="routed block formats: q4k-mxfp4 (the reference layout, configs[2]/[3]) or mxfp4-q80 "
                         "(configs[1]: MXFP4 gate/up, Q8_0 down)")
    ap.add_argument("--prefill-gate", default="mxfp4", choices=["mxfp4", "q4k"],
                    help="gate/up rows of the --prefill workload: MXFP4 (configs[4]) or Q4_K (the reference's "
                         "unit layout)")
    ap.add_argument("--act", default="q8", choices=["q8", "avx2"],
                    help="avx2: the decode workload through FRC_ACT_AVX2, the arithmetic of the reference's AVX2 "
                         "backend (host-buffer calls; 1 GPU)")
    ap.add_argument("--avx2-workers", type=int, default=1,
                    help="with --act avx2: the AVX2 backend worker count whose results the mode reproduces")
    ap.add_argument("--profile", action="store_true",
                    help="small case for ncu: 2 layers of every slice loaded (2.2 GB), 5 layer launches "
                         "(with --prefill: one layer, three 512-token calls)")
    args = ap.parse_args()
    set_formats(args.formats)
    set_prefill_gate(args.prefill_gate)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    # stdout carries exactly one JSON line: libraries that print (NCCL's
    # version banner) write to stderr instead
    global _out
    _out = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if args.profile and args.prefill:
        prefill_profile_case()
        return
    if args.profile:
        profile_case()
        return
    args.warmup = max(args.warmup, 3)
    if args.prefill:
        run_prefill_bench(args, rank, world, local)
        return
    if args.act == "avx2":
        run_avx2_bench(args, rank, world, local)
        return

    import torch
    import fronk_b200 as fb
    from fronk_b200.planner import owned_blocks
    from fronk_b200 import build as fbuild
    fbuild.build()

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    blocks = owned_blocks(rank, world)
    gt_, dt_, _ = FORMATS[FMT]
    g = fb.geometry(HIDDEN, LAYERS, gt_, dt_)
    ctx = fb.Context(local, HIDDEN, LAYERS, gt_, dt_)

    # units: a pool of distinct synthetic slices, copied on the device into every slot
    t0 = time.time()
    pool = np.concatenate([fb.synth_slice(g, SEED, i) for i in range(POOL)])
    ctx.pool_load(pool, fb.synth_shared(g, SEED, 1 << 20))
    for b in blocks:
        for l in range(LAYERS):
            ctx.fill_layer(b, l, SEED)
    log("rank %d: blocks %s filled in %.1fs" % (rank, blocks, time.time() - t0))
    # in-box reduce: the layer kernels sum the ranks' partials through each
    # other's inboxes over NVLink (FRC_RUN_PEER); --reduce nccl keeps an NCCL
    # all-reduce after every layer instead
    peer = world > 1 and args.reduce == "peer"
    if peer:
        handles = [None] * world
        dist.all_gather_object(handles, ctx.peer_export(world))
        ctx.peer_attach(rank, world, handles)
    run_flags = fb.RUN_RMSNORM | fb.RUN_OVERLAP | (fb.RUN_PEER if peer else 0)

    total = args.warmup + args.steps
    T = args.tokens
    ex, gt, x0 = step_routing(total, T)
    d_ex = torch.from_numpy(ex.astype(np.int16)).to(dev)          # ids < 512: int16 holds the u16 bits
    d_gt = torch.from_numpy(gt).to(dev)
    d_x0 = torch.from_numpy(x0).to(dev)
    cur_ex = torch.empty((LAYERS, T, TOPK), dtype=torch.int16, device=dev)
    cur_gt = torch.empty((LAYERS, T, 11), dtype=torch.float32, device=dev)
    X0 = torch.empty((T, HIDDEN), dtype=torch.float32, device=dev)
    H = [torch.zeros((T, HIDDEN), dtype=torch.float32, device=dev) for _ in range(2)]
    Y = [torch.zeros((T, HIDDEN), dtype=torch.float32, device=dev) for _ in range(2)]

    def p(t):
        return t.data_ptr()

    def one_pass(stream):
        s = stream.cuda_stream
        for l in range(LAYERS):
            x = X0 if l <= 1 else H[(l - 1) % 2]
            x_add = None if l == 0 else p(Y[(l - 1) % 2])
            x_out = None if l == 0 else p(H[l % 2])
            # consecutive layers overlap: layer l+1 plans and starts its weight copies while
            # layer l (or the all-reduce after it) finishes; it reads x only after that
            ctx.run_device(l, T, p(cur_ex[l]), p(cur_gt[l]), p(x), x_add, x_out, p(Y[l % 2]), fb.ACT_Q8,
                           run_flags, s)
            if dist is not None and not peer:
                dist.all_reduce(Y[l % 2])

    def load_step(s):
        cur_ex.copy_(d_ex[s], non_blocking=True)
        cur_gt.copy_(d_gt[s], non_blocking=True)
        X0.copy_(d_x0[s], non_blocking=True)

    stream = torch.cuda.current_stream()
    # capture one pass in a CUDA graph (launch-bound inner loop); eager if capture fails
    graph = None
    try:
        load_step(0)
        one_pass(stream)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            one_pass(torch.cuda.current_stream())
    except Exception as exc:  # noqa: BLE001
        log("graph capture failed, running eagerly:", exc)
        graph = None
    rc = ctx.status(stream.cuda_stream)
    if rc:
        raise fb.FrcError(rc, "warm-up pass", ctx.last_error)

    def step(s):
        load_step(s)
        if graph is not None:
            graph.replay()
        else:
            one_pass(stream)

    sampler = ClockSampler(local)
    sampler.start()
    for s in range(args.warmup):
        step(s)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler.mark_start()
    start.record(stream)
    for s in range(args.warmup, total):
        step(s)
    end.record(stream)
    torch.cuda.synchronize()
    sampler.mark_end()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = start.elapsed_time(end)
    rc = ctx.status(stream.cuda_stream)
    if rc:
        raise fb.FrcError(rc, "timed passes", ctx.last_error)
    if dist is not None:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_per_step = ms / args.steps
    tokens_s = T * 1000.0 / ms_per_step
    launches = LAYERS * args.steps
    # distinct experts a launch reads (the union over the step's tokens; 10 at T=1)
    unique = float(np.mean([len(np.unique(ex[s, l])) for s in range(args.warmup, total) for l in range(LAYERS)]))

    # ---- kernel alone: event-bracketed launches on the launching stream
    kt = []
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(LAYERS)]
    for s in range(min(total, 8)):
        load_step(s)
        for l in range(LAYERS):
            ev[l][0].record(stream)
            ctx.run_device(l, T, p(cur_ex[l]), p(cur_gt[l]), p(X0), None, None, p(Y[0]), fb.ACT_Q8,
                           fb.RUN_RMSNORM, stream.cuda_stream)
            ev[l][1].record(stream)
        torch.cuda.synchronize()
        kt += [a.elapsed_time(b) for a, b in ev]
    kernel_ms = statistics.mean(kt)
    bytes_per_launch = unique * len(blocks) * SLICE_BYTES
    peak, peak_src = peaks()
    # average launch duration over the timed region: at N=1 the passes hold
    # nothing but the layer kernel (profiles/layer_kernel_decode48_launches.md);
    # at N>1 it includes the per-layer all-reduce
    launch_us = ms_per_step * 1e3 / LAYERS
    achieved = bytes_per_launch / (launch_us * 1e-6) / 1e9
    alone = bytes_per_launch / (kernel_ms * 1e-3) / 1e9

    # ---- end to end through the C ABI with host buffers (reference-facing call)
    e2e_steps = max(3, min(args.steps, 50))
    e2e = e2e_run(ctx, fb, ex, gt, x0, e2e_steps, dist, dev, peer, T)

    # ---- parity at full size: one layer of the filled units vs the oracle
    # (at N>1 with the in-kernel reduce: the summed y over all 20 slices)
    if world > 1 and peer:
        parity = reduced_parity(ctx, fb, g, pool, rank, world, dist, dev)
    else:
        parity = full_size_parity(ctx, fb, g, pool, blocks)

    used_graph = graph is not None
    del graph
    if rank == 0:
        weight_bytes = LAYERS * unique * SLICES * SLICE_BYTES      # per step, all GPUs
        line = {
            "metric": METRIC, "value": tokens_s, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": config(world, args.reduce, T, unique),
            "weight_gbs": weight_bytes * 1e3 / ms_per_step / 1e9,
            "weight_frac_of_peak": weight_bytes * 1e3 / ms_per_step / 1e9 / peak,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": ncu_traffic(), "peak_source": peak_src,
                         "kernel": "moe_layer_kernel<Q8> (one launch per layer, %d token(s))" % T,
                         "algorithmic_bytes_per_launch": bytes_per_launch, "launch_us": launch_us,
                         "launch_us_source": "CUDA events over the timed passes / launches"
                                             + (" (includes the all-reduce)" if world > 1 else ""),
                         "kernel_alone_us": kernel_ms * 1e3, "kernel_alone_gbs": alone},
            "gpu_launches": launches, "graph": used_graph, "clocks": clocks, "e2e": e2e, "parity": parity,
            "limiter": decode_limiter(bytes_per_launch, peak, launch_us, kernel_ms * 1e3, world, T),
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(3, 1) if T == 1 else cpu_baseline(1, 1, T)
        emit(line)
    ctx.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def decode_limiter(bytes_per_launch, peak, launch_us, alone_us, world, T):
    """What bounds a layer launch, from this run's numbers: the time its
    weight bytes take at the measured HBM peak against the measured launch
    time.  Far above it, a layer is its chain of dependent steps (activation
    pass, gate/up, grid barrier, down terms, reduce) rather than HBM."""
    hbm_us = bytes_per_launch / (peak * 1e9) * 1e6
    if launch_us > 2 * hbm_us:
        what = ("the layer's dependent chain (activation pass, gate/up dot products, grid barrier, down terms, "
                "reduce: latency, %s), not HBM" % ("CUDA-core dot products of %d tokens" % T if T > 1
                                                   else "one token"))
        if world > 1:
            what += "; plus the in-kernel NVLink exchange of the partial rows each layer"
    else:
        what = "HBM bandwidth"
    return {"hbm_time_us": hbm_us, "launch_us": launch_us, "kernel_alone_us": alone_us,
            "launch_over_hbm": launch_us / hbm_us, "bound": what}


def prefill_limiter(stage_ms, gu_bytes, peak, world):
    """The prefill step's split: the tensor-core kernels against their HBM time,
    and the fixed stages (quantize, grouping, combine) that do not shrink with
    the slices a GPU holds."""
    gu_us, dn_us = stage_ms[2] * 1e3, stage_ms[3] * 1e3
    fixed_us = (stage_ms[0] + stage_ms[1] + stage_ms[4]) * 1e3
    hbm_us = gu_bytes / (peak * 1e9) * 1e6
    what = ("CUDA-core work around the MMAs in the gate/up kernel (exact block terms, SwiGLU, Q8 of the hidden "
            "slices) and the operand conversion; tensor pipe and HBM are mostly idle")
    if world > 1:
        what += "; the fixed stages and the NCCL all-reduce of the 4 MB partial grow as a share with N"
    return {"gate_up_us": gu_us, "gate_up_hbm_time_us": hbm_us, "down_us": dn_us, "fixed_stages_us": fixed_us,
            "bound": what}


def e2e_run(ctx, fb, ex, gt, x0, steps, dist, dev, peer=False, T=1, act=None):
    """tokens/s through the public call with host buffers: per layer the
    request is copied in, the layer runs, y is copied out (frc_run; at N>1
    the device entry point plus the all-reduce)."""
    act = fb.ACT_Q8 if act is None else act
    import torch
    h2d = LAYERS * T * (HIDDEN * 4 + TOPK * 2 + 11 * 4)
    d2h = LAYERS * (T * HIDDEN * 4 + (16 if dist is None else 0))  # y (+ the status word frc_run reads with it)
    if dist is None or peer:
        # the layer loop in C over the host-buffer call (frc_host_pass_flags ->
        # frc_run_flags per layer; at N>1 each rank holds its share of the
        # slices and the kernel sums every layer over the ranks: FRC_RUN_PEER)
        hs = [np.ascontiguousarray(x0[s], np.float32).copy() for s in range(steps)]
        es = [np.ascontiguousarray(ex[s], np.uint16) for s in range(steps)]
        flags = fb.RUN_PEER if dist is not None else 0
        if dist is not None:
            dist.barrier()
        t0 = time.perf_counter()
        for s in range(steps):
            ctx.host_pass(0, es[s], gt[s], hs[s], act, flags)
        dt = time.perf_counter() - t0
        if dist is not None:
            t = torch.tensor([dt], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            dt = float(t.item())
    else:
        pin_x = torch.empty((T, HIDDEN), dtype=torch.float32).pin_memory()
        pin_e = torch.empty((T, TOPK), dtype=torch.int16).pin_memory()
        pin_g = torch.empty((T, 11), dtype=torch.float32).pin_memory()
        pin_y = torch.empty((T, HIDDEN), dtype=torch.float32).pin_memory()
        dx, de, dg = torch.empty((T, HIDDEN), device=dev), torch.empty((T, TOPK), dtype=torch.int16, device=dev), \
            torch.empty((T, 11), device=dev)
        dy = torch.empty((T, HIDDEN), device=dev)
        st = torch.cuda.current_stream()
        dist.barrier()
        t0 = time.perf_counter()
        for s in range(steps):
            h = x0[s].copy()
            for l in range(LAYERS):
                x = (h / np.sqrt(np.mean(h * h, axis=-1, keepdims=True) + np.float32(1e-6))).astype(np.float32)
                pin_x.numpy()[:] = x
                pin_e.numpy()[:] = ex[s, l].astype(np.int16)
                pin_g.numpy()[:] = gt[s, l]
                dx.copy_(pin_x, non_blocking=True)
                de.copy_(pin_e, non_blocking=True)
                dg.copy_(pin_g, non_blocking=True)
                ctx.run_device(l, T, de.data_ptr(), dg.data_ptr(), dx.data_ptr(), None, None, dy.data_ptr(),
                               fb.ACT_Q8, fb.RUN_PEER if peer else 0, st.cuda_stream)
                if not peer:
                    dist.all_reduce(dy)
                pin_y.copy_(dy, non_blocking=True)
                st.synchronize()
                h = h + pin_y.numpy()
        dt = time.perf_counter() - t0
        t = torch.tensor([dt], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dt = float(t.item())
    rc = ctx.status(None)
    if rc:
        raise fb.FrcError(rc, "e2e", ctx.last_error)
    return {"value": T * steps / dt, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "steps": steps, "api": "frc_host_pass: frc_run per layer (host buffers, synchronous)" if dist is None else
            ("frc_host_pass_flags(FRC_RUN_PEER): frc_run_flags per layer on every rank, host buffers, the "
             "in-kernel NVLink reduce" if peer else
             "frc_run_device + NCCL all_reduce, pinned host copies each layer")}


def run_avx2_bench(args, rank, world, local):
    """The decode workload through FRC_ACT_AVX2 (fronk_b200/csrc/frc_avx2.cuh),
    the arithmetic of the reference's AVX2 backend: one GPU, all 20 slices of
    48 Q4_K/MXFP4 layers.  value: tokens/s of the device work of a pass, the
    CUDA-event durations of each layer call's three launches (activation
    quantization, one CTA a (block, expert) job, the worker-ordered
    reduction) summed over the 48 layers; e2e: frc_host_pass with host
    buffers, the call this mode is used through.  Parity: one full-size
    layer against the oracle's restatement at the same worker count."""
    import torch
    import fronk_b200 as fb
    from fronk_b200 import build as fbuild
    if world > 1 or FMT != "q4k-mxfp4":
        raise SystemExit("--act avx2: one GPU, the reference's native layout (--formats q4k-mxfp4)")
    fbuild.build()
    torch.cuda.set_device(local)
    blocks = list(range(SLICES))
    g = fb.geometry(HIDDEN, LAYERS, fb.Q4_K, fb.MXFP4)
    ctx = fb.Context(local, HIDDEN, LAYERS, fb.Q4_K, fb.MXFP4)
    pool = np.concatenate([fb.synth_slice(g, SEED, i) for i in range(POOL)])
    ctx.pool_load(pool, fb.synth_shared(g, SEED, 1 << 20))
    for b in blocks:
        for l in range(LAYERS):
            ctx.fill_layer(b, l, SEED)
    ctx.set_avx2_workers(args.avx2_workers)
    ctx.avx2_timing(True)
    T = args.tokens
    steps = max(3, min(args.steps, 20))
    total = args.warmup + steps
    ex, gt, x0 = step_routing(total, T)
    stage = []
    sampler = ClockSampler(local)
    sampler.start()
    for s in range(total):
        if s == args.warmup:
            sampler.mark_start()
        for l in range(LAYERS):
            rc, _ = ctx.run(l, ex[s, l], gt[s, l], x0[s], fb.ACT_AVX2)
            if rc:
                raise fb.FrcError(rc, "avx2 run", ctx.last_error)
            if s >= args.warmup:
                stage.append(ctx.avx2_times())
    sampler.mark_end()
    clocks = sampler.stop()
    stage = np.array(stage, np.float64)                      # [steps * layers][3] ms
    layer_ms = stage.sum(axis=1).mean()
    ms_per_step = layer_ms * LAYERS
    unique = float(np.mean([len(np.unique(ex[s, l])) for s in range(args.warmup, total) for l in range(LAYERS)]))
    bytes_per_launch = unique * len(blocks) * SLICE_BYTES
    job_ms = stage[:, 1].mean()
    peak, peak_src = peaks()
    achieved = bytes_per_launch / (job_ms * 1e-3) / 1e9
    e2e = e2e_run(ctx, fb, ex, gt, x0, max(3, min(args.steps, 20)), None, None, False, T, act=fb.ACT_AVX2)
    # parity: one full-size layer of the filled units against the restatement
    from oracle import Oracle
    orc = Oracle()
    e, gte, x = fb.synth_request(HIDDEN, 2, 777)      # no shared gate: the host copies hold routed slices
    layers = _host_layers(fb, g, pool, blocks, e)
    m = orc.model(HIDDEN, fb.Q4_K, fb.MXFP4, layers)
    rc, y = ctx.run(5, e, gte, x, fb.ACT_AVX2)
    rc2, want = orc.avx2_run(m, e, gte, x, workers=args.avx2_workers, libm_expf=False)
    parity = {"vs": "or_avx2_run (oracle restatement of backends/avx2.c, same worker count and exp form)",
              "layer": 5, "tokens": 2, "blocks": len(blocks),
              "bitwise_equal": bool(rc == rc2 == 0 and np.array_equal(np.asarray(y, np.float32).view(np.uint32),
                                                                      want.view(np.uint32))),
              "max_rel_l2": _rel(want, y) if rc == rc2 == 0 else None}
    if rank == 0:
        cfg = config(1, tokens=T, unique_per_layer=unique)
        cfg["activations"] = ("FRC_ACT_AVX2: the reference AVX2 backend's quantize8 (int8 per 256, int16 sums "
                              "per 32), its fp32 lane order, jobs dealt to %d worker(s)" % args.avx2_workers)
        line = {
            "metric": METRIC + " (FRC_ACT_AVX2)", "value": T * 1000.0 / ms_per_step, "unit": "tokens/s",
            "n_gpus": 1, "steps": steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic", "config": cfg,
            "value_source": "sum over the 48 layer calls of the CUDA-event durations of their three launches",
            "stage_us": {"quantize": stage[:, 0].mean() * 1e3, "jobs": job_ms * 1e3,
                         "reduce": stage[:, 2].mean() * 1e3},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": None, "peak_source": peak_src,
                         "kernel": "avx2_job_kernel (one CTA a (block, expert) job)",
                         "algorithmic_bytes_per_launch": bytes_per_launch, "launch_us": job_ms * 1e3},
            "gpu_launches": 4 * LAYERS * steps, "clocks": clocks, "e2e": e2e, "parity": parity,
        }
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(3, 1) if T == 1 else cpu_baseline(1, 1, T)
        emit(line)
    ctx.close()


def _host_layers(fb, g, pool, blocks, experts, layer=5):
    """Host copies of (block, layer) for the given experts, rebuilt from the
    pool the device filled them from (frc_pool_pick)."""
    sb, lb = fb.slice_bytes(g), fb.layer_bytes(g)
    layers = {}
    for b in blocks:
        arr = np.zeros(lb, np.uint8)
        for ident in set(int(v) for v in np.asarray(experts).ravel()):
            k = fb.pool_pick(SEED, b, layer, ident, POOL)
            arr[ident * sb:(ident + 1) * sb] = pool[k * sb:(k + 1) * sb]
        layers[b] = arr
    return layers


def _rel(ref, act):
    return max(float(np.sqrt(((ref[t].astype(np.float64) - act[t]) ** 2).sum() / (ref[t].astype(np.float64) ** 2).sum()))
               for t in range(ref.shape[0]))


def full_size_parity(ctx, fb, g, pool, blocks):
    """Layer 5 of the filled units on a fresh request, against the oracle's
    restatement of the same arithmetic (hidden values bit for bit) and against
    the reference's ref-q8 (or_ref_run, bit-identical to the compiled fr_ref_q8)
    on the host copies of the same slices."""
    try:
        from oracle import Oracle, Q4_K, MXFP4
    except Exception as exc:  # noqa: BLE001
        return {"skipped": str(exc)}
    orc = Oracle()
    e, gate, x = fb.synth_request(HIDDEN, 2, 777)
    rc, y = ctx.run(5, e, gate, x, fb.ACT_Q8)
    if rc:
        return {"error": ctx.last_error}
    h = ctx.debug_hidden()
    layers = _host_layers(fb, g, pool, blocks, e)  # held: the model keeps only their addresses
    m = orc.model(HIDDEN, FORMATS[FMT][0], FORMATS[FMT][1], layers)
    rc, y_ref, h_ref = orc.port_run(m, e, gate, x, want_hidden=True)
    rc2, y_q8 = orc.ref_run(m, e, gate, x, 1)
    return {"layer": 5, "tokens": 2, "blocks": len(blocks), "hidden_bitexact": bool(np.array_equal(
        h.view(np.uint32), h_ref.view(np.uint32))), "max_rel_l2": _rel(y_ref, y),
        "max_rel_l2_vs_ref_q8": _rel(y_q8, y) if rc2 == 0 else None, "tolerance": 1e-5}


def reduced_parity(ctx, fb, g, pool, rank, world, dist, dev):
    """N>1: one layer with the in-kernel NVLink reduce (FRC_RUN_PEER) on every
    rank; rank 0 checks that every rank holds the same y, bit for bit, and
    compares it with the oracle over all 20 slices (the reference's sum of the
    participants' parts, src/plane.c:110-121,325-345)."""
    import torch
    e, gate, x = fb.synth_request(HIDDEN, 2, 778)
    de = torch.from_numpy(e.astype(np.uint16).view(np.int16)).to(dev)
    dg, dx = torch.from_numpy(gate).to(dev), torch.from_numpy(x).to(dev)
    dy = torch.zeros((2, HIDDEN), dtype=torch.float32, device=dev)
    s = torch.cuda.current_stream().cuda_stream
    ctx.run_device(5, 2, de.data_ptr(), dg.data_ptr(), dx.data_ptr(), None, None, dy.data_ptr(), fb.ACT_Q8,
                   fb.RUN_PEER, s)
    rc = ctx.status(s)
    got = [None] * world
    dist.all_gather_object(got, (rc, dy.cpu().numpy()))
    if rank != 0:
        return None
    out = {"reduced": True, "layer": 5, "tokens": 2, "blocks": SLICES, "ranks": world,
           "ranks_status": [int(r[0]) for r in got],
           "ranks_bitwise_equal": all(np.array_equal(got[0][1].view(np.uint32), r[1].view(np.uint32)) for r in got),
           "tolerance": 1e-5}
    try:
        from oracle import Oracle, Q4_K, MXFP4
    except Exception as exc:  # noqa: BLE001
        out["skipped"] = str(exc)
        return out
    orc = Oracle()
    layers = _host_layers(fb, g, pool, range(SLICES), e)  # held: the model keeps only their addresses
    m = orc.model(HIDDEN, FORMATS[FMT][0], FORMATS[FMT][1], layers)
    rc1, y_ref, _ = orc.port_run(m, e, gate, x)
    rc2, y_q8 = orc.ref_run(m, e, gate, x, 1)
    y = got[0][1]
    out["max_rel_l2"] = _rel(y_ref, y) if rc1 == 0 else None
    out["max_rel_l2_vs_ref_q8"] = _rel(y_q8, y) if rc2 == 0 else None
    return out


def profile_case():
    """The layer kernel alone on a small device footprint: layers 0 and 1 of
    all 20 slices (2.2 GB), 5 launches with fresh routing (2 warm-up + 3)."""
    import torch
    import fronk_b200 as fb
    g = fb.geometry(HIDDEN)
    ctx = fb.Context(0, HIDDEN)
    pool = np.concatenate([fb.synth_slice(g, SEED, i) for i in range(POOL)])
    ctx.pool_load(pool, fb.synth_shared(g, SEED, 1 << 20))
    for b in range(SLICES):
        for l in range(2):
            ctx.fill_layer(b, l, SEED)
    ex, gt, x0 = step_routing(5)
    dev = torch.device("cuda", 0)
    x = torch.from_numpy(x0).to(dev)
    y = torch.zeros(HIDDEN, device=dev)
    e = torch.from_numpy(ex.astype(np.int16)).to(dev)
    gg = torch.from_numpy(gt).to(dev)
    s = torch.cuda.current_stream().cuda_stream
    for i in range(5):
        ctx.run_device(i % 2, 1, e[i, i % 2].data_ptr(), gg[i, i % 2].data_ptr(), x[i].data_ptr(), None, None,
                       y.data_ptr(), fb.ACT_Q8, fb.RUN_RMSNORM, s)
    rc = ctx.status(s)
    if rc:
        raise fb.FrcError(rc, "profile case", ctx.last_error)
    ctx.close()
    print("profile case ok")


# ---------------------------------------------------------------- prefill

PF_TOKENS, PF_ZIPF, PF_SETS = 512, 1.1, 8
PF_METRIC = "MoE prefill tokens/s (one layer, 512 tokens) at 1/2/4/8 B200; expert-weight GB/s vs HBM peak"
PF_GATE = "mxfp4"                                # --prefill-gate: configs[4]'s MXFP4, or q4k (the reference units)
PF_GU_BYTES = 2 * 32 * (HIDDEN * 17 // 32)       # 69,632: MXFP4 gate + up rows of one slice
PF_DN_BYTES = HIDDEN * 17                        # 34,816: MXFP4 down rows of one slice
PF_SLICE_BYTES = PF_GU_BYTES + PF_DN_BYTES       # 104,448


def set_prefill_gate(name):
    """Q4_K gate/up rows (144-byte super-blocks: 73,728 B of gate/up rows a
    slice, 108,544 B a slice) or MXFP4 ones."""
    global PF_GATE, PF_GU_BYTES, PF_SLICE_BYTES
    PF_GATE = name
    PF_GU_BYTES = 2 * 32 * (HIDDEN // 256 * 144 if name == "q4k" else HIDDEN * 17 // 32)
    PF_SLICE_BYTES = PF_GU_BYTES + PF_DN_BYTES


def pf_gate_type(fb):
    return fb.Q4_K if PF_GATE == "q4k" else fb.MXFP4


def prefill_config(n, unique=None):
    from fronk_b200.planner import equal_shares
    cfg = {"workload": "prefill512 (BASELINE configs[4]): one MoE layer, 512 tokens x d=2048, top-10 of 512 experts "
                       "with Zipf(1.1) popularity (seeded), MXFP4 gate/up/down, 20 slices split over the GPUs, "
                       "tcgen05 kind::i8 grouped GEMMs, partial sum by NCCL all-reduce at N>1",
           "hidden": HIDDEN, "layers": 1, "tokens_per_step": PF_TOKENS, "experts": 512, "top_k": TOPK,
           "zipf": PF_ZIPF, "slices": SLICES, "shares": equal_shares(n),
           "formats": "Q4_K gate/up, MXFP4 down (the reference's unit layout)" if PF_GATE == "q4k"
                      else "MXFP4 gate/up/down",
           "activations": "bf16 x on the device (FRC_RUN_X_BF16, widened exactly to fp32; the host call frc_run "
                          "takes the same values as fp32, as fr_backend.run does), Q8 per 64 (src/q4.c scheme), "
                          "int8 tensor-core dots of the values and of their dequantization residuals, exact block "
                          "terms summed in double",
           "routing_sets": PF_SETS,
           "parallelism": "slice-split x%d, NCCL all-reduce of the 512 x 2048 partial" % n if n > 1 else "1 GPU, all slices"}
    if unique is not None:
        cfg["unique_experts"] = unique
        cfg["weight_bytes_per_step"] = int(unique * SLICES * PF_SLICE_BYTES)
        cfg["l2"] = "inputs larger than L2: %.2f GB of expert weights per step" % (unique * SLICES * PF_SLICE_BYTES / 1e9)
    return cfg


def prefill_cpu_baseline(steps, warmup):
    """The reference's AVX2 backend on the same routing (512 tokens in bursts
    of 8, Zipf 1.1), one layer of all 20 slices.  The reference's unit layout
    fixes routed gate/up rows to Q4_K (src/native.h:1-3), so it runs the same
    routing and shapes with Q4_K gate/up instead of MXFP4 (1,152 vs 1,088
    bytes a row)."""
    exe = os.path.join(ROOT, "oracle", "_ref", "ref_bench_2048")
    if not os.path.exists(exe):
        return {"unavailable": "reference not compiled (oracle/_ref/ref_bench_2048 missing)"}
    t0 = time.time()
    out = subprocess.run([exe, "avx2", str(SLICES), str(POOL), str(steps), str(warmup), str(SEED), str(PF_TOKENS),
                          str(PF_ZIPF), "1"], capture_output=True, text=True, timeout=1800)
    if out.returncode:
        return {"unavailable": "ref_bench failed: " + out.stderr.strip()[-200:]}
    r = json.loads(out.stdout.strip().splitlines()[-1])
    return {"value": PF_TOKENS * 1e9 / r["ns_per_pass_mean"], "unit": "tokens/s", "cores": r["workers"],
            "kind": "reference",
            "sample": "reference backends/avx2.c (fr_avx2.run), one layer of all 20 slices, 512 tokens with Zipf(1.1) "
                      "routing in bursts of 8, %d timed passes after %d warm-up, d=2048 build, Q4_K gate/up (the "
                      "reference's routed layout; no MXFP4 gate/up backend)" % (steps, warmup),
            "host": {"cpu": r["cpu"], "cores": r["cores"], "logical_cores": r["logical_cores"]},
            "ms_per_pass": r["ns_per_pass_mean"] / 1e6, "wall_s": round(time.time() - t0, 1)}


def run_prefill_bench(args, rank, world, local):
    import torch
    import fronk_b200 as fb
    from fronk_b200.planner import owned_blocks
    from fronk_b200 import build as fbuild
    fbuild.build()
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    blocks = owned_blocks(rank, world)
    MX, GT = fb.MXFP4, pf_gate_type(fb)
    g = fb.geometry(HIDDEN, 1, GT, MX)
    ctx = fb.Context(local, HIDDEN, layers=1, gate_type=GT, down_type=MX)
    pool = np.concatenate([fb.synth_slice(g, SEED, i) for i in range(POOL)])
    ctx.pool_load(pool, fb.synth_shared(g, SEED, 1 << 20))
    for b in blocks:
        ctx.fill_layer(b, 0, SEED)
    # configs[4]'s bf16 activations: x rounded to bf16 once (the fp32 copies
    # hold the same values, for the host call and the parity check)
    reqs = []
    for i in range(PF_SETS):
        e, gt, x = fb.synth_request(HIDDEN, PF_TOKENS, fb.rand64(SEED, 7000 + i), zipf=PF_ZIPF)
        reqs.append((e, gt, torch.from_numpy(x).to(torch.bfloat16).float().numpy()))
    uniq = [len(np.unique(r[0])) for r in reqs]
    d_ex = torch.from_numpy(np.stack([r[0] for r in reqs]).astype(np.int16)).to(dev)
    d_gt = torch.from_numpy(np.stack([r[1] for r in reqs])).to(dev)
    d_x = torch.from_numpy(np.stack([r[2] for r in reqs])).to(dev).to(torch.bfloat16)
    cur_ex = torch.empty_like(d_ex[0]); cur_gt = torch.empty_like(d_gt[0]); cur_x = torch.empty_like(d_x[0])
    Y = torch.zeros((PF_TOKENS, HIDDEN), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream()

    def launch():
        ctx.run_device(0, PF_TOKENS, cur_ex.data_ptr(), cur_gt.data_ptr(), cur_x.data_ptr(), None, None,
                       Y.data_ptr(), fb.ACT_Q8, fb.RUN_X_BF16, torch.cuda.current_stream().cuda_stream)
        if dist is not None:
            dist.all_reduce(Y)

    def load(s):
        cur_ex.copy_(d_ex[s % PF_SETS], non_blocking=True)
        cur_gt.copy_(d_gt[s % PF_SETS], non_blocking=True)
        cur_x.copy_(d_x[s % PF_SETS], non_blocking=True)

    load(0)
    launch()
    torch.cuda.synchronize()
    rc = ctx.status(stream.cuda_stream)
    if rc:
        raise fb.FrcError(rc, "prefill warm-up", ctx.last_error)
    graph = None
    try:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            launch()
    except Exception as exc:  # noqa: BLE001
        log("graph capture failed, running eagerly:", exc)
        graph = None

    def step(s):
        load(s)
        if graph is not None:
            graph.replay()
        else:
            launch()

    sampler = ClockSampler(local)
    sampler.start()
    for s in range(args.warmup):
        step(s)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler.mark_start()
    start.record(stream)
    for s in range(args.warmup, args.warmup + args.steps):
        step(s)
    end.record(stream)
    torch.cuda.synchronize()
    sampler.mark_end()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = start.elapsed_time(end)
    rc = ctx.status(stream.cuda_stream)
    if rc:
        raise fb.FrcError(rc, "timed prefill", ctx.last_error)
    if dist is not None:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_per_step = ms / args.steps
    tokens_s = PF_TOKENS * 1000.0 / ms_per_step
    unique = float(np.mean([uniq[s % PF_SETS] for s in range(args.warmup, args.warmup + args.steps)]))

    # per-kernel durations: events around each of the five stages (seven launches:
    # the MMA stages launch the shared expert's items and the routed ones), eager calls
    ctx.prefill_timing(True)
    stage = []
    for s in range(2 * PF_SETS):
        load(s)
        ctx.run_device(0, PF_TOKENS, cur_ex.data_ptr(), cur_gt.data_ptr(), cur_x.data_ptr(), None, None,
                       Y.data_ptr(), fb.ACT_Q8, fb.RUN_X_BF16, stream.cuda_stream)
        stage.append(ctx.prefill_times())
    ctx.prefill_timing(False)
    stage = np.mean(np.stack(stage[2:]), axis=0)
    names = ["quantize", "group", "gate/up MMA", "down MMA", "combine"]
    u_all = float(np.mean(uniq))
    gu_bytes = u_all * len(blocks) * PF_GU_BYTES
    dn_bytes = u_all * len(blocks) * PF_DN_BYTES
    peak, peak_src = peaks()
    gu_gbs = gu_bytes / (stage[2] * 1e-3) / 1e9
    dn_gbs = dn_bytes / (stage[3] * 1e-3) / 1e9

    # end to end: host buffers through frc_run (N=1) / device call + all-reduce with pinned copies (N>1)
    e2e_steps = max(3, min(args.steps, 20))
    h2d = PF_TOKENS * (HIDDEN * (4 if dist is None else 2) + TOPK * 2 + 11 * 4)
    d2h = PF_TOKENS * HIDDEN * 4 + (16 if dist is None else 0)
    if dist is None:
        # the caller's output buffer is reused from call to call, as a serving
        # loop would (a fresh 4 MB array a call would time its page faults)
        y_out = np.zeros((PF_TOKENS, HIDDEN), np.float32)
        t0 = time.perf_counter()
        for s in range(e2e_steps):
            e, gt, x = reqs[s % PF_SETS]
            rc, _ = ctx.run(0, e, gt, x, out=y_out)
            if rc:
                raise fb.FrcError(rc, "e2e prefill", ctx.last_error)
        dt = time.perf_counter() - t0
    else:
        pin_x = torch.empty((PF_TOKENS, HIDDEN), dtype=torch.bfloat16).pin_memory()
        pin_e = torch.empty((PF_TOKENS, TOPK), dtype=torch.int16).pin_memory()
        pin_g = torch.empty((PF_TOKENS, 11), dtype=torch.float32).pin_memory()
        pin_y = torch.empty((PF_TOKENS, HIDDEN), dtype=torch.float32).pin_memory()
        dist.barrier()
        t0 = time.perf_counter()
        for s in range(e2e_steps):
            e, gt, x = reqs[s % PF_SETS]
            pin_x.copy_(torch.from_numpy(x))  # bf16 words
            pin_e.numpy()[:] = e.astype(np.int16)
            pin_g.numpy()[:] = gt
            cur_x.copy_(pin_x, non_blocking=True)
            cur_ex.copy_(pin_e, non_blocking=True)
            cur_gt.copy_(pin_g, non_blocking=True)
            launch()
            pin_y.copy_(Y, non_blocking=True)
            stream.synchronize()
        dt = time.perf_counter() - t0
        t = torch.tensor([dt], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dt = float(t.item())
    e2e = {"value": PF_TOKENS * e2e_steps / dt, "unit": "tokens/s", "h2d_bytes_per_step": h2d,
           "d2h_bytes_per_step": d2h, "steps": e2e_steps,
           "api": "frc_run (host buffers, synchronous)" if dist is None else
                  "frc_run_device + NCCL all_reduce, pinned host copies"}

    # parity on a sample of tokens of the first routing set (tokens are independent)
    parity = prefill_parity(ctx, fb, g, pool, blocks, reqs[0]) if rank == 0 else None
    used_graph = graph is not None
    del graph
    if rank == 0:
        line = {
            "metric": PF_METRIC, "value": tokens_s, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic", "config": prefill_config(world, unique),
            "weight_gbs": unique * SLICES * PF_SLICE_BYTES * 1e3 / ms_per_step / 1e9,
            "roofline": {"bound": "hbm", "achieved": gu_gbs, "peak": peak, "unit": "GB/s", "frac": gu_gbs / peak,
                         "traffic": ncu_traffic("prefill_mma_kernels_prefill512_full.md") if PF_GATE == "mxfp4"
                         else None, "peak_source": peak_src,
                         "kernel": "prefill_mma_kernel<gate/up%s> (tcgen05 kind::i8)" % (
                             ", Q4_K rows" if PF_GATE == "q4k" else ""),
                         "algorithmic_bytes_per_launch": gu_bytes, "launch_us": float(stage[2] * 1e3),
                         "launch_us_source": "CUDA events around the launch on its stream (eager calls)",
                         "down_kernel": {"bytes": dn_bytes, "us": float(stage[3] * 1e3), "gbs": dn_gbs,
                                         "frac": dn_gbs / peak},
                         "stage_us": {n: float(v * 1e3) for n, v in zip(names, stage)}},
            "gpu_launches": 7 * args.steps, "graph": used_graph, "clocks": clocks,
            "limiter": prefill_limiter(stage, gu_bytes, peak, world),
            "e2e": e2e, "parity": parity,
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = prefill_cpu_baseline(2, 1)
        emit(line)
    ctx.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def prefill_profile_case():
    """The prefill path alone on its bench workload (one layer of all 20
    slices, 1.07 GB on the device): three eager calls of 512 tokens."""
    import torch
    import fronk_b200 as fb
    MX, GT = fb.MXFP4, pf_gate_type(fb)
    g = fb.geometry(HIDDEN, 1, GT, MX)
    ctx = fb.Context(0, HIDDEN, layers=1, gate_type=GT, down_type=MX)
    pool = np.concatenate([fb.synth_slice(g, SEED, i) for i in range(POOL)])
    ctx.pool_load(pool, fb.synth_shared(g, SEED, 1 << 20))
    for b in range(SLICES):
        ctx.fill_layer(b, 0, SEED)
    dev = torch.device("cuda", 0)
    y = torch.zeros((PF_TOKENS, HIDDEN), device=dev)
    s = torch.cuda.current_stream().cuda_stream
    for i in range(3):
        e, gt, x = fb.synth_request(HIDDEN, PF_TOKENS, fb.rand64(SEED, 7000 + i), zipf=PF_ZIPF)
        de = torch.from_numpy(e.astype(np.int16)).to(dev)
        dg = torch.from_numpy(gt).to(dev)
        dx = torch.from_numpy(x).to(dev)
        ctx.run_device(0, PF_TOKENS, de.data_ptr(), dg.data_ptr(), dx.data_ptr(), None, None, y.data_ptr(),
                       fb.ACT_Q8, 0, s)
        torch.cuda.synchronize()
    rc = ctx.status(s)
    if rc:
        raise fb.FrcError(rc, "prefill profile case", ctx.last_error)
    ctx.close()
    print("prefill profile case ok")


def prefill_parity(ctx, fb, g, pool, blocks, req):
    try:
        from oracle import Oracle
    except Exception as exc:  # noqa: BLE001
        return {"skipped": str(exc)}
    e, gt, x = req
    rc, y = ctx.run(0, e, gt, x)
    if rc:
        return {"error": ctx.last_error}
    sample = [0, 5, 100, 300, 511]
    sb = fb.slice_bytes(g)
    layers = {}
    for b in blocks:
        arr = np.zeros(fb.layer_bytes(g), np.uint8)
        for ident in set(int(v) for v in e[sample].ravel()):
            k = fb.pool_pick(SEED, b, 0, ident, POOL)
            arr[ident * sb:(ident + 1) * sb] = pool[k * sb:(k + 1) * sb]
        layers[b] = arr
    orc = Oracle()
    m = orc.model(HIDDEN, pf_gate_type(fb), fb.MXFP4, layers)
    rc, y_ref, _, _ = orc.prefill_run(m, e[sample], gt[sample], x[sample])
    if rc:
        return {"error": "oracle rc %d" % rc}
    return {"tokens_checked": sample, "blocks": len(blocks), "bitexact": bool(np.array_equal(
        y[sample].view(np.uint32), y_ref.view(np.uint32)))}


def ncu_traffic(name="layer_kernel_decode48_full.md"):
    """DRAM bytes per launch of the dominant kernel from a committed ncu summary, if any."""
    try:
        with open(os.path.join(ROOT, "profiles", name)) as f:
            for line in f:
                if line.startswith("dram_bytes_per_launch:"):
                    return int(line.split(":")[1])
    except (OSError, ValueError):
        pass
    return None


if __name__ == "__main__":
    main()
