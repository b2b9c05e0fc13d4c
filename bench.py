"""Benchmark of the B200 selective-scan hot path.

Default workload: the fused selective scan forward + backward, fp32, with D skip,
SiLU(z) gate and softplus(delta + delta_bias): b=8, L=2048, D=512, N=16 (one block of a
d_model=256, expand=2 Sift model).  One step = one forward (with state checkpoints)
plus one backward over one batch of seeded synthetic inputs.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

With N > 1 (torchrun, one rank per GPU) each rank runs its own batch (weak scaling:
batch rows are independent channels of the scan, no collective on the data path).
The default line also carries, measured at the same N, the other two halves of the
metric: "lm_train" (Sift LM training tokens/s, data parallel with one NCCL all-reduce of
the gradients per step; its all-reduce time alone is reported) and "long_scan" (the
b=4, L=65536, D=2048 bf16 forward, sequence parallel over the ranks: chunk forward,
peer-to-peer boundary exchange, correction; its phase split is reported).
Metric: algorithmic GB/s (each input read once, each output written once; 375.4 MB
per step at b=8) summed over ranks, timed on the device with CUDA events, max over
ranks.  Prints one JSON line on rank 0.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "selective-scan fwd+bwd GB/s & % HBM peak; Sift LM train tokens/s at 1/2/4/8 B200"
CFG = dict(b=8, L=2048, D=512, N=16)
FALLBACK_HBM_GBS = 6650.0


def alg_bytes(b, L, D, N, es=4):
    """Algorithmic bytes of one fwd+bwd: fwd reads u, delta, z, B, C and writes out;
    bwd reads u, delta, z, dout, B, C and writes du, ddelta, dz, dB, dC.
    (Parameters A, D, delta_bias and their grads are O(D*N) and not counted.)"""
    bld, bln = b * L * D * es, b * L * N * es
    fwd = 3 * bld + 2 * bln + bld
    bwd = 4 * bld + 2 * bln + 3 * bld + 2 * bln
    return fwd, bwd


def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


BWD_PROFILE = "scan_bwd_seg_kernel_8x2048x512.md"


def profiled_traffic():
    """dram bytes of one backward call (its summary, main and finalize launches) from the
    committed ncu summary of the current backward kernels (BWD_PROFILE)."""
    p = os.path.join(ROOT, "profiles", BWD_PROFILE)
    try:
        with open(p) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_launch:"):
                    return int(float(line.split(":")[1]))
    except Exception:
        pass
    return None


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for nm, v in zip(names, parts[4:8]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and args.impl == "ours":
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x, world, device):
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ----------------------------------------------------------------- our arm
def run_ours(args, world, rank, local):
    from swiftx_b200 import _lib
    from swiftx_b200.selective_scan import scan_backward, scan_forward
    from swiftx_b200.workloads import config_inputs

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    b, L, D, N = CFG["b"], CFG["L"], CFG["D"], CFG["N"]
    inp = config_inputs(b, L, D, N, seed=rank, device=dev)
    args_f = (inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["D"], inp["z"], inp["delta_bias"], True)

    ev = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731

    pre = torch.empty((b, L, D), device=dev, dtype=torch.float32)

    def step(rec=None):
        # the same calls the autograd Function makes: forward with checkpoints and the saved
        # pre-gate output, then the backward reading them
        if rec is not None:
            rec[0].record()
        _, ck, _ = scan_forward(*args_f, checkpoints=True, pre_out=pre)
        if rec is not None:
            rec[1].record()
        scan_backward(*args_f, None, ck, inp["dout"], y_pre=pre)
        if rec is not None:
            rec[2].record()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    # per-kernel split from eager steps (CUDA events between the two calls)
    recs = [[ev(), ev(), ev()] for _ in range(args.steps)]
    for k in range(args.steps):
        step(recs[k])
    torch.cuda.synchronize()
    fwd_ms = statistics.mean(r[0].elapsed_time(r[1]) for r in recs)
    bwd_ms = statistics.mean(r[1].elapsed_time(r[2]) for r in recs)
    eager_ms = statistics.mean(r[0].elapsed_time(r[2]) for r in recs)

    # the timed steps: the same calls captured once in a CUDA graph (no launch gaps between
    # the forward, backward and finalize kernels), replayed K times
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        step()
    torch.cuda.current_stream(dev).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    sampler = ClockSampler(local) if local == 0 else None
    if sampler:
        sampler.__enter__()
    barrier(world)
    torch.cuda.synchronize()
    t0, t1 = ev(), ev()
    t0.record()
    for k in range(args.steps):
        graph.replay()
    t1.record()
    torch.cuda.synchronize()
    barrier(world)
    if sampler:
        sampler.__exit__()
    ms = t0.elapsed_time(t1) / args.steps
    ms = max_over_ranks(ms, world, dev)
    del graph

    fwd_b, bwd_b = alg_bytes(b, L, D, N)
    step_bytes = fwd_b + bwd_b
    value = step_bytes * world / (ms * 1e-3) / 1e9

    # end to end through the public API with host buffers (pinned), copies inside the region
    e2e = run_e2e(args, inp, dev, world)

    peak, peak_kind = measured_peak()
    # the dominant kernel is the backward's main kernel; it is timed with the two short
    # launches of the same scan_backward call (its segment summaries before it, the dB/dC
    # finalize after it), which the traffic figure also covers
    dom_ms, dom_bytes, dom_name = (bwd_ms, bwd_b, "scan_bwd_seg_kernel (+ scan_bwd_summary_kernel, "
                                   "scan_bwd_seg_finalize_kernel: one scan_backward call)") if bwd_ms >= fwd_ms else \
        (fwd_ms, fwd_b, "scan_fwd_kernel")
    achieved = dom_bytes / (dom_ms * 1e-3) / 1e9
    res = {
        "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded; u, z, dout ~ N(0,1), delta_raw ~ N(0,0.5), inverse-softplus bias of log-uniform dt, A = -(1..N), B, C ~ N(0,1))",
        "config": {"workload": "selective_scan fwd+bwd, fp32, D-skip + SiLU(z) gate + softplus(delta+bias)",
                   "batch": b, "seqlen": L, "d_inner": D, "d_state": N, "per_gpu_batch": b,
                   "parallelism": f"batch-sharded x{world}" if world > 1 else "single GPU",
                   "l2": "inputs larger than L2 (working set ~440 MB/step > 126 MB)",
                   "alg_bytes_per_step": step_bytes,
                   "timing": "the step's scan_forward + scan_backward calls captured in one CUDA graph, "
                             "replayed K times; fwd_ms / bwd_ms / eager_ms_per_step from eager steps"},
        "fwd_ms": round(fwd_ms, 4), "bwd_ms": round(bwd_ms, 4), "eager_ms_per_step": round(eager_ms, 4),
        "frac_of_hbm_step": round(value / world / peak, 4),
        "roofline": {"bound": "hbm", "kernel": dom_name, "achieved": round(achieved, 1), "peak": peak,
                     "peak_kind": peak_kind, "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "traffic": profiled_traffic() if bwd_ms >= fwd_ms else None,
                     "traffic_source": "profiles/" + BWD_PROFILE, "alg_bytes_per_launch": dom_bytes},
        "gpu_launches": 4 * args.steps,
        "e2e": e2e,
    }
    if sampler:
        res["clocks"] = sampler.summary()
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline(args)
    if not args.scan_only:
        # the other two halves of the headline metric, at the same N: Sift LM training
        # (data parallel, gradient all-reduce) and the long-sequence scan (sequence parallel)
        for name, fn in (("lm_train", run_lm_train), ("long_scan", run_long_scan)):
            sub = fn(args, world, rank, local)
            keep = ("value", "unit", "ms_per_step", "scaling", "dtype", "config", "clocks", "e2e", "allreduce_ms",
                    "allreduce_bytes", "phases_ms", "step_latency_ms", "gpu_launches")
            res[name] = {k: sub[k] for k in keep if k in sub}
        res["gpu_launches"] += res["lm_train"]["gpu_launches"] + res["long_scan"]["gpu_launches"]
    return res


def run_e2e(args, inp, dev, world):
    """The scan workload through the host-buffer API: every step copies its inputs from
    pinned host memory, runs forward + backward, and copies every result back
    (HostScanPipeline).  The headline runs consecutive steps chained -- the next step's
    inputs stream in while the previous step's kernels and copies out finish, as a
    loader feeding batch after batch does; every step still moves all of its own bytes
    inside the timed region, and the timed region starts on an idle device and ends
    when the last step's results are on the host.  The unchained figure (each step
    queued behind the current stream, row chunks overlapped within the step) is
    reported beside it."""
    from swiftx_b200.host_pipeline import HostScanPipeline
    b, L, D, N = CFG["b"], CFG["L"], CFG["D"], CFG["N"]
    host = {k: (v.cpu().pin_memory() if v is not None else None) for k, v in inp.items()}
    keys_in = ["u", "delta", "z", "B", "C", "dout", "A", "D", "delta_bias"]
    h2d = sum(host[k].numel() * host[k].element_size() for k in keys_in)

    def measure(pipe):
        res = pipe.allocate_host_outputs()

        def step():
            pipe.forward_backward(host["u"], host["delta"], host["A"], host["B"], host["C"], host["dout"],
                                  D=host["D"], z=host["z"], delta_bias=host["delta_bias"], out=res)

        for _ in range(max(1, args.warmup)):
            step()
        torch.cuda.synchronize()
        barrier(world)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(args.steps):
            step()
        t1.record()
        torch.cuda.synchronize()
        return max_over_ranks(t0.elapsed_time(t1) / args.steps, world, dev), pipe.d2h_bytes(res)

    fwd_b, bwd_b = alg_bytes(b, L, D, N)
    gbs = lambda ms: round((fwd_b + bwd_b) * world / (ms * 1e-3) / 1e9, 2)  # noqa: E731
    chained = HostScanPipeline(b, L, D, N, rows_per_chunk=args.e2e_rows, n_compute=args.e2e_streams,
                               nbuf=args.e2e_bufs, device=dev, chain_calls=True)
    ms, d2h = measure(chained)
    desc = (f"{len(chained.chunks)} row chunk(s) of {chained.rows} rows, {chained.nbuf} device buffer sets")
    del chained
    plain = HostScanPipeline(b, L, D, N, rows_per_chunk=1, n_compute=2, nbuf=3, device=dev)
    ms_plain, _ = measure(plain)
    del plain
    return {"value": gbs(ms), "unit": "GB/s", "ms_per_step": round(ms, 3), "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h,
            "api": "swiftx_b200.host_pipeline.HostScanPipeline.forward_backward (C ABI kernels) on pinned "
                   f"host tensors; {desc}; consecutive steps chained (the next step's inputs stream in under "
                   "the previous step's kernels and copies out)",
            "unchained": {"value": gbs(ms_plain), "ms_per_step": round(ms_plain, 3),
                          "api": "same call, each step queued behind the current stream; 8 one-row chunks "
                                 "whose copies and kernels overlap within the step"}}


# ----------------------------------------------------------------- CPU oracle (reference arm / baseline)
def _oracle_inputs():
    """The default workload's inputs (all 8 rows) as float64 arrays for the oracle."""
    from swiftx_b200.workloads import config_inputs
    inp = config_inputs(CFG["b"], CFG["L"], CFG["D"], CFG["N"], seed=0)
    return {k: (v.double().numpy() if v is not None else None) for k, v in inp.items()}


def _oracle_step(a):
    """One fwd+bwd of the workload through the oracle port of the reference's scan
    (float64 C, OpenMP over all host threads); returns the seconds it took."""
    import oracle
    t = time.perf_counter()
    oracle.scan_fwd(a["u"], a["delta"], a["A"], a["B"], a["C"], D=a["D"], z=a["z"],
                    delta_bias=a["delta_bias"], delta_softplus=True)
    oracle.scan_bwd(a["u"], a["delta"], a["A"], a["B"], a["C"], a["dout"], D=a["D"], z=a["z"],
                    delta_bias=a["delta_bias"], delta_softplus=True)
    return time.perf_counter() - t


def cpu_baseline(args, min_seconds=10.0, max_reps=40):
    """The oracle port timed on the host cores over the whole workload (8 rows), repeated
    until at least min_seconds of CPU work (at most max_reps fwd+bwd passes)."""
    import oracle
    oracle.set_num_threads(os.cpu_count() or 1)
    a = _oracle_inputs()
    _oracle_step(a)                                   # untimed: page in, thread pool up
    times = []
    while sum(times) < min_seconds and len(times) < max_reps:
        times.append(_oracle_step(a))
    fwd_b, bwd_b = alg_bytes(CFG["b"], CFG["L"], CFG["D"], CFG["N"])
    mean = statistics.mean(times)
    return {"value": round((fwd_b + bwd_b) / mean / 1e9, 4), "unit": "GB/s", "cores": oracle.num_threads(),
            "kind": "port", "seconds_per_sample": round(mean, 3),
            "sample": f"the full workload (b={CFG['b']}, L={CFG['L']}, D={CFG['D']}, N={CFG['N']}, fwd+bwd), "
                      f"mean of {len(times)} passes, {sum(times):.1f} s of CPU time"}


def run_reference(args, world, rank):
    """The reference arm: the oracle port of the reference's CPU scan on the host cores,
    one full fwd+bwd of the workload per step (rank 0 only)."""
    if rank != 0:
        return None
    import oracle
    oracle.set_num_threads(os.cpu_count() or 1)
    a = _oracle_inputs()
    for _ in range(args.warmup):
        _oracle_step(a)
    times = [_oracle_step(a) for _ in range(args.steps)]
    fwd_b, bwd_b = alg_bytes(CFG["b"], CFG["L"], CFG["D"], CFG["N"])
    ms = statistics.mean(times) * 1e3
    v = (fwd_b + bwd_b) / (ms * 1e-3) / 1e9
    sample = (f"the full workload per step (b={CFG['b']}, L={CFG['L']}, D={CFG['D']}, N={CFG['N']}, fwd+bwd), "
              f"mean of {len(times)} steps")
    return {"impl": "reference", "metric": METRIC, "value": round(v, 4), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 1), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic (seeded)",
            "config": {"workload": "selective_scan fwd+bwd, D-skip + SiLU(z) gate + softplus(delta+bias)",
                       "batch": CFG["b"], "seqlen": CFG["L"], "d_inner": CFG["D"], "d_state": CFG["N"]},
            "cpu_baseline": {"value": round(v, 4), "unit": "GB/s", "cores": oracle.num_threads(), "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(v, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


# ----------------------------------------------------------------- other workloads
def timed_steps(step, args, world, local, dev):
    """Warm up, then time exactly args.steps calls of step() with CUDA events between a
    barrier + synchronize on both sides; returns (ms per step, max over ranks; clocks)."""
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    sampler = ClockSampler(local) if local == 0 else None
    if sampler:
        sampler.__enter__()
    barrier(world)
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        step()
    t1.record()
    torch.cuda.synchronize()
    barrier(world)
    if sampler:
        sampler.__exit__()
    ms = max_over_ranks(t0.elapsed_time(t1) / args.steps, world, dev)
    return ms, (sampler.summary() if sampler else None)


def base_line(args, world, metric, value, unit, ms, dtype, config, scaling="weak"):
    return {"metric": metric, "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": scaling,
            "vs_baseline": None, "dtype": dtype, "data": "synthetic (seeded)", "config": config}


def run_lm_train(args, world, rank, local):
    """Sift byte-level LM training step: 8 layers, d_model 256, expand 2, d_state 16, d_conv 4,
    vocab 256, tied embedding, batch 16 x 512 i.i.d. random bytes per GPU, AdamW lr 3e-4
    (betas 0.9/0.95, weight decay 0.1 on matrices), grad clip 1.0, bf16 autocast as the
    reference trainer (training/train.py:133-172).  Data parallel: gradients live in one
    flat fp32 buffer that is all-reduced (NCCL, average) once per step.  The forward +
    backward and the clip + AdamW update are each replayed as a CUDA graph (the step is
    otherwise bound by kernel-launch overhead); --no-graph runs them eagerly.  The backward
    assigns each parameter's gradient (FlatGradients(accumulate=False)): no zero fill and
    no per-parameter accumulation add; one multi-tensor copy packs them into the flat
    buffer (the all-reduced one).  The parameters live in two flat buffers (with and
    without weight decay, FlatParameters) laid out like the gradient buffer, so the clip
    is one norm and one scale of the flat gradient and AdamW runs over two tensors."""
    from swiftx_b200.data_parallel import FlatGradients, FlatParameters, broadcast_parameters
    from swiftx_b200.sift import SiftConfig, SiftLM
    dev = torch.device("cuda", local)
    torch.manual_seed(0)
    model = SiftLM(SiftConfig(vocab_size=256, d_model=256, n_layers=8, d_state=16, d_conv=4, expand=2)).to(dev)
    params = list(model.parameters())
    broadcast_parameters(params)                    # identical start on every rank
    decay = [p for p in params if p.dim() >= 2 and not getattr(p, "_no_weight_decay", False)]
    ids = {id(p) for p in decay}
    no_decay = [p for p in params if id(p) not in ids]
    flat_params = FlatParameters([decay, no_decay])
    grads = FlatGradients(decay + no_decay, accumulate=False)     # the backward assigns gradients (no adds)
    flat_params.bind_gradients(grads)
    graphed = not args.no_graph
    opt = torch.optim.AdamW([{"params": [flat_params.flats[0]], "weight_decay": 0.1},
                             {"params": [flat_params.flats[1]], "weight_decay": 0.0}],
                            lr=3e-4, betas=(0.9, 0.95), fused=True, capturable=graphed)
    B, L = 16, 512
    g = torch.Generator().manual_seed(1234 + rank)
    host = torch.randint(0, 256, (B, L + 1), generator=g, dtype=torch.long).pin_memory()
    tok = host.to(dev)

    def fwd_bwd():
        grads.zero_()
        with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
            _, loss = model(tok[:, :-1], tok[:, 1:])
        loss.backward()
        grads.pack_(always=True)                        # into the flat buffer the optimizer reads
        return loss.detach()

    def update():
        # clip_grad_norm_(params, 1.0) over the flat buffer: the global 2-norm, then one scale
        norm = torch.linalg.vector_norm(grads.flat)
        grads.flat.mul_(torch.clamp(1.0 / (norm + 1e-6), max=1.0))
        opt.step()

    def allreduce():
        grads.all_reduce_()

    if graphed:
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(3):
                fwd_bwd()
                allreduce()
                update()
        torch.cuda.current_stream().wait_stream(side)
        g_fb, g_up = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_fb):
            static_loss = fwd_bwd()
        with torch.cuda.graph(g_up):
            update()

        def train_step():
            g_fb.replay()
            allreduce()
            g_up.replay()
            return static_loss
    else:
        def train_step():
            loss = fwd_bwd()
            allreduce()
            update()
            return loss

    ms, clocks = timed_steps(train_step, args, world, local, dev)
    tokens = B * L * world
    # the gradient all-reduce alone (the step's only collective), same buffer, same count
    ms_ar, _ = timed_steps(allreduce, args, world, local, dev) if world > 1 else (0.0, None)

    def e2e_step():
        tok.copy_(host, non_blocking=True)
        return train_step().to("cpu", non_blocking=True)
    ms_e2e, _ = timed_steps(e2e_step, args, world, local, dev)
    res = base_line(args, world, METRIC, round(tokens / (ms * 1e-3), 1), "tokens/s", ms, "bf16",
                    {"workload": "Sift LM train step, 8 layers d_model 256, batch 16 x 512 per GPU", "model": "SiftLM 8L d256 e2 N16 vocab256",
                     "global_batch": B * world, "seq_len": L, "parallelism": f"dp{world}",
                     "cuda_graph": graphed, "l2": "activations and weights per step exceed L2"})
    res["e2e"] = {"value": round(tokens / (ms_e2e * 1e-3), 1), "unit": "tokens/s", "h2d_bytes_per_step":
                  host.numel() * host.element_size(), "d2h_bytes_per_step": 4}
    res["allreduce_ms"] = round(ms_ar, 4)
    res["allreduce_bytes"] = grads.flat.numel() * grads.flat.element_size() if world > 1 else 0
    # per layer: conv fwd, scan fwd, conv bwd x2, scan bwd x2; 9 RMSNorms (8 layers + norm_f):
    # fwd, bwd, weight-gradient sum; token embedding backward: slice partials + slice sum
    res["gpu_launches"] = (6 * 8 + 9 * 3 + 2) * args.steps
    res["clocks"] = clocks
    return res


def run_long_scan(args, world, rank, local):
    """Long-sequence forward scan, bf16 u/delta/B/C/z, fp32 state and output, gated:
    b=4, L=65536, D=2048, N=16, split along the sequence over the ranks (sequence
    parallel: each rank's full forward from a zero state, the boundary values sent peer to
    peer to the later ranks, prefix combine, initial-state correction on ranks > 0).  The
    split is seqpar.chunk_bounds: rank 0, which has no correction to run, takes the
    longer chunk."""
    import math

    from swiftx_b200.selective_scan import scan_correct, scan_forward
    from swiftx_b200.seqpar import chunk_bounds, combine_prefix, exchange_boundaries, sequence_parallel_scan
    dev = torch.device("cuda", local)
    b, L, D, N = 4, 65536, 2048, 16
    bounds = chunk_bounds(L, world)
    Lr = bounds[rank + 1] - bounds[rank]
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    bf = torch.bfloat16
    u = torch.randn(b, Lr, D, generator=g, device=dev).to(bf)
    dr = (torch.randn(b, Lr, D, generator=g, device=dev) * 0.5).to(bf)
    z = torch.randn(b, Lr, D, generator=g, device=dev).to(bf)
    Bm = torch.randn(b, Lr, N, generator=g, device=dev).to(bf)
    Cm = torch.randn(b, Lr, N, generator=g, device=dev).to(bf)
    gc = torch.Generator().manual_seed(0)
    dt = torch.exp(torch.rand(D, generator=gc) * (math.log(0.1) - math.log(1e-3)) + math.log(1e-3))
    bias = (dt + torch.log(-torch.expm1(-dt))).to(dev)
    A = -torch.arange(1, N + 1, dtype=torch.float32).repeat(D, 1).to(dev)
    Dsk = torch.ones(D, device=dev)

    def step():
        if world > 1:
            return sequence_parallel_scan(u, dr, A, Bm, Cm, Dsk, z, bias, True, out_dtype=torch.float32)
        return scan_forward(u, dr, A, Bm, Cm, Dsk, z, bias, True, out_dtype=torch.float32)[0]

    ms, clocks = timed_steps(step, args, world, local, dev)
    alg = (3 * b * L * D * 2 + 2 * b * L * N * 2 + b * L * D * 4)        # whole job
    res = base_line(args, world, METRIC, round(alg / (ms * 1e-3) / 1e9, 1), "GB/s", ms, "bf16-in/f32-state",
                    {"workload": "long-sequence scan fwd, b=4 L=65536 D=2048 N=16, bf16 in / fp32 state", "batch": b, "seqlen": L, "d_inner": D,
                     "d_state": N, "parallelism": f"sequence-parallel x{world}" if world > 1 else "single GPU",
                     "chunk_bounds": bounds, "alg_bytes": alg,
                     "timing": "K independent batches issued back to back (a rank starts the next batch's "
                               "forward while later ranks correct the previous one); step_latency_ms: one "
                               "batch alone"}, scaling="strong")
    res["clocks"] = clocks
    # phase split of one step on this rank (CUDA events; max over ranks): the chunk's
    # forward, the peer-to-peer exchange of boundary values, the combine + correction
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    barrier(world)
    torch.cuda.synchronize()
    ev[0].record()
    out, _, h_end, dsum = scan_forward(u, dr, A, Bm, Cm, Dsk, z, bias, True, out_dtype=torch.float32,
                                       return_last_state=True, return_delta_sum=True)
    ev[1].record()
    if world > 1:
        h_ends, dsums = exchange_boundaries(h_end, dsum)
    ev[2].record()
    if world > 1 and rank > 0:
        scan_correct(out, combine_prefix(h_ends, dsums, A, rank), u, dr, A, Bm, Cm, z=z, delta_bias=bias,
                     delta_softplus=True)
    ev[3].record()
    torch.cuda.synchronize()
    mine = torch.tensor([ev[i].elapsed_time(ev[i + 1]) for i in range(3)], dtype=torch.float64, device=dev)
    if world > 1:
        import torch.distributed as dist
        every = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(every, mine)
    else:
        every = [mine]
    # per rank (rank order): the exchange phase of a later rank includes its wait for the
    # earlier ranks' longer forwards
    res["phases_ms"] = {name: [round(float(t[i]), 4) for t in every]
                        for i, name in enumerate(("chunk_forward", "exchange", "combine_and_correct"))}
    # one step alone (nothing queued behind it; median of 3, max over ranks): a later rank
    # cannot start its correction before every earlier rank's forward is done, so this is
    # longer than ms_per_step, where a rank starts the next batch while later ranks correct
    lat = []
    for _ in range(3):
        barrier(world)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        step()
        e1.record()
        torch.cuda.synchronize()
        lat.append(max_over_ranks(e0.elapsed_time(e1), world, dev))
    res["step_latency_ms"] = round(statistics.median(lat), 4)
    # kernel launches per step on the slowest rank: forward; correction = block sums,
    # their prefix, correct
    res["gpu_launches"] = (1 + (3 if world > 1 else 0)) * args.steps
    return res


def run_small_batch(args, world, rank, local):
    """Long rows at a small batch, fwd + bwd through the public calls: b=1, L=65536, D=2048,
    N=16, bf16 inputs, fp32 state, gated, softplus (a long-context training step of one
    block at batch 1).  Whole-row kernels would leave most SMs idle: the forward cuts
    each row into segments (SWX_SCAN_SPLIT_FWD; --no-split turns it off) and the
    backward's segment plan counts the single row.  One row per rank (weak scaling)."""
    from swiftx_b200.selective_scan import scan_backward, scan_forward
    from swiftx_b200.workloads import config_inputs
    dev = torch.device("cuda", local)
    b, L, D, N = 1, 65536, 2048, 16
    inp = config_inputs(b, L, D, N, seed=rank, device=dev, dtype=torch.bfloat16)
    fargs = (inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["D"], inp["z"], inp["delta_bias"], True)
    pre = torch.empty((b, L, D), device=dev, dtype=torch.float32)

    def step():
        _, ck, _ = scan_forward(*fargs, checkpoints=True, pre_out=pre, split=not args.no_split)
        scan_backward(*fargs, None, ck, inp["dout"], y_pre=pre)

    ms, clocks = timed_steps(step, args, world, local, dev)
    fwd_b, bwd_b = alg_bytes(b, L, D, N, es=2)
    alg = fwd_b + bwd_b
    res = base_line(args, world, METRIC, round(alg * world / (ms * 1e-3) / 1e9, 1), "GB/s", ms, "bf16-in/f32-state",
                    {"workload": f"selective_scan fwd+bwd at batch 1, L={L} D={D} N={N}, bf16 in",
                     "batch": b, "seqlen": L, "d_inner": D, "d_state": N, "split_forward": not args.no_split,
                     "parallelism": f"one row per rank x{world}" if world > 1 else "single GPU",
                     "alg_bytes_per_step": alg, "l2": "inputs larger than L2"})
    res["clocks"] = clocks
    return res


def run_correct(args, world, rank, local):
    """The sequence-parallel initial-state correction alone, on one rank's chunk of the
    long-sequence workload: b=4, L=32768 (half of 65536), D=2048, N=16, bf16 u/delta/C/z,
    fp32 output read and written in place, gated, softplus.  Reads delta, z (bf16), C and
    the output; writes the output.  One chunk per rank (weak scaling)."""
    import math

    from swiftx_b200.selective_scan import scan_correct
    dev = torch.device("cuda", local)
    b, L, D, N = 4, args.corr_len, 2048, 16
    g = torch.Generator(device=dev).manual_seed(2000 + rank)
    bf = torch.bfloat16
    u = torch.randn(b, L, D, generator=g, device=dev).to(bf)
    dr = (torch.randn(b, L, D, generator=g, device=dev) * 0.5).to(bf)
    z = torch.randn(b, L, D, generator=g, device=dev).to(bf)
    Bm = torch.randn(b, L, N, generator=g, device=dev).to(bf)
    Cm = torch.randn(b, L, N, generator=g, device=dev).to(bf)
    gc = torch.Generator().manual_seed(0)
    dt = torch.exp(torch.rand(D, generator=gc) * (math.log(0.1) - math.log(1e-3)) + math.log(1e-3))
    bias = (dt + torch.log(-torch.expm1(-dt))).to(dev)
    A = -torch.arange(1, N + 1, dtype=torch.float32).repeat(D, 1).to(dev)
    out = torch.randn(b, L, D, generator=g, device=dev)
    h_in = torch.randn(b, D, N, generator=g, device=dev) * 0.1

    def step():
        scan_correct(out, h_in, u, dr, A, Bm, Cm, z=z, delta_bias=bias, delta_softplus=True)

    ms, clocks = timed_steps(step, args, world, local, dev)
    alg = b * L * D * (2 + 2 + 4 + 4) + b * L * N * 2
    peak, kind = measured_peak()
    achieved = alg / (ms * 1e-3) / 1e9
    res = base_line(args, world, METRIC, round(alg * world / (ms * 1e-3) / 1e9, 1), "GB/s", ms, "bf16-in/f32-out",
                    {"workload": f"sequence-parallel initial-state correction, b=4 L={L} D=2048 N=16",
                     "batch": b, "seqlen": L, "d_inner": D, "d_state": N,
                     "parallelism": f"one chunk per rank x{world}" if world > 1 else "single GPU",
                     "l2": "inputs larger than L2", "alg_bytes_per_step": alg})
    res["roofline"] = {"bound": "mufu (16 decays + softplus + silu per channel-step); hbm fraction shown",
                       "kernel": "scan_correct_kernel (+ scan_correct_sums_kernel, scan_correct_prefix_kernel)",
                       "achieved": round(achieved, 1), "peak": peak, "peak_kind": kind, "unit": "GB/s",
                       "frac": round(achieved / peak, 4), "traffic": None, "alg_bytes_per_launch": alg}
    res["clocks"] = clocks
    res["gpu_launches"] = 3 * args.steps
    return res


def run_linear_scan(args, world, rank, local):
    """parallel_scan forward + backward (h_t = a_t h_{t-1} + x_t and its adjoint) on the
    (b, L, D, N) = (8, 2048, 512, 16) fp32 tensors the reference's _SelectiveScanFn feeds
    its _scan: forward reads a, x and writes h; backward reads a, h, dh and writes da, dx
    (8 x 537 MB per step).  One batch per rank (weak scaling)."""
    from swiftx_b200 import parallel_scan
    dev = torch.device("cuda", local)
    b, L, D, N = args.ls_batch, 2048, 512, 16
    g = torch.Generator(device=dev).manual_seed(3000 + rank)
    a = (torch.rand(b, L, D, N, device=dev, generator=g) * 0.2 + 0.8).requires_grad_()
    x = torch.randn(b, L, D, N, device=dev, generator=g).requires_grad_()
    dh = torch.randn(b, L, D, N, device=dev, generator=g)

    def step():
        a.grad = x.grad = None
        parallel_scan(a, x).backward(dh)

    ms, clocks = timed_steps(step, args, world, local, dev)
    elems = b * L * D * N
    alg = 8 * elems * 4
    peak, kind = measured_peak()
    achieved = alg / (ms * 1e-3) / 1e9
    res = base_line(args, world, METRIC, round(alg * world / (ms * 1e-3) / 1e9, 1), "GB/s", ms, "f32",
                    {"workload": "linear recurrence parallel_scan fwd+bwd", "batch": b, "seqlen": L,
                     "width": D * N, "parallelism": f"batch-sharded x{world}" if world > 1 else "single GPU",
                     "l2": "inputs larger than L2", "alg_bytes_per_step": alg})
    res["roofline"] = {"bound": "hbm", "kernel": "linear_scan_fwd_kernel + linear_scan_bwd_kernel",
                       "achieved": round(achieved, 1), "peak": peak, "peak_kind": kind, "unit": "GB/s",
                       "frac": round(achieved / peak, 4), "traffic": None, "alg_bytes_per_launch": alg // 2}
    res["clocks"] = clocks
    res["gpu_launches"] = 2 * args.steps
    return res


def run_decode(args, world, rank, local):
    """Recurrent decode: batch 256 (sharded over the ranks), 24 layers, D=2048, N=16,
    d_conv=4, fp32 state ~ N(0, 0.1); per layer one fused conv-window shift + state update
    + C readout + gate launch (the persistent streaming kernel at this shape); the 24-layer
    step is replayed as one CUDA graph."""
    import math

    from swiftx_b200.decode import decode_step
    dev = torch.device("cuda", local)
    btot, layers, D, N, K = 256, 24, 2048, 16, 4
    b = btot // world
    g = torch.Generator(device=dev).manual_seed(2000 + rank)
    gc = torch.Generator().manual_seed(0)
    lay = []
    for _ in range(layers):
        dt = torch.exp(torch.rand(D, generator=gc) * (math.log(0.1) - math.log(1e-3)) + math.log(1e-3))
        lay.append({
            "cw": (torch.randn(D, K, generator=gc) * 0.5).to(dev), "cb": torch.randn(D, generator=gc).to(dev),
            "A": -torch.arange(1, N + 1, dtype=torch.float32).repeat(D, 1).to(dev), "Dsk": torch.ones(D, device=dev),
            "bias": (dt + torch.log(-torch.expm1(-dt))).to(dev),
            "cs": torch.randn(b, D, K, generator=g, device=dev), "ss": torch.randn(b, D, N, generator=g, device=dev) * 0.1,
            "x": torch.randn(b, D, generator=g, device=dev), "z": torch.randn(b, D, generator=g, device=dev),
            "dr": torch.randn(b, D, generator=g, device=dev) * 0.5,
            "B": torch.randn(b, N, generator=g, device=dev), "C": torch.randn(b, N, generator=g, device=dev)})

    def token_step():
        for p in lay:
            p["y"] = decode_step(p["x"], p["cs"], p["cw"], p["cb"], p["dr"], p["B"], p["C"], p["A"], p["ss"],
                                 Dskip=p["Dsk"], z=p["z"], delta_bias=p["bias"])

    for _ in range(3):
        token_step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        token_step()
    ms, clocks = timed_steps(graph.replay, args, world, local, dev)
    per_layer = b * D * (2 * N * 4 + 2 * K * 4 + 4 * 4) + b * 2 * N * 4
    res = base_line(args, world, METRIC, round(btot / (ms * 1e-3), 1), "tokens/s", ms, "f32",
                    {"workload": "recurrent decode step, batch 256, 24 layers, D=2048 N=16 K=4", "batch": btot, "layers": layers, "d_inner": D,
                     "d_state": N, "d_conv": K, "parallelism": f"batch-sharded x{world}" if world > 1 else "single GPU",
                     "cuda_graph": True}, scaling="strong")
    res["latency_ms_per_token"] = round(ms, 4)
    del graph
    torch.cuda.synchronize()
    # the whole model's recurrent step (embedding, 24 x [in_proj, conv-window kernel,
    # x_proj, dt_proj, state-update kernel, out_proj], norms, head) replayed from one graph
    from swiftx_b200.sift import GraphedStep, SiftConfig, SiftLM
    lay.clear()
    torch.manual_seed(0)
    model = SiftLM(SiftConfig(vocab_size=256, d_model=1024, n_layers=layers, d_state=N, d_conv=K,
                              expand=2)).to(dev).eval()
    tok = torch.randint(0, 256, (b,), device=dev, generator=g)
    res["model_step"] = {"model": f"SiftLM d_model 1024 (D={D}), {layers} layers, N={N}, vocab 256; fp32 state",
                         "batch": btot, "cuda_graph": "whole step (GraphedStep)"}
    for name, amp in (("fp32", None), ("bf16_projections", torch.bfloat16)):
        stepper = GraphedStep(model, b, dev, autocast_dtype=amp)
        ms_m, _ = timed_steps(lambda: stepper(tok), args, world, local, dev)
        res["model_step"][name] = {"tokens_per_s": round(btot / (ms_m * 1e-3), 1), "ms_per_token": round(ms_m, 4)}
        del stepper
    achieved = per_layer * layers / (ms * 1e-3) / 1e9
    peak, kind = measured_peak()
    res["roofline"] = {"bound": "hbm", "kernel": "decode_stream_kernel", "achieved": round(achieved, 1), "peak": peak,
                       "peak_kind": kind, "unit": "GB/s", "frac": round(achieved / peak, 4), "traffic": None,
                       "alg_bytes_per_launch": per_layer}
    res["clocks"] = clocks
    res["gpu_launches"] = layers * args.steps
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--scan-only", action="store_true",
                    help="default workload: skip the lm_train and long_scan sub-objects")
    ap.add_argument("--no-graph", action="store_true", help="lm_train: run the step eagerly, no CUDA graphs")
    ap.add_argument("--e2e-rows", type=int, default=8, help="scan e2e: batch rows per pipelined chunk")
    ap.add_argument("--ls-batch", type=int, default=8, help="linear_scan: batch rows (8 = the measured size)")
    ap.add_argument("--e2e-streams", type=int, default=1, help="scan e2e: compute streams of the pipeline")
    ap.add_argument("--e2e-bufs", type=int, default=2, help="scan e2e: device buffer sets of the pipeline")
    ap.add_argument("--corr-len", type=int, default=32768, help="correct: chunk length")
    ap.add_argument("--no-split", action="store_true", help="small_batch: whole-row forward")
    ap.add_argument("--workload", choices=["scan", "lm_train", "long_scan", "decode", "linear_scan", "correct",
                                           "small_batch"],
                    default="scan",
                    help="scan: fused scan fwd+bwd at b=8 L=2048 D=512 N=16 (default); lm_train: Sift LM training step; "
                         "long_scan: b=4 L=65536 D=2048 forward; decode: batch-256 24-layer recurrent step; "
                         "linear_scan: parallel_scan fwd+bwd at (8, 2048, 512, 16); "
                         "correct: the sequence-parallel correction kernel on a b=4 L=32768 D=2048 chunk; "
                         "small_batch: fwd+bwd at b=1 L=65536 D=2048 bf16")
    args = ap.parse_args()
    world, rank, local = dist_setup(args)
    if args.impl == "reference":
        if args.workload != "scan":
            res = {"impl": "reference", "unavailable": "the reference arm is the CPU oracle port of the scan "
                   "(default workload); the other workloads have no CPU reference run"} if rank == 0 else None
        else:
            res = run_reference(args, world, rank)
    elif args.workload == "lm_train":
        res = run_lm_train(args, world, rank, local)
    elif args.workload == "long_scan":
        res = run_long_scan(args, world, rank, local)
    elif args.workload == "decode":
        res = run_decode(args, world, rank, local)
    elif args.workload == "linear_scan":
        res = run_linear_scan(args, world, rank, local)
    elif args.workload == "correct":
        res = run_correct(args, world, rank, local)
    elif args.workload == "small_batch":
        res = run_small_batch(args, world, rank, local)
    else:
        res = run_ours(args, world, rank, local)
    if rank == 0 and res is not None:
        print(json.dumps(res), flush=True)
    if world > 1 and args.impl == "ours":
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
