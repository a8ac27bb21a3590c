#!/usr/bin/env python
"""Benchmark of the MoE FFN hot path on B200.

Metric: MoE-layer tokens/s (one step = one forward of one MoE layer over T
tokens), with the roofline fraction of the dominant kernel. Default
workload: config 2 of the benchmark set (Qwen3-MoE layer, hidden 2048, 128
experts, top-8, intermediate 768, Q4_K weights), decode batch T=64, seeded
synthetic inputs; the T=1..32 sweep and one entry per other configuration
(config 1 T=32, config 3 T=2048, config 4 T=512 and 4096, config 5 T=8192)
are reported beside it.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

--impl reference times the CPU restatement of the reference MoE path (the
reference is Rust and cannot be built here) on this host's cores, on the same
workload, with layers built by the restatement's own generator and quantiser
(the product library is not loaded). Under torchrun with N>1 the layer runs
expert-parallel: rank g holds experts [g*E/N, (g+1)*E/N), routes its own T
tokens and exchanges the routed rows with the owning ranks
(moe_forward_ep); value = N*T tokens per step over the slowest rank's time
(weak scaling). --strong splits T over the ranks instead.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "jero-engine_b200"))

FLUSH_BYTES = 256 << 20   # > 126 MB L2
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
METRIC, UNIT = "MoE-layer tokens/s", "tokens/s"
# the other configurations, one timed entry each (N = 1 only)
EXTRA_CONFIGS = ((1, 32), (3, 2048), (4, 512), (4, 4096), (5, 8192))
PARITY_ROWS = 16


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", type=int, default=2)
    ap.add_argument("--tokens", type=int, default=0, help="T of the headline workload (default: largest of the config)")
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-configs", action="store_true", help="skip the entries of the other configurations")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--strong", action="store_true", help="with N>1: T is the global batch, split over the ranks")
    ap.add_argument("--flags", type=int, default=0, help="MOE_FLAG_* bits of the context (e.g. 1: tensor cores always)")
    return ap.parse_args()


def rank_info():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))


def measured_traffic(workload, kernel):
    """DRAM bytes per launch of `kernel` from the committed ncu summary, or None."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            return json.load(f).get(workload, {}).get(kernel)
    except Exception:
        return None


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def tensor_peak():
    """Dense f16/bf16 tensor throughput (TFLOP/s): the sustained measurement,
    since the expert GEMMs run inside a long step."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured (sustained)"
    except Exception:
        return FALLBACK_BF16_TFLOPS, "fallback"


def workload_config(cfg, T, world, strong, U):
    """The workload both arms report (no timing method, no model keys)."""
    return {"workload": f"{cfg.name} T={T}", "T": T, "H": cfg.H, "E": cfg.E, "k": cfg.k, "I": cfg.I, "S": cfg.S,
            "quant": "Q4_K" if cfg.quant == 12 else "Q8_0", "experts_routed": int(U),
            "global_batch": int(world * T),
            "parallelism": f"ep{world}" if world > 1 else "single"}


def kernel_flops(cfg, T, routed_rows=None):
    """Algorithmic FLOPs of the tensor-core expert GEMMs (no padding counted).
    Expert parallel (routed_rows = rows this rank's experts received): the
    launches time the routed experts only; the shared expert is its own pass."""
    routed = 2 * (T * cfg.k if routed_rows is None else routed_rows) * cfg.H * cfg.I
    shared = 2 * T * cfg.H * cfg.S if routed_rows is None else 0
    return {"gate_up_tc": 2 * routed + 2 * shared, "down_tc": routed + shared}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 100 ms."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu):
        self.gpu = gpu
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def wait_first(self, timeout=5.0):
        """Blocks until nvidia-smi has written its first sample (it needs a few
        hundred ms to start), so the samples cover the timed region."""
        t0 = time.time()
        while self.proc and time.time() - t0 < timeout:
            self.f.flush()
            if os.path.getsize(self.path) > 0:
                return
            time.sleep(0.05)

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                c = [x.strip() for x in line.split(",")]
                if len(c) < 9:
                    continue
                try:
                    sm.append(float(c[1]))
                    smax.append(float(c[2]))
                except ValueError:
                    continue
                for n, v in zip(names, c[5:9]):
                    if v.lower().startswith("active"):
                        reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def kernel_bytes(cfg, weights, sel_idx, T, expert_range=None, routed_rows=None):
    """Algorithmic bytes per launch of the expert kernels and of the whole layer.
    Weights of each routed expert are read once; activations travel as int8
    blocks (1 byte + 8 bytes of scales per 32 values = 1.25 B/value). With
    expert parallelism, sel_idx holds every rank's choices, expert_range the
    rank's experts and routed_rows the rows it received; T its own tokens."""
    import numpy as np
    chosen = np.unique(sel_idx[sel_idx >= 0])
    if expert_range is not None:
        chosen = chosen[(chosen >= expert_range[0]) & (chosen < expert_range[1])]
    U = len(chosen)
    routed = T * cfg.k if routed_rows is None else routed_rows
    slots = routed + (T if cfg.S else 0)
    per = {m: weights.tensor(f"blk.0.ffn_{m}_exps.weight").data.nbytes // cfg.E for m in ("gate", "up", "down")}
    sh = {m: (weights.tensor(f"blk.0.ffn_{m}_shexp.weight").data.nbytes if cfg.S else 0)
          for m in ("gate", "up", "down")}
    W = max(cfg.I, cfg.S)
    if expert_range is None:
        gate_up = U * (per["gate"] + per["up"]) + sh["gate"] + sh["up"] + T * cfg.H * 1.25 + slots * W * 1.25
        down = U * per["down"] + sh["down"] + slots * W * 1.25 + slots * cfg.H * 4
    else:   # the routed expert stage over the received rows (the shared expert is its own pass)
        gate_up = U * (per["gate"] + per["up"]) + routed * cfg.H * 1.25 + routed * cfg.I * 1.25
        down = U * per["down"] + routed * cfg.I * 1.25 + routed * cfg.H * 4
    layer = (U * sum(per.values()) + sum(sh.values()) + cfg.E * cfg.H * 4 + 2 * T * cfg.H * 4 + T * cfg.k * 8)
    if expert_range is not None:   # activation rows out and expert outputs back through the exchange
        layer += routed * cfg.H * 1.25 + routed * cfg.H * 4
    # the fused small-batch launch streams both projections
    return {"gate_up": gate_up, "down": down, "experts_tc": gate_up + down, "experts_i8": gate_up + down,
            "layer": layer, "U": U,
            "routed_rows": routed}


def roofline_of(cfg, T, prof, kb, workload, rows_here=None, ep=False, tensor_peaks=None):
    """Roofline of the dominant expert kernel of one forward from the per-stage
    profile: HBM-bound paths by algorithmic bytes, the prefill tensor-core path
    by algorithmic FLOPs (against the sustained bf16 peak, with the fraction of
    this run's own f16 and int8 probe peaks beside it)."""
    tc = "gate_up_tc" in prof
    i8 = "gate_up_i8" in prof
    fused = [k for k in ("experts_i8", "experts_tc") if k in prof]
    cands = ("gate_up_tc", "down_tc") if tc else (("gate_up_i8", "down_i8") if i8 else
                                                  (tuple(fused) if fused else ("gate_up", "down")))
    dom = max(cands, key=lambda k: prof.get(k, (0, 1))[0])
    dom_ms = prof[dom][0] / prof[dom][1]
    traffic = None if ep else measured_traffic(workload, dom)   # captures are single-GPU workloads
    if tc:
        fl = kernel_flops(cfg, T, rows_here)[dom]
        tpk, tpk_kind = tensor_peak()
        ach = fl / (dom_ms / 1e3) / 1e12
        r = {"bound": "tensor", "kernel": dom, "achieved": round(ach, 1), "peak": tpk, "unit": "TFLOP/s",
             "frac": round(ach / tpk, 4), "traffic": traffic, "peak_source": tpk_kind,
             "algorithmic_flops_per_launch": int(fl),
             "operands": "f16 (weights dequantised from GGUF blocks in shared memory), f32 accumulate"}
        if tensor_peaks:
            r["frac_of_probe_f16"] = round(ach / tensor_peaks["f16_tflops"], 4)
            r["frac_of_probe_int8"] = round(ach / tensor_peaks["int8_tops"], 4)
        return r
    hbm, peak_kind = peaks()
    b = kb[dom if dom.startswith("experts") else dom.replace("_i8", "")]
    ach = b / (dom_ms / 1e3) / 1e9
    return {"bound": "hbm", "kernel": dom, "achieved": round(ach, 1), "peak": hbm, "unit": "GB/s",
            "frac": round(ach / hbm, 4), "traffic": traffic, "peak_source": peak_kind,
            "algorithmic_bytes_per_launch": int(b)}


def row_rel_err(out, ref):
    import numpy as np
    return np.abs(out - ref).max(axis=1) / np.maximum(np.abs(ref).max(axis=1), 1e-30)


def oracle_parity(cfg, weights, x_rows, out_rows, si_rows, threads):
    """Rows of this run's output against the CPU oracle: routing bit-exact and
    the max per-row relative error (the contract is 1e-2)."""
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as orc
    L = orc.Layer(weights, 0, cfg.E, cfg.k, cfg.S > 0, cfg.route, hidden=cfg.H)
    ro, rsi, _ = L.forward(x_rows, threads)
    return {"rows_checked": int(len(x_rows)), "routing_exact": bool(np.array_equal(si_rows, rsi)),
            "max_row_rel_err": float(row_rel_err(out_rows, ro).max())}


def cpu_baseline(cfg, weights, x, seconds, threads):
    """The CPU oracle (restatement of the reference path, one token at a time,
    matvec rows split over a persistent pool) on rows of the same workload."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as orc
    L = orc.Layer(weights, 0, cfg.E, cfg.k, cfg.S > 0, cfg.route, hidden=cfg.H)
    L.forward(x[:1], threads)
    done, t0 = 0, time.perf_counter()
    while True:
        L.forward(x, threads)
        done += x.shape[0]
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return done / el, done, el


def run_reference(args):
    """The reference arm: the CPU restatement timed on this host's cores over
    the same workload and configuration as our arm (the global batch at N>1),
    each step a bounded sample of it. Rank 0 alone runs; the layer is built by
    the restatement's own generator and quantiser (same bytes as the library's),
    so the product library is never loaded."""
    rank, _, world = rank_info()
    if rank != 0:
        return
    import numpy as np
    import synth
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as orc
    synth.use_backend(orc)
    cfg = synth.CONFIGS[args.config]
    T_arg = args.tokens or max(cfg.tokens)
    ep = world > 1
    T = T_arg // world if (ep and args.strong) else T_arg
    glob = T * world
    threads = os.cpu_count() or 1
    weights = synth.build_weights(cfg)
    x = synth.gen_x(cfg, glob)
    L = orc.Layer(weights, 0, cfg.E, cfg.k, cfg.S > 0, cfg.route, hidden=cfg.H)
    sample = min(glob, 256)   # tokens per timed step
    for _ in range(args.warmup):
        L.forward(x[:1], threads)
    times, sel = [], []
    for i in range(args.steps):
        lo = (i * sample) % glob
        rows = x[lo:lo + sample] if lo + sample <= glob else np.concatenate([x[lo:], x[:lo + sample - glob]])
        t0 = time.perf_counter()
        _, si, _ = L.forward(rows, threads)
        times.append(time.perf_counter() - t0)
        sel.append(si)
    total = sum(times)
    value = sample * args.steps / total
    # experts routed by the whole global batch (the oracle's routing is the product's, bit for bit)
    router = weights.tensor("blk.0.ffn_gate_inp.weight").data.reshape(cfg.E, cfg.H)
    chosen = set()
    for t in range(glob):
        idx, _ = L.select(orc.router_logits(router, x[t]))
        chosen.update(int(e) for e in idx)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * total / args.steps, 3), "higher_is_better": True,
        "scaling": "strong" if (ep and args.strong) else "weak",
        "vs_baseline": None, "dtype": "int8", "data": "synthetic (seeded N(0,1) activations, N(0,0.02) weights "
                                                     "quantised to GGUF blocks)",
        "config": workload_config(cfg, T, world, args.strong, len(chosen)),
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{sample} of the {glob} tokens of the workload per step, {args.steps} steps, "
                                   f"one token at a time (CPU restatement of the reference MoE path, "
                                   f"oracle/moe_oracle.c)"},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


class Timer:
    """Forwards of one context timed with CUDA events on its stream, the L2
    flushed (256 MiB write) before every step."""

    def __init__(self, torch, ctx, stream, flush, step, barrier, world):
        self.torch, self.ctx, self.stream, self.flush = torch, ctx, stream, flush
        self.step, self.barrier, self.world = step, barrier, world

    def run(self, t, steps, profile):
        torch = self.torch
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        self.barrier()
        torch.cuda.synchronize()
        if profile:
            self.ctx.set_profiling(True)
        for i in range(steps):
            self.flush.fill_(i & 0xFF)
            evs[i][0].record(self.stream)
            self.step(t)
            evs[i][1].record(self.stream)
        torch.cuda.synchronize()
        self.barrier()
        prof = None
        if profile:
            prof = self.ctx.profile_read()
            self.ctx.set_profiling(False)
        return [a.elapsed_time(b) for a, b in evs], prof

    def stages(self, t, n):
        """Per-stage times from n profiled forwards, one at a time: for each
        stage the median over the forwards of its time per forward, so a single
        slow forward (a clock dip, a first launch) does not move the figure.
        Returns ({stage: (ms per forward, launches per forward)}, n)."""
        import statistics
        per = {}
        for _ in range(n):
            _, (prof, _) = self.run(t, 1, True)
            for k, (ms, launches) in prof.items():
                a = per.setdefault(k, ([], []))
                a[0].append(ms)
                a[1].append(launches)
        return {k: (statistics.median(v[0]), max(1, int(statistics.median(v[1])))) for k, v in per.items()}, n


def probe_peaks(jm):
    """This GPU's dense tensor peaks from the library's probe (one issuing warp
    per SM, M = 128, N = 256, A in TMEM): f16 and int8."""
    try:
        f16, _ = jm.probe_tensor(0, 0, 128, 256, True, 1, 1, 8192)
        i8, _ = jm.probe_tensor(0, 1, 128, 256, True, 1, 1, 8192)
        return {"f16_tflops": round(f16, 1), "int8_tops": round(i8, 1),
                "how": "moe_probe_tensor: 8192 back-to-back tcgen05.mma M128 N256 (A in TMEM) per SM, CUDA events"}
    except Exception as e:   # the headline does not depend on it
        return {"error": str(e)[:200]}


def extra_config(torch, jm, synth, cid, T, stream, flush, tensor_peaks, steps=10):
    """One timed entry of another configuration at N = 1: tokens/s, the
    dominant kernel's roofline and a parity sample against the oracle."""
    import numpy as np
    cfg = synth.CONFIGS[cid]
    weights = synth.build_weights(cfg)
    x = synth.gen_x(cfg, T)
    ctx = jm.Context(0, T, 1)
    try:
        ctx.set_stream(stream.cuda_stream)
        d, keep = synth.desc_for(cfg, weights)
        ctx.upload(0, d)
        x_dev = torch.from_numpy(x).cuda()
        out_dev = torch.empty_like(x_dev)
        si_dev = torch.empty((T, cfg.k), dtype=torch.int32, device="cuda")
        sw_dev = torch.empty((T, cfg.k), dtype=torch.float32, device="cuda")

        def step(t):
            ctx.forward_ptrs(0, t, x_dev.data_ptr(), out_dev.data_ptr(), si_dev.data_ptr(), sw_dev.data_ptr())

        tm = Timer(torch, ctx, stream, flush, step, lambda: None, 1)
        tm.run(T, 3, False)
        ms, _ = tm.run(T, steps, False)
        prof, _ = tm.stages(T, max(5, steps // 2))
        sel = si_dev.cpu().numpy()
        kb = kernel_bytes(cfg, weights, sel, T)
        wl = f"{cfg.name} T={T}"
        m = statistics.median(ms)
        rows = np.sort(np.random.default_rng(cid).choice(T, min(8, T), replace=False))
        par = oracle_parity(cfg, weights, x[rows], out_dev.cpu().numpy()[rows], sel[rows], os.cpu_count() or 1)
        return {"workload": wl, "T": T, "tokens_per_s": round(T / (m / 1e3), 1), "ms_per_step": round(m, 4),
                "experts_routed": kb["U"], "steps": steps,
                "roofline": roofline_of(cfg, T, prof, kb, wl, tensor_peaks=tensor_peaks),
                "layer_hbm_frac": round(kb["layer"] / (m / 1e3) / 1e9 / peaks()[0], 4),
                "kernels": {k: round(1e3 * v[0] / v[1], 2) for k, v in prof.items()}, "parity": par}
    finally:
        ctx.close()


def run_ours(args):
    import numpy as np
    import torch
    import torch.distributed as dist
    import jeromoe as jm
    import synth

    rank, local_rank, world = rank_info()
    torch.cuda.set_device(local_rank)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=torch.device("cuda", local_rank))
    cfg = synth.CONFIGS[args.config]
    T_arg = args.tokens or max(cfg.tokens)
    ep = world > 1
    # tokens of this rank: T (weak scaling) or T / world of a global batch of T (--strong)
    T = T_arg // world if (ep and args.strong) else T_arg
    if T < 1:
        raise SystemExit(f"--strong needs at least {world} tokens")
    sweep_T = [] if (args.no_sweep or ep) else [t for t in cfg.tokens if t != T]
    tensor_peaks = probe_peaks(jm) if (world == 1 and not args.no_configs) else None
    weights = synth.build_weights(cfg)
    Tmax = max([T] + sweep_T)
    x_all = synth.gen_x(cfg, Tmax * world)
    x_host = x_all[rank * Tmax:(rank + 1) * Tmax].copy()
    ctx = jm.Context(local_rank, Tmax, 1, flags=args.flags)
    if ep:
        ids = [jm.ep_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(ids, src=0)
        ctx.ep_init(rank, world, ids[0])
    d, keep = synth.desc_for(cfg, weights)
    ctx.upload(0, d)
    # one dedicated stream for the library, the flush and the timing events
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    ctx.set_stream(stream.cuda_stream)
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    x_dev = torch.from_numpy(x_host).cuda()
    out_dev = torch.empty_like(x_dev)
    si_dev = torch.empty((x_dev.shape[0], cfg.k), dtype=torch.int32, device="cuda")
    sw_dev = torch.empty((x_dev.shape[0], cfg.k), dtype=torch.float32, device="cuda")

    def step(t):
        if ep:
            ctx.forward_ep_ptrs(0, t, x_dev.data_ptr(), out_dev.data_ptr())
        else:
            ctx.forward_ptrs(0, t, x_dev.data_ptr(), out_dev.data_ptr(), si_dev.data_ptr(), sw_dev.data_ptr())

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    tm = Timer(torch, ctx, stream, flush, step, barrier, world)
    sampler = ClockSampler(local_rank)
    sampler.start()
    for i in range(args.warmup):
        flush.fill_(i & 0xFF)
        step(T)
    torch.cuda.synchronize()
    if ep:
        # every rank's choices (one extra forward with selection output), for the rank's byte count
        _, sel_local, _ = ctx.forward_ep(0, x_host[:T])
        gathered = [torch.empty((T, cfg.k), dtype=torch.int32, device="cuda") for _ in range(world)]
        dist.all_gather(gathered, torch.from_numpy(sel_local).cuda())
        sel = torch.cat(gathered).cpu().numpy()
        El = cfg.E // world
        mine = (sel >= rank * El) & (sel < (rank + 1) * El)
        kb = kernel_bytes(cfg, weights, sel, T, (rank * El, (rank + 1) * El), int(mine.sum()))
        U_global = len(np.unique(sel))
    else:
        sel = si_dev[:T].cpu().numpy()
        kb = kernel_bytes(cfg, weights, sel, T)
        U_global = kb["U"]
    sampler.wait_first()
    # keep the GPU busy until the timed region starts so the samples see it under load
    for i in range(max(args.warmup, 20)):
        flush.fill_(i & 0xFF)
        step(T)
    step_ms, _ = tm.run(T, args.steps, False)
    clocks = sampler.stop()
    # per-stage breakdown from a second pass with an event at every stage
    # boundary (the events serialise the stages, so it is not the timed pass)
    prof, n_fwd = tm.stages(T, args.steps)
    total_ms = sum(step_ms)
    if world > 1:
        tt = torch.tensor([total_ms], device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        total_ms = float(tt.item())
    value = world * T * args.steps / (total_ms / 1e3)
    wl = f"{cfg.name} T={T}"
    roofline = roofline_of(cfg, T, prof, kb, wl, kb["routed_rows"] if ep else None, ep=ep, tensor_peaks=tensor_peaks)
    layer_ms = total_ms / args.steps
    # per launch (median forward), and the launches of the timed pass
    kernels = {k: {"avg_us": round(1e3 * v[0] / v[1], 2), "launches": v[1] * args.steps} for k, v in prof.items()}
    launches = sum(v[1] for v in prof.values()) * args.steps

    # parity of the timed run's output, outside the timed region: sampled rows
    # against the CPU oracle; with expert parallelism also every row against a
    # single-GPU context holding all experts, on the same GPU and tokens
    out_np = out_dev[:T].cpu().numpy()
    rows = np.sort(np.random.default_rng(rank).choice(T, min(PARITY_ROWS, T), replace=False))
    sel_rows = None
    if ep:
        _, si_ep, _ = ctx.forward_ep(0, x_host[:T])   # collective: every rank takes part
        sel_rows = si_ep[rows]
    else:
        sel_rows = si_dev[:T].cpu().numpy()[rows]
    par = oracle_parity(cfg, weights, x_host[rows], out_np[rows], sel_rows,
                        max(1, (os.cpu_count() or 1) // world))
    if ep:
        with jm.Context(local_rank, T, 1) as one:
            d1, keep1 = synth.desc_for(cfg, weights)
            one.upload(0, d1)
            o1, s1, _ = one.forward(0, x_host[:T])
        par["routing_exact_vs_single_gpu"] = bool(np.array_equal(s1, si_ep))
        par["max_row_rel_err_vs_single_gpu"] = float(row_rel_err(out_np, o1).max())
        par["rows_vs_single_gpu"] = int(T)
        agg = torch.tensor([par["max_row_rel_err"], par["max_row_rel_err_vs_single_gpu"],
                            0.0 if (par["routing_exact"] and par["routing_exact_vs_single_gpu"]) else 1.0],
                           device="cuda", dtype=torch.float64)
        dist.all_reduce(agg, op=dist.ReduceOp.MAX)
        par.update({"max_row_rel_err": float(agg[0]), "max_row_rel_err_vs_single_gpu": float(agg[1]),
                    "routing_exact": bool(agg[2] == 0.0), "routing_exact_vs_single_gpu": bool(agg[2] == 0.0),
                    "ranks": world, "rows_checked": par["rows_checked"] * world,
                    "rows_vs_single_gpu": par["rows_vs_single_gpu"] * world})

    sweep = []
    for t in sweep_T:
        ms, _ = tm.run(t, 10, False)
        for _ in range(2):
            step(t)
        torch.cuda.synchronize()
        selt = si_dev[:t].cpu().numpy()
        b = kernel_bytes(cfg, weights, selt, t)["layer"]
        m = statistics.median(ms)
        hbm = peaks()[0]
        sweep.append({"T": t, "tokens_per_s": round(t / (m / 1e3), 1), "us_per_layer": round(1e3 * m, 2),
                      "layer_gbs": round(b / (m / 1e3) / 1e9, 1), "layer_hbm_frac": round(b / (m / 1e3) / 1e9 / hbm, 4)})

    # end to end through the C ABI with pinned host buffers (copies inside the timed region)
    xh = torch.from_numpy(x_host[:T].copy()).pin_memory()
    oh = torch.empty_like(xh).pin_memory()
    sih = torch.empty((T, cfg.k), dtype=torch.int32).pin_memory()
    swh = torch.empty((T, cfg.k), dtype=torch.float32).pin_memory()
    e2e_s = 0.0
    for i in range(args.steps):
        flush.fill_(i & 0xFF)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        if ep:
            ctx.forward_ep_ptrs(0, T, xh.data_ptr(), oh.data_ptr(), jm.PTR_HOST)
        else:
            ctx.forward_ptrs(0, T, xh.data_ptr(), oh.data_ptr(), sih.data_ptr(), swh.data_ptr(), jm.PTR_HOST)
        e2e_s += time.perf_counter() - t0
    if world > 1:
        tt = torch.tensor([e2e_s], device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e_s = float(tt.item())
    e2e = world * T * args.steps / e2e_s

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        threads = os.cpu_count() or 1
        v, n, el = cpu_baseline(cfg, weights, x_host[:T], args.cpu_seconds, threads)
        cpu = {"value": round(v, 3), "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"{n} tokens of the T={T} workload in {el:.1f} s (oracle, one token at a time)"}

    configs = []
    if world == 1 and not args.no_configs:
        ctx.close()   # frees the headline layer before the larger ones
        for cid, t in EXTRA_CONFIGS:
            if cid == args.config and t == T:
                continue
            try:
                configs.append(extra_config(torch, jm, synth, cid, t, stream, flush, tensor_peaks))
            except Exception as e:
                configs.append({"workload": f"{synth.CONFIGS[cid].name} T={t}", "error": str(e)[:300]})

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(layer_ms, 5),
            "higher_is_better": True, "scaling": "strong" if (ep and args.strong) else "weak",
            "vs_baseline": None, "dtype": "int8",
            "data": "synthetic (seeded N(0,1) activations, N(0,0.02) weights quantised to GGUF blocks)",
            "config": workload_config(cfg, T, world, args.strong, U_global),
            "timing": "L2 flushed between timed steps (256 MiB write); per-step CUDA events on the library's "
                      "stream; max over ranks" + (f"; context flags {args.flags}" if args.flags else ""),
            "roofline": roofline,
            "layer_roofline": {"bytes": int(kb["layer"]), "gbs": round(kb["layer"] / (layer_ms / 1e3) / 1e9, 1),
                               "frac": round(kb["layer"] / (layer_ms / 1e3) / 1e9 / peaks()[0], 4)},
            "kernels": kernels,
            "gpu_launches": int(launches),
            "parity": par,
            "e2e": {"value": round(e2e, 1), "unit": UNIT,
                    "h2d_bytes_per_step": int(T * cfg.H * 4),
                    "d2h_bytes_per_step": int(T * cfg.H * 4 + (0 if ep else T * cfg.k * 8))},
            "sweep": sweep,
            "configs": configs,
            "tensor_peaks": tensor_peaks,
            "cpu_baseline": cpu,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    ctx.close()
    if world > 1:
        dist.destroy_process_group()


def main():
    args = parse()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
