#!/usr/bin/env python
"""Benchmark of the fused-MoE hot path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfg3] [--impl ours|reference]

Workload (BASELINE metric "fused-MoE ms/call and TFLOP/s (H7168,E256,top8,4096 tok) vs tensor-core
peak"): cfg3 = T=4096 tokens, H=7168, I=2048, E=256 experts, top-8, fp16, seeded synthetic inputs
(weights ~ N(0, 1/fan_in), hidden ~ N(0,1), softmax-top-8 routing of N(0,1) logits). One step = one
``fused_moe`` call (routing alignment, gather, Stage1, Stage2 + combine). The weights (22.5 GB) are
far larger than L2 (126 MB), so every step streams them from HBM; no L2 flush is needed.

value  = algorithmic TFLOP/s = 2 * T * k * 3 * H * I / (device time per step), all ranks summed;
e2e    = the same metric through the public API with host inputs: pinned hidden_states, topk_ids and
         topk_weights copied in and the output copied back inside the timed region each step;
roofline = Stage1 (the dominant kernel): algorithmic bytes / measured average launch time vs the
         measured HBM copy bandwidth (MEASURED_PEAKS.json);
cpu_baseline = the oracle (a port of the reference's PyTorch operator) on the host cores, on a
         bounded sample of experts, rank 0 at N=1 only.
With --gpus N > 1 the step is the expert-parallel fused MoE (muxi_race_b200.ep): the 256 experts
are sharded E/N per GPU (load-balanced placement from a calibration routing sample) and tokens are
dispatched and combined with NCCL all-to-all (--ep-mode nccl, default) or over NVLink peer memory by
the library's kernels (--ep-mode p2p). Default: weak scaling, 4096 tokens per rank (N = 1 is
exactly cfg3, N = 8 is the 32768-token cfg5 size); --config cfg5: strong scaling, 32768 tokens in
total with the Zipf-skewed routing. value = all ranks' algorithmic FLOPs / the slowest rank's time.
--impl reference times the reference's CPU operator (the oracle port) instead.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
METRIC = "fused-MoE ms/call and TFLOP/s (H7168,E256,top8,4096 tok) vs tensor-core peak"
UNIT = "TFLOP/s"
STAGES = ["align", "gather", "stage1", "stage2"]


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples (200 ms) of this GPU's SM clock and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: torch.device):
        self.samples = []
        self.proc = None
        props = torch.cuda.get_device_properties(device)
        dom, bus, dv = (getattr(props, a, None) for a in ("pci_domain_id", "pci_bus_id", "pci_device_id"))
        self.sel = f"{dom:08X}:{bus:02X}:{dv:02X}.0" if None not in (dom, bus, dv) else None

    def start(self):
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"]
        if self.sel:
            cmd += ["-i", self.sel]
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.samples.append(parts)

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=5)
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if s[5 + i].lower() == "active"})
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(mx) if mx else None,
            "reasons": reasons,
            "samples": len(self.samples),
        }


# ----------------------------------------------------------------------------- distributed
def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def gather_over_ranks(v: float, world: int) -> list:
    if world == 1:
        return [v]
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    out = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [round(float(x.item()), 4) for x in out]


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ----------------------------------------------------------------------------- CPU baseline
_CPU_WEIGHTS: dict = {}


def cpu_sample(cfg, ids_cpu, w_cpu, x_cpu, budget_s: float, seed: int = 0, max_weight_bytes: float = 1.5e9):
    """Oracle (port of the reference's PyTorch operator) on a subset of experts, on the host cores.

    Returns (flops, seconds, n_experts, rows). Weights of the sampled experts are generated on the
    CPU with the workload's distribution (the values do not change the arithmetic cost); at most
    max_weight_bytes of them, so host memory stays bounded, and the subset is run repeatedly until
    about budget_s seconds of work have been timed.
    """
    from oracle.moe_ref import fused_moe_ref

    E, H, I, k = cfg.E, cfg.H, cfg.I, cfg.topk
    flat = ids_cpu.reshape(-1).long()
    elt = 1 if cfg.int8 else 2
    n_mem = int(max(1, min(E, max_weight_bytes // (3 * H * I * elt))))

    def make(n):
        sel = torch.arange(n)
        remap = torch.full((E,), -1, dtype=torch.long)
        remap[sel] = torch.arange(n)
        ids_r = remap[flat].reshape(ids_cpu.shape)
        key = (cfg.name, n)
        if key not in _CPU_WEIGHTS:  # generated once per process: the values do not change the cost
            g = torch.Generator().manual_seed(seed)
            if len(_CPU_WEIGHTS) >= 2:  # the one-expert estimate and the sampled subset
                _CPU_WEIGHTS.pop(next(iter(_CPU_WEIGHTS)))
            _CPU_WEIGHTS[key] = ((torch.randn((n, 2 * I, H), generator=g) * H ** -0.5).to(cfg.dtype),
                                 (torch.randn((n, H, I), generator=g) * I ** -0.5).to(cfg.dtype))
        w13, w2 = _CPU_WEIGHTS[key]
        return ids_r, w13, w2, int((ids_r >= 0).sum())

    ids_r, w13, w2, rows = make(1)  # estimate (also warms the BLAS threads)
    t0 = time.perf_counter()
    fused_moe_ref(x_cpu, w13, w2, ids_r, w_cpu)
    t1 = time.perf_counter() - t0
    n = int(max(1, min(n_mem, budget_s / max(t1, 1e-3))))
    ids_r, w13, w2, rows = make(n)
    flops = dt = 0.0
    while True:
        t0 = time.perf_counter()
        fused_moe_ref(x_cpu, w13, w2, ids_r, w_cpu)
        dt += time.perf_counter() - t0
        flops += 2.0 * rows * 3 * H * I
        if dt >= 0.5 * budget_s or dt + dt / max(flops, 1.0) * 2.0 * rows * 3 * H * I > budget_s:
            break
    return flops, dt, n, rows


# ----------------------------------------------------------------------------- our arm
def bench_ours(args, world, rank, local):
    if world > 1:
        return bench_ep(args, world, rank, local)
    import muxi_race_b200 as m
    from muxi_race_b200 import _lib
    from muxi_race_b200.workloads import CONFIGS, make_hidden, make_router_logits, make_routing, make_weights

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    cfg = CONFIGS[args.config]
    peaks, peak_kind = load_peaks()
    variant = args.variant
    if cfg.int8 and variant in ("ordered", "router"):
        raise SystemExit(f"--variant {variant} runs the fp16/bf16 route; {cfg.name} is an int8 configuration")
    q8 = cfg.int8 or variant == "fp8"

    w13, w2 = make_weights(cfg, seed=0, device=dev)
    x = make_hidden(cfg, seed=1 + rank, device=dev)
    ids, tw = make_routing(cfg, seed=2 + rank, device=dev)
    # inputs of one call after x: (topk_ids, topk_weights), or the router logits for "router"
    ins = [make_router_logits(cfg, seed=2 + rank, device=dev)] if variant == "router" else [ids, tw]
    if q8:
        quant = m.quantize_rows_fp8 if variant == "fp8" else m.quantize_rows_int8
        fused_q = m.fused_moe_fp8 if variant == "fp8" else m.fused_moe_int8
        w13q, w13s = quant(w13)
        w2q, w2s = quant(w2)
        del w13, w2
        fn = lambda xx, ii, ww, oo: fused_q(xx, w13q, w13s, w2q, w2s, ii, ww, out=oo)  # noqa: E731
    elif variant == "router":
        fn = lambda xx, lg, oo: m.fused_moe_router(xx, w13, w2, lg, cfg.topk, out=oo)  # noqa: E731
    else:
        det = variant == "ordered"
        fn = lambda xx, ii, ww, oo: m.fused_moe(xx, w13, w2, ii, ww, out=oo, deterministic=det)  # noqa: E731
    out = torch.empty((cfg.T, cfg.H), dtype=cfg.dtype, device=dev)
    routes = cfg.T * cfg.topk
    active = int(torch.unique(ids).numel())
    flops = cfg.flops()
    n_ev = 6 if q8 else 5

    for _ in range(args.warmup):
        fn(x, *ins, out)
    torch.cuda.synchronize()
    st = m.device_status()
    assert st == 0, f"device status {st} (bit 0 wait timeout, 1 bad expert, 2 bad route) after warm-up"

    # ---- device-resident timing, with stage-boundary events on the launch stream
    stream = torch.cuda.current_stream(dev)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(n_ev)] for _ in range(args.steps)]
    for row in evs:
        for e in row:
            e.record(stream)  # materialise the handles
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(dev)
    torch.cuda.synchronize()
    barrier(world)
    clocks.start()
    start.record(stream)
    for k in range(args.steps):
        _lib.set_profile_events(evs[k])
        fn(x, *ins, out)
    _lib.set_profile_events(None)
    end.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    ms_local = start.elapsed_time(end) / args.steps
    ms = max_over_ranks(ms_local, world)

    def stage_ms(a, b):
        return sum(evs[k][a].elapsed_time(evs[k][b]) for k in range(args.steps)) / args.steps

    stages = {"align": stage_ms(0, 1), "gather": stage_ms(1, 2), "stage1": stage_ms(2, 3)}
    if q8:
        stages["requant"] = stage_ms(3, 4)
        stages["stage2"] = stage_ms(4, 5)
    else:
        stages["stage2"] = stage_ms(3, 4)
    # With the single-kernel MoE (the default where a call averages < 1.8 routing blocks per
    # expert) the library records the Stage1 and Stage2 boundary events around one launch: the
    # Stage2 interval is then empty and the Stage1 interval covers both stages.
    single = not q8 and stages["stage2"] < 0.02 * stages["stage1"]
    if single:
        stages = {"align": stages["align"], "gather": stages["gather"], "single_kernel": stages["stage1"]}

    # ---- end to end through the public API with host buffers: every step uploads its inputs
    #      from pinned host memory and downloads its result; by default through HostPipeline
    #      (copies of consecutive calls overlapped with compute on two copy streams), with the
    #      serial copy -> call -> copy loop as the fallback and with --e2e serial
    hosts = [t.cpu().pin_memory() for t in [x] + ins]
    out_h = torch.empty(out.shape, dtype=out.dtype).pin_memory()

    def e2e_serial():
        devs = [torch.empty_like(t) for t in [x] + ins]

        def step():
            for d, h in zip(devs, hosts):
                d.copy_(h, non_blocking=True)
            fn(*devs, out)
            out_h.copy_(out, non_blocking=True)

        torch.cuda.synchronize()
        barrier(world)  # the ranks enter the end-to-end phase together
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        barrier(world)
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record(stream)
        for _ in range(args.steps):
            step()
        e2.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        return s2.elapsed_time(e2) / args.steps

    def e2e_overlapped():
        from muxi_race_b200.host_pipeline import HostPipeline

        pipe = HostPipeline(fn, [x] + ins, out)
        # one pinned host output per buffer slot: downloads of calls in flight at the same time
        # never write the same host memory
        outs_h = [out_h] + [torch.empty_like(out_h).pin_memory() for _ in range(pipe.depth - 1)]
        torch.cuda.synchronize()
        barrier(world)
        for i in range(args.warmup):
            pipe.submit(hosts, outs_h[i % pipe.depth])
        pipe.synchronize()
        torch.cuda.synchronize()
        barrier(world)
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record(stream)
        pipe.up.wait_event(s2)  # the first upload starts inside the timed region
        for i in range(args.steps):
            pipe.submit(hosts, outs_h[i % pipe.depth])
        pipe.join(stream)  # the last download ends inside it
        e2.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        # the last call's host result against the device-resident call on the same inputs (the
        # top-k combine's atomic order differs between calls: the fused tests' tolerance)
        last = outs_h[(args.steps - 1) % pipe.depth].float()
        ref = out.float().cpu()
        err = (last - ref).abs()
        e2e_checked["max_abs_err"] = float(err.max())
        e2e_checked["ok"] = bool((err <= 1e-2 + 1e-2 * ref.abs()).all())
        return s2.elapsed_time(e2) / args.steps

    e2e_mode = "serial (copy, call, copy on one stream)"
    e2e_checked = {}
    serial_local = e2e_serial()  # always measured; reported beside the overlapped leg
    e2e_local = serial_local
    if args.e2e == "overlapped":
        try:
            e2e_local = e2e_overlapped()
            e2e_mode = "overlapped (HostPipeline: uploads and downloads of consecutive calls on two copy streams)"
        except Exception as ex:  # noqa: BLE001 - keep the serial measurement, and say so
            torch.cuda.synchronize()
            e2e_mode = f"serial after HostPipeline failed ({type(ex).__name__}: {ex})"
    e2e_ms = max_over_ranks(e2e_local, world)
    serial_ms = max_over_ranks(serial_local, world)
    clock_info = clocks.stop()  # sampled across both timed regions
    h2d = sum(h.numel() * h.element_size() for h in hosts)
    d2h = out_h.numel() * out_h.element_size()
    st = m.device_status()
    assert st == 0, f"device status {st} (bit 0 wait timeout, 1 bad expert, 2 bad route) after timing"

    # ---- roofline of the dominant kernel (Stage1, or the single kernel that runs both stages):
    #      algorithmic bytes per launch / launch time. Stage1: the active experts' gate and up
    #      weights, the routed token rows and U; Stage2: the down weights, U and the token-major
    #      output (its combine's adds of a token's rows meet in L2).
    elt = 1 if q8 else 2
    s1_bytes = active * 2 * cfg.I * cfg.H * elt + routes * cfg.H * elt + routes * cfg.I * 2
    s2_bytes = active * cfg.H * cfg.I * elt + routes * cfg.I * 2 + cfg.T * cfg.H * 2
    if single:
        k_name, k_bytes, k_ms, k_traffic = ("moe_single_kernel (Stage1 + Stage2)", s1_bytes + s2_bytes,
                                            stages["single_kernel"], "single_dram_bytes_per_launch")
    else:
        k_name, k_bytes, k_ms, k_traffic = ("stage1 (moe_gemm_kernel<kStage1>)", s1_bytes, stages["stage1"],
                                            "stage1_dram_bytes_per_launch")
    k_gbs = k_bytes / (k_ms * 1e-3) / 1e9
    traffic = None
    tp = os.path.join(ROOT, "profiles", f"traffic_{cfg.name}.json")
    # the committed capture is of the default fp16 call: no traffic figure for other variants
    if os.path.exists(tp) and variant == "default" and not q8:
        with open(tp) as f:
            traffic = json.load(f).get(k_traffic)
    roofline = {
        "bound": "hbm", "kernel": k_name, "achieved": round(k_gbs, 1),
        "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": round(k_gbs / peaks["hbm_gbs"], 4),
        "traffic": traffic, "algorithmic_bytes": k_bytes, "peak_kind": peak_kind,
    }
    total_bytes = float(active) * 3 * cfg.H * cfg.I * elt + cfg.io_bytes()  # elt: 1 for int8 and fp8
    t_roof_ms = max(flops / (peaks["bf16_tflops"] * 1e12), total_bytes / (peaks["hbm_gbs"] * 1e9)) * 1e3

    result = {
        "metric": METRIC,
        "value": round(world * flops / (ms * 1e-3) / 1e12, 2),
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp8" if variant == "fp8" else "int8" if cfg.int8 else ("fp16" if cfg.dtype == torch.float16 else "bf16"),
        "data": "synthetic (seeded; weights N(0,1/fan_in), hidden N(0,1), softmax-top-k of N(0,1) logits)",
        "config": {
            "workload": f"{cfg.name}: fused MoE T={cfg.T} H={cfg.H} I={cfg.I} E={cfg.E} top-{cfg.topk}",
            "tokens_per_rank": cfg.T, "routed_rows_per_rank": routes, "active_experts": active,
            "parallelism": "replicas" if world > 1 else "single",
            "l2": f"inputs larger than L2 ({active * 3 * cfg.H * cfg.I * elt / 1e9:.1f} GB of "
                  "expert weights streamed per step)",
            **({} if variant == "default" else {"variant": variant}),
        },
        "ms_per_call": round(ms, 4),
        "tflops_per_gpu": round(flops / (ms * 1e-3) / 1e12, 2),
        "stage_ms": {k: round(v, 4) for k, v in stages.items()},
        "call_roofline": {"ms": round(t_roof_ms, 4), "frac": round(t_roof_ms / ms, 4),
                          "bytes": total_bytes, "flops": flops,
                          "tensor_peak_frac_spec": round(flops / (ms * 1e-3) / 2.25e15, 4),
                          "tensor_peak_frac_measured": round(flops / (ms * 1e-3) / (peaks["bf16_tflops"] * 1e12), 4)},
        "roofline": roofline,
        "e2e": {"value": round(world * flops / (e2e_ms * 1e-3) / 1e12, 2), "unit": UNIT, "ms_per_step": round(e2e_ms, 4),
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "transfers": e2e_mode,
                "serial": {"value": round(world * flops / (serial_ms * 1e-3) / 1e12, 2),
                           "ms_per_step": round(serial_ms, 4)},
                **({"output_check": e2e_checked} if e2e_checked else {})},
        # per call: alignment (count or router, scan, scatter), block groups, gather, Stage1, Stage2;
        # 8-bit routes add the intermediate requantisation, the ordered combine its two kernels
        "gpu_launches": args.steps * (8 if q8 else 9 if variant == "ordered" else 6 if single else 7),
        "clocks": clock_info,
    }
    if world == 1 and cfg.name == "cfg3" and variant == "default" and not args.no_north_star:
        # the 1-GPU denominator of the north star's scaling target (cfg5 on one GPU, same weights)
        result["north_star_cfg5"] = time_cfg5_strong(args, 1, rank, local, w13, w2)
    if world == 1 and not args.no_cpu_baseline:
        f, dt, n, rows = cpu_sample(cfg, ids.cpu(), tw.cpu(), x.cpu(), budget_s=args.cpu_budget)
        result["cpu_baseline"] = {
            "value": round(f / dt / 1e12, 6), "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"oracle fused_moe_ref over the {rows} routed rows of {n}/{cfg.E} experts "
                      f"({dt:.1f} s); full call extrapolates to {flops / (f / dt):.1f} s",
        }
    if rank == 0:
        print(json.dumps(result), flush=True)



# ----------------------------------------------------------------------------- north-star EP case
def time_cfg5_strong(args, world, rank, local, w13_full=None, w2_full=None):
    """The north star's expert-parallel case: cfg5 (32768 tokens in total, Zipf(1.1)-skewed routing,
    H=7168, I=2048, E=256, top-8) split evenly over the ranks (strong scaling). On one GPU the
    fused call on all 32768 tokens (``w13_full`` / ``w2_full``: cfg3's weights, same shapes). Returns
    {"ms": max over ranks, "tokens_per_s", "tflops"}; every rank takes the same collective steps."""
    import muxi_race_b200 as m
    from muxi_race_b200.workloads import CONFIGS, make_hidden, make_routing, make_weights

    dev = torch.device("cuda", local)
    cfg = CONFIGS["cfg5"]
    T_rank = cfg.T // world
    steps, warm = max(3, min(args.steps, 10)), max(3, args.warmup)
    x = make_hidden(cfg, seed=1 + rank, device=dev, T=T_rank)
    ids, tw = make_routing(cfg, seed=2 + rank, device=dev, T=T_rank)
    if world == 1:
        out = torch.empty((T_rank, cfg.H), dtype=cfg.dtype, device=dev)
        fn = lambda: m.fused_moe(x, w13_full, w2_full, ids, tw, out=out)  # noqa: E731
        moe = None
    else:
        from muxi_race_b200.ep import ExpertParallelMoE, ExpertPlacement, PeerMemoryEP

        cal_ids, _ = make_routing(cfg, seed=999, device=dev, T=8192)
        loads = torch.bincount(cal_ids.flatten().long(), minlength=cfg.E).float().cpu().tolist()
        placement = ExpertPlacement.balanced(loads, world)
        w13, w2 = make_weights(cfg, seed=0, device=dev, experts=placement.local_experts(rank))
        if args.ep_mode == "p2p":
            moe = PeerMemoryEP(w13, w2, placement, max_tokens=T_rank, topk=cfg.topk, combine=args.ep_combine)
        else:
            moe = ExpertParallelMoE(w13, w2, placement, chunks=args.ep_chunks)
        fn = lambda: moe(x, ids, tw)  # noqa: E731
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    barrier(world)
    stream = torch.cuda.current_stream(dev)
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record(stream)
    for _ in range(steps):
        fn()
    s1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(s0.elapsed_time(s1) / steps, world)
    if moe is not None and hasattr(moe, "close"):
        moe.close()
    st = m.device_status()
    assert st == 0, f"device status {st} after the cfg5 strong-scaling measurement"
    peaks, peak_kind = load_peaks()
    tflops = cfg.flops() / (ms * 1e-3) / 1e12
    per_gpu = tflops / world
    burst = peaks.get("bf16_tflops")
    sustained = peaks.get("bf16_tflops_sustained")
    return {"workload": f"cfg5: T={cfg.T} in total ({T_rank} per rank), Zipf({cfg.zipf_s}) routing, "
                        f"H={cfg.H} I={cfg.I} E={cfg.E} top-{cfg.topk}",
            "n_gpus": world, "steps": steps, "ms": round(ms, 4), "tokens_per_s": round(cfg.T / (ms * 1e-3)),
            "tflops": round(tflops, 2),
            # per GPU, against the dense 16-bit tensor peak (the north star's 60% target is of peak)
            "tensor_peak_frac_per_gpu": {"spec_2250": round(per_gpu / 2250.0, 4),
                                         "measured_burst": round(per_gpu / burst, 4) if burst else None,
                                         "measured_sustained": round(per_gpu / sustained, 4) if sustained else None,
                                         "peak_kind": peak_kind}}

# ----------------------------------------------------------------------------- expert parallel
def bench_ep(args, world, rank, local):
    import torch.distributed as dist

    import muxi_race_b200 as m
    from muxi_race_b200 import _lib
    from muxi_race_b200.ep import ExpertParallelMoE, ExpertPlacement, PeerMemoryEP
    from muxi_race_b200.workloads import CONFIGS, make_hidden, make_routing, make_weights

    dev = torch.device("cuda", local)
    cfg = CONFIGS[args.config]
    strong = args.config == "cfg5"
    T_rank = cfg.T // world if strong else cfg.T
    peaks, peak_kind = load_peaks()

    # load-balanced placement from a calibration sample (same on every rank)
    cal_ids, _ = make_routing(cfg, seed=999, device=dev, T=8192)
    loads = torch.bincount(cal_ids.flatten().long(), minlength=cfg.E).float().cpu().tolist()
    placement = ExpertPlacement.balanced(loads, world)
    mine = placement.local_experts(rank)
    w13, w2 = make_weights(cfg, seed=0, device=dev, experts=mine)
    x = make_hidden(cfg, seed=1 + rank, device=dev, T=T_rank)
    ids, tw = make_routing(cfg, seed=2 + rank, device=dev, T=T_rank)
    p2p = args.ep_mode == "p2p"
    if p2p:
        moe = PeerMemoryEP(w13, w2, placement, max_tokens=T_rank, topk=cfg.topk, combine=args.ep_combine)
    else:
        moe = ExpertParallelMoE(w13, w2, placement, chunks=args.ep_chunks)
    n_chunks = 1 if p2p else args.ep_chunks

    for _ in range(args.warmup):
        moe(x, ids, tw)
    torch.cuda.synchronize()
    st = m.device_status()
    assert st == 0, f"device status {st} (bit 0 wait timeout, 1 bad expert, 2 bad route) after warm-up"

    # stage-boundary events for every local fused-MoE call (one per chunk) of every timed step
    stream = torch.cuda.current_stream(dev)
    evs = [[[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(n_chunks)]
           for _ in range(args.steps)]
    for step in evs:
        for row in step:
            for e in row:
                e.record(stream)
    slot = {"k": 0, "c": 0}
    if not p2p:
        local_moe = moe.ops.local_moe

        def profiled_local_moe(*a, **kw):
            _lib.set_profile_events(evs[slot["k"]][min(slot["c"], n_chunks - 1)])
            slot["c"] += 1
            return local_moe(*a, **kw)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(dev) if rank == 0 else None
    torch.cuda.synchronize()
    barrier(world)
    if clocks:
        clocks.start()
    start.record(stream)
    if not p2p:
        moe.ops.local_moe = profiled_local_moe
    for k in range(args.steps):
        slot["k"], slot["c"] = k, 0
        if p2p:
            _lib.set_profile_events(evs[k][0])
        moe(x, ids, tw)
    if not p2p:
        moe.ops.local_moe = local_moe
    _lib.set_profile_events(None)
    end.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(start.elapsed_time(end) / args.steps, world)
    rank_ms = gather_over_ranks(start.elapsed_time(end) / args.steps, world)
    # per-step wall on the device: from one step's first stage event to the next step's
    steps_ms = [evs[k][0][0].elapsed_time(evs[k + 1][0][0]) for k in range(args.steps - 1)]
    rank_step_max = gather_over_ranks(max(steps_ms) if steps_ms else 0.0, world)
    rank_step_med = gather_over_ranks(statistics.median(steps_ms) if steps_ms else 0.0, world)

    def stage_ms(a, b):  # summed over the chunks of a step
        return sum(row[a].elapsed_time(row[b]) for step in evs for row in step) / args.steps

    local_ms = {"align": stage_ms(0, 1), "gather": stage_ms(1, 2), "stage1": stage_ms(2, 3), "stage2": stage_ms(3, 4)}
    local_ms["exchange_and_rest"] = start.elapsed_time(end) / args.steps - sum(local_ms.values())

    # algorithmic work: all ranks' routed rows; this rank's local Stage1 rows and experts
    tot = torch.tensor([float(T_rank * cfg.topk)], dtype=torch.float64, device=dev)
    dist.all_reduce(tot)
    flops_total = 2.0 * float(tot.item()) * 3 * cfg.H * cfg.I
    # this rank's local routes and active experts, from every rank's routing
    all_ids = [torch.empty_like(ids) for _ in range(world)]
    dist.all_gather(all_ids, ids)
    routed = torch.cat(all_ids).flatten().long()
    mine_mask = placement.expert_rank.to(dev)[routed] == rank
    local_routes = int(mine_mask.sum().item())
    local_active = int(torch.unique(routed[mine_mask]).numel())
    s1_flops = 2.0 * local_routes * 2 * cfg.I * cfg.H
    s1_bytes = local_active * 2 * cfg.I * cfg.H * 2 + local_routes * cfg.H * 2 + local_routes * cfg.I * 2
    # the single-kernel MoE records the Stage1 and Stage2 events around one launch
    single = local_ms["stage2"] < 0.02 * local_ms["stage1"]
    if single:
        s1_flops += 2.0 * local_routes * cfg.I * cfg.H
        s1_bytes += local_active * cfg.H * cfg.I * 2 + local_routes * cfg.I * 2 + local_routes * cfg.H * 2
    s1_s = local_ms["stage1"] * 1e-3
    t_mem = s1_bytes / (peaks["hbm_gbs"] * 1e9)
    t_cmp = s1_flops / (peaks["bf16_tflops"] * 1e12)
    if t_cmp >= t_mem:
        roofline = {"bound": "tensor", "achieved": round(s1_flops / s1_s / 1e12, 1), "peak": peaks["bf16_tflops"],
                    "unit": "TFLOP/s", "frac": round(s1_flops / s1_s / 1e12 / peaks["bf16_tflops"], 4)}
    else:
        roofline = {"bound": "hbm", "achieved": round(s1_bytes / s1_s / 1e9, 1), "peak": peaks["hbm_gbs"],
                    "unit": "GB/s", "frac": round(s1_bytes / s1_s / 1e9 / peaks["hbm_gbs"], 4)}
    roofline.update({"kernel": ("single kernel" if single else "stage1") + " (rank 0's local fused MoE)",
                     "traffic": None, "peak_kind": peak_kind,
                     "algorithmic_bytes": s1_bytes, "algorithmic_flops": s1_flops})

    # end to end: host inputs in, output back, every step
    x_h, ids_h, tw_h = x.cpu().pin_memory(), ids.cpu().pin_memory(), tw.cpu().pin_memory()
    out_h = torch.empty((T_rank, cfg.H), dtype=cfg.dtype).pin_memory()
    x_d, ids_d, tw_d = torch.empty_like(x), torch.empty_like(ids), torch.empty_like(tw)

    def e2e_step():
        x_d.copy_(x_h, non_blocking=True)
        ids_d.copy_(ids_h, non_blocking=True)
        tw_d.copy_(tw_h, non_blocking=True)
        out_h.copy_(moe(x_d, ids_d, tw_d), non_blocking=True)

    def e2e_serial():
        torch.cuda.synchronize()
        barrier(world)  # the ranks enter the end-to-end phase together
        for _ in range(args.warmup):
            e2e_step()
        torch.cuda.synchronize()
        barrier(world)
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record(stream)
        for _ in range(args.steps):
            e2e_step()
        e2.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        return s2.elapsed_time(e2) / args.steps

    def e2e_overlapped():
        # the same forwards through HostPipeline: uploads and downloads of neighbouring steps on two
        # copy streams, one pinned host output per buffer slot; every rank submits the same steps
        from muxi_race_b200.host_pipeline import HostPipeline

        pipe = HostPipeline(lambda xx, ii, ww, oo: oo.copy_(moe(xx, ii, ww)), [x, ids, tw],
                            torch.empty((T_rank, cfg.H), dtype=cfg.dtype, device=dev))
        outs_h = [out_h] + [torch.empty_like(out_h).pin_memory() for _ in range(pipe.depth - 1)]
        torch.cuda.synchronize()
        barrier(world)
        for i in range(args.warmup):
            pipe.submit([x_h, ids_h, tw_h], outs_h[i % pipe.depth])
        pipe.synchronize()
        torch.cuda.synchronize()
        barrier(world)
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record(stream)
        pipe.up.wait_event(s2)
        for i in range(args.steps):
            pipe.submit([x_h, ids_h, tw_h], outs_h[i % pipe.depth])
        pipe.join(stream)
        e2.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        return s2.elapsed_time(e2) / args.steps

    serial_ms = max_over_ranks(e2e_serial(), world)
    e2e_ms, e2e_mode = serial_ms, "serial (copy, forward, copy on one stream)"
    if args.e2e == "overlapped":
        e2e_ms = max_over_ranks(e2e_overlapped(), world)
        e2e_mode = "overlapped (HostPipeline: uploads and downloads of consecutive steps on two copy streams)"
    clock_info = clocks.stop() if clocks else None  # sampled across both timed regions
    st = m.device_status()
    assert st == 0, f"device status {st} (bit 0 wait timeout, 1 bad expert, 2 bad route) after timing"
    h2d = x_h.numel() * x_h.element_size() + ids_h.numel() * ids_h.element_size() + tw_h.numel() * tw_h.element_size()
    d2h = out_h.numel() * out_h.element_size()
    send, recv = moe.last_counts if not p2p else (None, None)
    if p2p:
        moe.close()
    north = None
    if not strong and not args.no_north_star:
        del moe, w13, w2
        torch.cuda.empty_cache()
        north = time_cfg5_strong(args, world, rank, local)

    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": round(flops_total / (ms * 1e-3) / 1e12, 2), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": "strong" if strong else "weak", "vs_baseline": None, "dtype": "fp16",
            "data": "synthetic (seeded; weights N(0,1/fan_in), hidden N(0,1), softmax-top-k of N(0,1) logits"
                    + (" + log-Zipf(1.1) expert bias)" if cfg.zipf_s else ")"),
            "config": {"workload": f"expert-parallel fused MoE, {cfg.name} shapes H={cfg.H} I={cfg.I} E={cfg.E} "
                                   f"top-{cfg.topk}, {T_rank} tokens per rank, {T_rank * world} in total",
                       "tokens_per_rank": T_rank, "parallelism": f"ep{world}", "experts_per_rank": len(mine),
                       "placement": "balanced (greedy LPT from an 8192-token calibration sample)",
                       "ep_exchange": ("peer memory: NVLink loads of the token rows and "
                                       + ("Stage2 adding into the home ranks' regions (push combine)"
                                          if args.ep_combine == "push" else "loads of the partial outputs")
                                       + " inside the library's kernels, flag barriers; no collectives library; "
                                       + f"token gather: {os.environ.get('MOE_B200_EP_GATHER') or 'dedup'}")
                       if p2p else f"NCCL all_to_all_single, {n_chunks} chunk(s)",
                       "l2": "inputs larger than L2 (expert weights streamed per step)"},
            "ms_per_call": round(ms, 4), "tflops_per_gpu": round(flops_total / world / (ms * 1e-3) / 1e12, 2),
            "rank0_stage_ms": {k: round(v, 4) for k, v in local_ms.items()},
            "rank_ms": rank_ms, "rank_step_ms_median": rank_step_med, "rank_step_ms_max": rank_step_max,
            "rank0_rows": {"send": send, "recv": recv, "local_routes": local_routes, "local_active_experts": local_active},
            "roofline": roofline,
            "e2e": {"value": round(flops_total / (e2e_ms * 1e-3) / 1e12, 2), "unit": UNIT, "ms_per_step": round(e2e_ms, 4),
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "transfers": e2e_mode,
                    "serial": {"value": round(flops_total / (serial_ms * 1e-3) / 1e12, 2),
                               "ms_per_step": round(serial_ms, 4)}},
            # per chunk: plan 4 (pair keys + 3 alignment), pack 1, local MoE 7 (3 alignment, block
            # groups, gather, Stage1, Stage2), combine 1
            # p2p: stage, 2 barriers, route, local MoE 7, combine = 12
            "gpu_launches": args.steps * ((11 if args.ep_combine == "push" else 12) if p2p else 13 * n_chunks),
            "clocks": clock_info,
            **({"north_star_cfg5": north} if north else {}),
        }), flush=True)


# ----------------------------------------------------------------------------- contest cases
# The reference's own benchmark shapes (初审材料/源代码/benchmark/remote_bench.py:21-29, cases 1-3) and
# its published C500 times for them: v755 on the contest's online judge
# (xpuoj_data/oj_submission_record_v755_8033.json, README.md:62-66) and that online judge's PyTorch
# baseline T_b (OJ_最终提交_SPJ报告.md:11,22,33).
CONTEST = {
    1: dict(experts=16, hidden=2048, intermediate=8192, valid=2272, high_experts=8, low_size=124,
            c500_ms=2.544, c500_torch_ms=11.251),
    2: dict(experts=32, hidden=7168, intermediate=2048, valid=4544, high_experts=22, low_size=112,
            c500_ms=4.520, c500_torch_ms=18.610),
    3: dict(experts=64, hidden=7168, intermediate=2048, valid=9088, high_experts=23, low_size=127,
            c500_ms=8.926, c500_torch_ms=35.875),
}


def contest_group_sizes(c):
    """remote_bench.py:60-75: low-size experts and high experts, interleaved."""
    high, low = c["high_experts"], c["experts"] - c["high_experts"]
    sizes = [c["low_size"]] * low
    q, r = divmod(c["valid"] - sum(sizes), high)
    sizes += [q + (i < r) for i in range(high)]
    return sizes[::2] + sizes[1::2]


def bench_run_kernel(args):
    """The reference drop-in (run_kernel) on the reference's own contest cases, one GPU."""
    import math

    import muxi_race_b200 as m

    c = CONTEST[args.case]
    dev = torch.device("cuda", 0)
    E, H, I = c["experts"], c["hidden"], c["intermediate"]
    gs = torch.tensor(contest_group_sizes(c), dtype=torch.int32)
    go = torch.cat([torch.zeros(1, dtype=torch.int32), torch.cumsum(gs, 0, dtype=torch.int32)])
    padded = (gs + 127) // 128 * 128
    gpo = torch.cat([torch.zeros(1, dtype=torch.int32), torch.cumsum(padded, 0, dtype=torch.int32)])
    gidx = torch.repeat_interleave(torch.arange(E, dtype=torch.int32), padded // 128)
    P = int(gpo[-1])
    g = torch.Generator(device=dev).manual_seed(args.case)
    x = torch.randn((P, H), generator=g, device=dev).half()
    gate = (torch.randn((E, I, H), generator=g, device=dev) / math.sqrt(I)).half()
    up = (torch.randn((E, I, H), generator=g, device=dev) / math.sqrt(I)).half()
    down = (torch.randn((E, H, I), generator=g, device=dev) / math.sqrt(H)).half()
    routed = torch.rand((c["valid"],), generator=g, device=dev)
    meta = [t.to(dev) for t in (gs, go, gpo, gidx)]
    out = torch.empty((P, H), dtype=torch.float16, device=dev)
    call = lambda: m.run_kernel(x, gate, up, down, routed, *meta, out)  # noqa: E731
    if args.graph:  # one CUDA-graph launch per call instead of the library's launches
        from muxi_race_b200.graphs import GraphedMoE

        call = GraphedMoE(lambda xx, rr, oo: m.run_kernel(xx, gate, up, down, rr, *meta, oo), x, routed, out).replay
    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        call()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / args.steps
    flops = 2.0 * c["valid"] * 3 * H * I
    wbytes = E * 3 * H * I * 2
    peaks, kind = load_peaks()
    print(json.dumps({
        "metric": f"run_kernel ms/call, contest case {args.case}", "value": round(ms, 4), "unit": "ms",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": False,
        "config": {"workload": f"reference drop-in run_kernel, contest case {args.case}: E={E} H={H} I={I} "
                               f"valid rows={c['valid']} padded rows={P}", "dtype": "fp16",
                   "launch": "CUDA graph replay" if args.graph else "direct"},
        "tflops": round(flops / (ms * 1e-3) / 1e12, 1),
        "roofline_ms": round(max(flops / (peaks['bf16_tflops'] * 1e12), (wbytes + 2 * P * H * 2) / (peaks["hbm_gbs"] * 1e9)) * 1e3, 4),
        "reference_c500": {"ms": c["c500_ms"], "contest_torch_ms": c["c500_torch_ms"],
                           "note": "published MetaX C500 times of the reference's final operator and the contest "
                                   "online judge's "
                                   "PyTorch baseline on the same shapes (different hardware)"},
    }), flush=True)


def bench_sweep(args):
    """Tile sweep (tuning, one GPU): for each configuration name in --sweep, force it for the
    stage(s) given by --sweep-stage and time the fused call on --config with stage-boundary events;
    each output is compared with the automatic choice's output (max |diff|, relative L2) and the
    device status word is checked. One JSON line per configuration, then a summary line."""
    import muxi_race_b200 as m
    from muxi_race_b200 import _lib
    from muxi_race_b200.workloads import CONFIGS, make_hidden, make_routing, make_weights

    dev = torch.device("cuda", 0)
    cfg = CONFIGS[args.config]
    w13, w2 = make_weights(cfg, seed=0, device=dev)
    x = make_hidden(cfg, seed=1, device=dev)
    ids, tw = make_routing(cfg, seed=2, device=dev)
    ref = m.fused_moe(x, w13, w2, ids, tw)
    torch.cuda.synchronize()
    assert m.device_status() == 0
    stream = torch.cuda.current_stream(dev)
    rows = []
    for name in [t for t in args.sweep.split(",") if t]:
        rec = {"tile": name, "stage": args.sweep_stage, "config": cfg.name}
        try:
            _lib.set_tile(args.sweep_stage, name)
            out = torch.empty_like(ref)
            for _ in range(args.warmup):
                m.fused_moe(x, w13, w2, ids, tw, out=out)
            torch.cuda.synchronize()
            st = m.device_status()
            evs = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(args.steps)]
            for row in evs:
                for e in row:
                    e.record(stream)
            torch.cuda.synchronize()
            for k in range(args.steps):
                _lib.set_profile_events(evs[k])
                m.fused_moe(x, w13, w2, ids, tw, out=out)
            _lib.set_profile_events(None)
            torch.cuda.synchronize()
            st |= m.device_status()
            ms = lambda a, b: sum(r[a].elapsed_time(r[b]) for r in evs) / args.steps  # noqa: E731
            d = (out.float() - ref.float())
            rec.update({"status": st, "ms_call": round(ms(0, 4), 4), "ms_stage1": round(ms(2, 3), 4),
                        "ms_stage2": round(ms(3, 4), 4), "max_abs_diff": float(d.abs().max()),
                        "rel_l2": float(d.norm() / ref.float().norm())})
        except Exception as ex:  # noqa: BLE001 - report and go on with the next configuration
            rec["error"] = f"{type(ex).__name__}: {ex}"
        finally:
            _lib.set_profile_events(None)
            _lib.set_tile(0, None)
        rows.append(rec)
        print(json.dumps(rec), flush=True)
    ok = [r for r in rows if r.get("status") == 0 and r.get("rel_l2", 1.0) < 1e-2]
    best = min(ok, key=lambda r: r["ms_call"]) if ok else None
    print(json.dumps({"sweep": cfg.name, "stage": args.sweep_stage, "best": best and best["tile"],
                      "best_ms_call": best and best["ms_call"], "n": len(rows), "passed": len(ok)}), flush=True)


# ----------------------------------------------------------------------------- reference arm
def bench_reference(args, world, rank):
    """The reference's CPU operator (oracle port of its PyTorch implementation) on the host cores."""
    from muxi_race_b200.workloads import CONFIGS, make_hidden, make_routing

    if rank != 0:
        return
    cfg = CONFIGS[args.config]
    x = make_hidden(cfg, device="cpu")
    ids, tw = make_routing(cfg, device="cpu")
    budget = max(0.2, min(args.cpu_budget, 150.0 / max(1, args.steps + args.warmup)))
    for _ in range(args.warmup):
        cpu_sample(cfg, ids, tw, x, budget_s=budget)
    tot_f = tot_t = 0.0
    last = None
    for k in range(args.steps):
        f, dt, n, rows = cpu_sample(cfg, ids, tw, x, budget_s=budget, seed=k)
        tot_f += f
        tot_t += dt
        last = (n, rows, dt)
    value = tot_f / tot_t / 1e12
    flops = cfg.flops()
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 6), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(flops / (value * 1e12) * 1e3, 1),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32 (fp16 inputs)",
        "data": "synthetic (seeded)",
        "config": {"workload": f"{cfg.name}: fused MoE T={cfg.T} H={cfg.H} I={cfg.I} E={cfg.E} top-{cfg.topk}",
                   "parallelism": "cpu"},
        "cpu_baseline": {"value": round(value, 6), "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
                         "sample": f"per step: oracle over the routed rows of a subset of experts "
                                   f"(last step {last[0]} experts, {last[1]} rows, {last[2]:.1f} s); "
                                   f"ms_per_step extrapolates one full call"},
        "e2e": {"value": round(value, 6), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="cfg3")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-budget", type=float, default=15.0,
                    help="seconds of CPU work for cpu_baseline (per step for --impl reference)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-north-star", action="store_true",
                    help="skip the cfg5 strong-scaling measurement (north-star EP case) added to the default line")
    ap.add_argument("--ep-mode", default="p2p", choices=["p2p", "nccl"],
                    help="expert parallelism: over peer memory in the library's kernels (default), or NCCL all-to-all")
    ap.add_argument("--ep-combine", default="pull", choices=["pull", "push"],
                    help="peer-memory mode: pull the owners' partial rows after the second barrier, or push them "
                         "from Stage2's epilogue into the home ranks' regions")
    ap.add_argument("--ep-chunks", type=int, default=1,
                    help="expert parallelism: token chunks whose exchanges overlap the local MoE of the others")
    ap.add_argument("--path", default="fused", choices=["fused", "run_kernel"],
                    help="run_kernel: the reference drop-in on the reference's contest case --case")
    ap.add_argument("--case", type=int, default=3, choices=sorted(CONTEST))
    ap.add_argument("--graph", action="store_true", help="--path run_kernel: replay the call as a CUDA graph")
    ap.add_argument("--sweep", default="",
                    help="tuning: comma-separated tile names to time one by one (prints one line each)")
    ap.add_argument("--sweep-stage", type=int, default=1, choices=[0, 1, 2],
                    help="stage the swept tile is forced for (0 = both)")
    ap.add_argument("--e2e", default="overlapped", choices=["overlapped", "serial"],
                    help="end-to-end leg: host transfers overlapped across calls (HostPipeline) or serial")
    ap.add_argument("--variant", default="default", choices=["default", "ordered", "router", "fp8"],
                    help="single-GPU fused call: ordered (deterministic) combine, routing from router logits "
                         "on the device, or the fp8 route")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.sweep:
        bench_sweep(args)
        return
    if args.path == "run_kernel":
        bench_run_kernel(args)
        return
    if args.impl == "reference":
        world, rank = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0"))
        bench_reference(args, world, rank)
        return
    world, rank, local = dist_setup()
    try:
        bench_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
