"""Benchmark of the NVFP4 grouped GEMM (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfg2] [--impl ours|reference]

A step is one grouped-GEMM call over the whole configuration (default: cfg2,
G=8 experts, M_g=1024, N=4096, K=7168, per-group global scale U[0.5, 2]).

Our arm (default):
  * `value`: whole-job NVFP4 TFLOP/s with inputs resident in HBM, timed with CUDA
    events on the launching stream over exactly K calls (barrier + synchronize on
    both sides, max over ranks). Inputs (232 MB for cfg2) exceed the 126 MB L2.
  * `e2e`: the same metric through the public API with host buffers: every step
    copies the operands from pinned host memory, calls custom_kernel and copies
    the fp16 outputs back (two buffer sets: a step's H2D overlaps the previous
    step's call and D2H; `e2e.serial` keeps everything on one stream).
  * `roofline`: the grouped-GEMM kernel against the dense FP4 tensor peak derived
    from MEASURED_PEAKS.json (4 x the measured cuBLAS bf16 figure: the sustained one for
    `value`, which is timed after a 1 s load window with the clocks sampled around it;
    `burst` reports the same calls timed right after warm-up against the burst figure).
  * `cpu_baseline`: the CPU oracle (numpy restatement of the reference's
    ref_kernel) on the full configuration, rank 0 at N=1 only.
  * `nvfp4_peak`: cuBLASLt's dense NVFP4 rate measured on the same GPU (8192^3);
    `roofline.frac_of_measured_nvfp4` divides by it.
  * `sharded_cfg5` (every N): cfg5's 256 experts split over the N ranks (strong
    scaling of one configuration), with and (N > 1) without the NCCL all-gather
    of all fp16 outputs to every rank.
  * `configs` + `geomean_us_per_call` (N = 1): BASELINE's headline form, us per
    isolated call of configs 1-5, their geomean and each one's roofline fraction.
  * `reference_kernel` (N = 1): the reference's own sm_100 CuTe-DSL kernel through its
    own custom_kernel (installed unmodified by baseline/install_reference.py) on the
    same inputs, timed beside this library's custom_kernel, outputs compared.
With N GPUs each rank runs its own set of experts of the same shape for `value` (weak
scaling; expert parallelism needs no collective on the data path).

Reference arm (--impl reference): the reference's CPU path (the oracle port of
ref_kernel) timed on the host cores; rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PEAK_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
L2_BYTES = 126 * 1000 * 1000
FP4_PER_BF16 = 4.0  # dense FP4 : dense BF16 tensor throughput on B200 (9 : 2.25 PFLOP/s)
NOMINAL_FP4_TFLOPS = 9000.0  # B200 dense FP4, nominal


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="cfg2")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "reference_gpu"])
    ap.add_argument("--tile-n", type=int, default=None)
    ap.add_argument("--cta", default=None, choices=[None, "pair", "single", "weights"])
    ap.add_argument("--split-k", action="store_true",
                    help="let single-CTA launches split the K loop of their last partial wave")
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-clocks", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the measured NVFP4 peak, the cfg5 expert split and the "
                         "configs 1-5 record")
    ap.add_argument("--op", default="gemm", choices=["gemm", "quantize", "moe"],
                    help="gemm: the grouped GEMM (default); quantize: the NVFP4 activation "
                         "quantiser on the configuration's A rows (bf16 [sum M_g, K]); moe: the "
                         "whole MoE block (route, quantise, gated GEMM, quantise, down GEMM, "
                         "combine) at cfg5's shape")
    ap.add_argument("--experts", default=None,
                    help="START:STOP - run only this contiguous expert shard of the configuration")
    ap.add_argument("--shard-experts", action="store_true",
                    help="N > 1: rank r runs expert_shard(G, N, r) of ONE configuration (strong "
                         "scaling; cfg5 = 256/N experts per GPU); default: every rank its own "
                         "full configuration (weak scaling)")
    ap.add_argument("--tokens", type=int, default=32768,
                    help="--op moe: tokens per step (32768 = cfg5's 262144 routed rows; 64 = a "
                         "decode step)")
    ap.add_argument("--ep", action="store_true",
                    help="--op moe on one GPU: the expert-parallel block as a single rank "
                         "(its exchange kernels included) instead of MoEBlock")
    ap.add_argument("--ep-return", default="both", choices=["sums", "rows", "both"],
                    help="--op moe over N > 1 GPUs: how expert outputs return to their tokens' "
                         "ranks (owner-side sums, per-pair rows, or both timed in turn)")
    return ap.parse_args()


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return d, "measured"
    return PEAK_FALLBACK, "fallback"


def load_traffic(kernel_tag: str, config: str):
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(path):
        return None
    with open(path) as f:
        d = json.load(f)
    e = d.get(f"{kernel_tag}:{config}")
    return None if e is None else e.get("dram_bytes_per_launch")


class ClockSampler:
    """nvidia-smi clock/throttle samples taken while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int, enabled: bool = True):
        self.gpu = gpu_index
        self.proc = None
        self.path = None
        if not enabled:
            return
        try:
            import torch

            # nvidia-smi numbers GPUs physically; the UUID names this process's device
            # whatever CUDA_VISIBLE_DEVICES maps it to.
            ident = str(gpu_index)
            uuid = getattr(torch.cuda.get_device_properties(gpu_index), "uuid", None)
            if uuid is not None:
                u = str(uuid)
                ident = u if u.startswith("GPU-") else f"GPU-{u}"
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={ident}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None, "reasons": reasons,
                "samples": len(rows)}


def _cpu_problem(cfg: str):
    """The configuration's inputs on the host (seed 0, as rank 0 of the GPU arm) as numpy
    arrays for the CPU oracle."""
    import submission

    pkg = submission.load_package()
    prob = pkg.workloads.make_config(cfg, seed=0, device="cpu")
    groups = [g for g in range(prob.num_groups) if prob.m[g] > 0]
    arrays = [(prob.a[g].numpy(), prob.b[g].numpy(), prob.sfa_plain[g].numpy(),
               prob.sfb_plain[g].numpy(), prob.b2[g].numpy() if prob.gated else None,
               prob.sfb2_plain[g].numpy() if prob.gated else None, prob.alpha[g],
               prob.alpha2[g] if prob.gated else 1.0) for g in groups]
    return prob, groups, arrays


def _cpu_step(cfg: str, prob, groups, arrays, budget_s: float) -> dict:
    """One bounded sample of the configuration through the CPU oracle (numpy restatement of
    ref_kernel): groups in order until all are done or `budget_s` has passed."""
    from oracle import nvfp4_oracle as O

    done_flops = 0.0
    t0 = time.perf_counter()
    calls = 0
    for (a, b, sfa, sfb, b2, sfb2, al, al2), g in zip(arrays, groups):
        if b2 is not None:
            O.ref_gated(a, b, b2, sfa, sfb, sfb2, al, al2)
        else:
            O.ref_gemm(a, b, sfa, sfb, al)
        done_flops += 2.0 * prob.m[g] * prob.n * prob.k * (2 if prob.gated else 1)
        calls += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    threads = os.cpu_count()
    return {"value": done_flops / dt / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{cfg}: {calls} of {prob.num_groups} groups through the numpy oracle "
                      f"(dequantise + fp32 BLAS matmul + fp16), {dt:.2f} s",
            "us_per_call_extrapolated": dt / max(done_flops, 1.0) * prob.flops() * 1e6}


def cpu_baseline(cfg: str, budget_s: float = 20.0) -> dict:
    """Time the CPU oracle (numpy restatement of ref_kernel) on the configuration."""
    prob, groups, arrays = _cpu_problem(cfg)
    return _cpu_step(cfg, prob, groups, arrays, budget_s)


def workload_config(args, prob, world: int, strong: bool) -> dict:
    """The `config` record of a line: the workload both arms run."""
    flush_l2 = prob.input_bytes() < L2_BYTES
    return {"workload": args.config + (f"[experts {args.experts}]" if args.experts else ""),
            "groups_per_gpu": prob.num_groups,
            "m_per_group": prob.m if len(prob.m) <= 16 else f"{sum(prob.m)} rows",
            "n": prob.n, "k": prob.k, "gated": prob.gated,
            "input_bytes_per_gpu": prob.input_bytes(),
            "l2": ("inputs smaller than L2 (126 MB): 256 MiB flush before every timed "
                   "call, outside its events" if flush_l2 else
                   "inputs larger than L2 (126 MB); no flush"),
            "parallelism": f"ep{world} (" + ("experts of one configuration split over "
                                              "the ranks" if strong else "every rank its own "
                                              "experts") + ", no data-path collective)",
            **({"split_k": True} if args.split_k else {})}


def run_reference(args):
    """The reference arm: the reference's arithmetic (ref_kernel, restated by the CPU oracle;
    the reference's own ref_kernel needs torch._scaled_mm on a GPU) on the host cores, on the
    GPU arm's workload, metric and step counts. Rank 0 alone runs it."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    prob, groups, arrays = _cpu_problem(args.config)
    # Each step is a bounded sample, so that the whole run stays within about two minutes.
    warmup = max(args.warmup, 3)
    budget = max(0.5, 100.0 / max(1, args.steps + warmup))
    for _ in range(warmup):
        _cpu_step(args.config, prob, groups, arrays, budget)
    res = [_cpu_step(args.config, prob, groups, arrays, budget) for _ in range(args.steps)]
    v = statistics.median(r["value"] for r in res)
    strong = args.shard_experts and world > 1 and not args.experts
    line = {
        "impl": "reference", "metric": f"NVFP4 grouped GEMM TFLOP/s ({args.config})",
        "value": v, "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": warmup, "higher_is_better": True,
        "scaling": "strong" if strong else "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded; e2m1 codes uniform over 16, E4M3 scales 2^U{-4..3})",
        "config": workload_config(args, prob, world, strong),
        "cpu_baseline": {**res[len(res) // 2], "value": v,
                         "sample": res[len(res) // 2]["sample"] +
                         f" per step; median of {args.steps} steps after {warmup} warm-up"},
        "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


HEADLINE_CONFIGS = ("cfg1", "cfg2", "cfg3", "cfg4", "cfg5")


def measure_nvfp4_peak(dev, seconds: float = 2.0) -> dict:
    """Dense block-scaled NVFP4 rate of the library GEMM on this GPU: torch._scaled_mm
    (cuBLASLt, E4M3 scales per 16 elements, fp16 out) at M = N = K = 8192, the shape of the
    bf16 figures in MEASURED_PEAKS.json. `burst`: best of 10 calls right after warm-up;
    `sustained`: calls back to back for `seconds`, the median rate of the second half's
    chunks of 20 calls."""
    import torch

    M = N = K = 8192
    g = torch.Generator(device=dev).manual_seed(5)
    # The reference generator's value set (codes {0, +-0.5, +-1, +-1.5}, scales {1, 2}).
    a = torch.randint(0, 256, (M, K // 2), dtype=torch.uint8, device=dev, generator=g) & 0xBB
    b = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, device=dev, generator=g) & 0xBB
    sf = lambda rows: (0x38 + 8 * torch.randint(0, 2, (rows * K // 16,), device=dev,
                                                generator=g, dtype=torch.int32)).to(torch.uint8)
    f4, e4 = torch.float4_e2m1fn_x2, torch.float8_e4m3fn
    a4, bt = a.view(f4), b.view(f4).t()
    sa, sb = sf(M).view(e4), sf(N).view(e4)
    flops = 2.0 * M * N * K

    def call():
        return torch._scaled_mm(a4, bt, sa, sb, out_dtype=torch.float16)

    for _ in range(3):
        call()
    torch.cuda.synchronize(dev)
    best = float("inf")
    for _ in range(10):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        call()
        e1.record()
        torch.cuda.synchronize(dev)
        best = min(best, e0.elapsed_time(e1))
    rates = []
    t_end = time.perf_counter() + seconds
    while time.perf_counter() < t_end:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(20):
            call()
        e1.record()
        torch.cuda.synchronize(dev)
        rates.append(20 * flops / (e0.elapsed_time(e1) * 1e-3) / 1e12)
    tail = rates[len(rates) // 2:] or rates
    return {"burst_tflops": flops / (best * 1e-3) / 1e12,
            "sustained_tflops": statistics.median(tail),
            "what": f"torch._scaled_mm NVFP4 (cuBLASLt block-scaled, fp16 out) {M}x{N}x{K}: "
                    f"best of 10 (burst); back to back for {seconds:.0f} s (sustained)"}


def headline_configs(pkg, dev, steps: int, warmup: int, peaks: dict, nvfp4_peak: dict | None,
                     sample_clocks: bool = True):
    """BASELINE's headline form: microseconds per call of configs 1-5 through the prepared
    launch (one GPU, device-resident inputs, a 256 MiB L2 flush before each call of a
    configuration whose inputs fit in L2; events around each call, median), their
    geometric mean, and each configuration's fraction of its roofline (burst peaks: every
    call is timed on its own)."""
    import math

    import torch

    tensor_peak = FP4_PER_BF16 * float(peaks["bf16_tflops"])
    hbm_peak = float(peaks["hbm_gbs"])
    fp4_peak = nvfp4_peak["burst_tflops"] if nvfp4_peak else None
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    per = {}
    clocks = ClockSampler(dev.index if dev.index is not None else 0, enabled=sample_clocks)
    for cfg in HEADLINE_CONFIGS:
        prob = pkg.workloads.make_config(cfg, seed=0, device=dev)
        plan = pkg.GroupedGemmPlan(prob.a, prob.b, prob.sfa, prob.sfb, prob.c,
                                   prob.problem_sizes(), alpha=prob.alpha, b2=prob.b2,
                                   sfb2=prob.sfb2, alpha2=prob.alpha2)
        for _ in range(max(warmup, 3)):
            plan.run()
        torch.cuda.synchronize(dev)
        small = prob.input_bytes() < L2_BYTES
        times = []
        for _ in range(steps):
            if small:
                flush.fill_(1)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            plan.run()
            e1.record()
            torch.cuda.synchronize(dev)
            times.append(e0.elapsed_time(e1) * 1e3)
        us = sorted(times)[len(times) // 2]
        flops, nbytes = prob.flops(), prob.algorithmic_bytes()
        tflops = flops / (us * 1e-6) / 1e12
        bound = "tensor" if flops / nbytes >= tensor_peak * 1e12 / (hbm_peak * 1e9) else "hbm"
        frac = tflops / tensor_peak if bound == "tensor" else nbytes / (us * 1e-6) / 1e9 / hbm_peak
        entry = {"us_per_call": us, "tflops": tflops, "gbs": nbytes / (us * 1e-6) / 1e9,
                 "bound": bound, "frac_of_roofline": frac,
                 "flops": flops, "algorithmic_bytes": nbytes,
                 "device_error_bits": plan.check_device_errors()}
        if bound == "tensor" and fp4_peak:
            entry["frac_of_measured_nvfp4_burst"] = tflops / fp4_peak
        per[cfg] = entry
        del plan, prob
        torch.cuda.empty_cache()
    geo = math.exp(sum(math.log(v["us_per_call"]) for v in per.values()) / len(per))
    return {"geomean_us_per_call": geo, "per_config": per, "clocks": clocks.stop(),
            "timing": "one call per event pair, median of --steps calls; a 256 MiB L2 flush "
                      "before each call of a configuration whose inputs fit in L2",
            "peaks": "tensor-bound: 4 x burst bf16 (MEASURED_PEAKS.json) and the measured "
                     "NVFP4 burst rate; hbm-bound: hbm_gbs"}


def run_all_configs(args):
    """`--config all`: the headline configurations alone, one JSON line."""
    import torch

    import submission

    pkg = submission.load_package()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    peaks, kind = load_peaks()
    rec = headline_configs(pkg, dev, args.steps, args.warmup, peaks, None, not args.no_clocks)
    print(json.dumps({
        "metric": "us/call (geomean of configs 1-5)", "value": rec["geomean_us_per_call"],
        "unit": "us", "n_gpus": 1, "steps": args.steps, "warmup": max(args.warmup, 3),
        "higher_is_better": False, "scaling": "weak", "vs_baseline": None,
        "dtype": "e2m1xe4m3->f32->f16", "data": "synthetic (seeded)",
        "config": {"workload": "cfg1..cfg5", "timing": rec["timing"]},
        "per_config": rec["per_config"], "peak_source": f"{kind}: burst bf16 x 4 / HBM copy",
    }), flush=True)


def sharded_cfg5(pkg, dev, world: int, rank: int, steps: int, warmup: int, barrier,
                 max_over_ranks, sum_over_ranks, tensor_peak: float, gather_group_ok: bool):
    """cfg5 (256 gated experts, 262144 routed rows) with its experts split over the ranks:
    rank r computes expert_shard(256, P, r) (strong scaling of the one configuration;
    P = 1 is the whole configuration on one GPU). Calls back to back, events around
    `steps` calls, max over ranks. With P > 1 the same calls followed by the NCCL
    all-gather of every expert's fp16 output to every rank (the GEMM writes into the
    gather's send slab; ExpertOutputGather)."""
    import torch
    import torch.distributed as dist

    EP = pkg.expert_parallel
    G = len(pkg.workloads.config_rows("cfg5")[0])
    sh = EP.expert_shard(G, world, rank)
    prob = pkg.workloads.make_config("cfg5", seed=0, device=dev, experts=slice(sh.start, sh.stop))
    all_m = prob.meta["all_m"]
    gat = None
    if world > 1 and gather_group_ok:
        gat = EP.ExpertOutputGather(all_m, prob.n, dev)
        prob.c = list(gat.local_outputs)
    plan = pkg.GroupedGemmPlan(prob.a, prob.b, prob.sfa, prob.sfb, prob.c, prob.problem_sizes(),
                               alpha=prob.alpha, b2=prob.b2, sfb2=prob.sfb2, alpha2=prob.alpha2)
    stream = torch.cuda.current_stream(dev)

    def timed(fn, n):
        for _ in range(max(warmup, 3)):
            fn()
        torch.cuda.synchronize(dev)
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(n):
            fn()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
        return max_over_ranks(e0.elapsed_time(e1) / n)

    n = max(3, min(steps, 20))
    ms = timed(lambda: plan.run(stream), n)
    flops_job = sum_over_ranks(prob.flops())
    tf = flops_job / (ms * 1e-3) / 1e12
    rec = {"us_per_call": ms * 1e3, "tflops": tf, "steps": n,
           "frac_of_per_gpu_peak": tf / (world * tensor_peak),
           "experts_per_rank": len(sh), "rows_this_rank": int(sum(prob.m)),
           "flops_total": flops_job, "scaling": "strong",
           "device_error_bits": plan.check_device_errors(stream),
           "what": "GroupedGemmPlan.run of this rank's expert shard, back to back, max over "
                   "ranks; frac against P x 4 x sustained bf16"}
    if gat is not None:
        def both():
            plan.run(stream)
            gat.run()

        gms = timed(both, n)
        rec["with_gather"] = {
            "us_per_call": gms * 1e3, "tflops": flops_job / (gms * 1e-3) / 1e12,
            "bytes_received_per_rank": gat.bytes_received,
            "what": "the same calls, each followed by one NCCL all_gather_into_tensor of the "
                    "fp16 output slabs (every expert's output on every rank)"}
        # The same exchange fused into the GEMM: its epilogue stores every output tile into
        # each peer's copy of the output slabs over NVLink (nvfp4_grouped_gemm_replicated);
        # a one-element all-reduce per call orders the ranks.
        del plan
        # Every rank must agree before the collective timing below: a rank that could not
        # set up the symmetric-memory gather makes all of them skip it.
        try:
            fused = EP.FusedOutputGather(all_m, prob.n, dev)
            fused_err = None
        except Exception as exc:  # reported in the line, not fatal to the bench
            fused, fused_err = None, f"{type(exc).__name__}: {exc}"[:200]
        agree = torch.tensor([0 if fused is None else 1], dtype=torch.int32, device=dev)
        dist.all_reduce(agree, op=dist.ReduceOp.MIN)
        if int(agree.item()) == 0:
            rec["fused_gather"] = {"unavailable": fused_err or "set-up failed on another rank"}
            del fused
            plan = gat = None
            del plan, gat, prob
            torch.cuda.empty_cache()
            return rec

        def fused_call():
            fused.gemm(prob.a, prob.b, prob.sfa, prob.sfb, prob.problem_sizes(),
                       alpha=prob.alpha, b2=prob.b2, sfb2=prob.sfb2, alpha2=prob.alpha2,
                       stream=stream)
            fused.barrier()

        fms = timed(fused_call, n)
        rec["fused_gather"] = {
            "us_per_call": fms * 1e3, "tflops": flops_job / (fms * 1e-3) / 1e12,
            "bytes_sent_per_rank": fused.bytes_sent,
            "device_error_bits": fused.check_device_errors(stream),
            "equal_to_nccl_gather": all(
                torch.equal(x.view(torch.int16), y.view(torch.int16))
                for x, y in zip(fused.outputs, gat.outputs)),
            "what": "one kernel per call: the grouped GEMM whose epilogue also stores every "
                    "output tile into every other rank's copy of the output slabs over NVLink "
                    "(every expert's output on every rank), then a one-element NCCL "
                    "all-reduce as the cross-rank barrier"}
        del fused
        plan = gat = None
    del plan, gat, prob
    torch.cuda.empty_cache()
    return rec


REFERENCE_MODULE = os.path.join(ROOT, "baseline", "_ref", "submission.py")


def load_reference_module():
    """The reference's own kernel module (its submission.py, installed unmodified into
    baseline/_ref by baseline/install_reference.py), imported under another name so that
    it does not shadow this repository's submission.py. None if it is not installed."""
    import importlib.util

    if not os.path.exists(REFERENCE_MODULE):
        return None
    ref_dir = os.path.dirname(REFERENCE_MODULE)
    if ref_dir not in sys.path:
        sys.path.insert(0, ref_dir)  # its `from task import input_t, output_t`
    spec = importlib.util.spec_from_file_location("nvfp4_reference_submission", REFERENCE_MODULE)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def reference_kernel_leg(pkg, dev, cfg: str, steps: int, warmup: int, ref=None) -> dict:
    """The reference's own sm_100 kernel (CuTe DSL, submission.py:80-589) through its own
    custom_kernel (submission.py:788-858, the 4-tuple grouped path) against this
    library's custom_kernel, on the same device-resident inputs of configuration `cfg`
    (global scale 1: the reference has none). Its JIT compile (the first call) is timed
    apart and excluded. Both are timed the same two ways: one call per event pair (median;
    a 256 MiB L2 flush before each call when the inputs fit in L2) and `steps` calls back
    to back between one event pair. Outputs: the reference's and ours compared bit for bit,
    and both against the CPU oracle on up to two groups (rtol = atol = 1e-2)."""
    import numpy as np
    import torch

    from oracle import nvfp4_oracle as O

    if ref is None:
        ref = load_reference_module()
    if ref is None:
        return {"unavailable": "baseline/_ref/submission.py not installed "
                               "(python baseline/install_reference.py REFERENCE_DIR)"}
    prob = pkg.workloads.make_config(cfg, seed=0, device=dev)
    if prob.gated:
        return {"unavailable": f"{cfg} is gated: the reference's grouped path has no gated form"}
    prob.alpha = [1.0] * prob.num_groups
    data = prob.reference_data()
    data = (data[0], data[1], data[2], [tuple(ps) for ps in data[3]])
    stream = torch.cuda.current_stream(dev)
    t0 = time.perf_counter()
    ref.custom_kernel(data)
    torch.cuda.synchronize(dev)
    compile_s = time.perf_counter() - t0
    ref_out = [c.clone() for c in prob.c]
    for c in prob.c:
        c.fill_(float("nan"))
    pkg.custom_kernel(data)
    torch.cuda.synchronize(dev)
    ours_out = [c.clone() for c in prob.c]
    equal = sum(int(torch.equal(x.view(torch.int16), y.view(torch.int16)))
                for x, y in zip(ref_out, ours_out))
    oracle = {}
    for g in [g for g in range(prob.num_groups) if prob.m[g] > 0][:2]:
        a, b = prob.a[g].cpu().numpy(), prob.b[g].cpu().numpy()
        ref32 = O.ref_gemm_fp32(a, b, prob.sfa_plain[g].cpu().numpy(), prob.sfb_plain[g].cpu().numpy())
        with np.errstate(over="ignore"):
            exp = ref32.astype(np.float16)
        r_ref = O.compare_fp16(ref_out[g].cpu().numpy(), exp, ref32, rtol=1e-2, atol=1e-2)
        r_ours = O.compare_fp16(ours_out[g].cpu().numpy(), exp, ref32, rtol=1e-2, atol=1e-2)
        oracle[f"group{g}"] = {"reference_ok": bool(r_ref["ok"]), "ours_ok": bool(r_ours["ok"]),
                               "reference_mismatches": int(r_ref.get("mismatches", 0)),
                               "ours_mismatches": int(r_ours.get("mismatches", 0))}
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    small = prob.input_bytes() < L2_BYTES

    def isolated(fn):
        for _ in range(max(warmup, 3)):
            fn()
        torch.cuda.synchronize(dev)
        times = []
        for _ in range(steps):
            if small:
                flush.fill_(1)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn()
            e1.record(stream)
            torch.cuda.synchronize(dev)
            times.append(e0.elapsed_time(e1) * 1e3)
        return sorted(times)[len(times) // 2]

    def back_to_back(fn):
        torch.cuda.synchronize(dev)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) * 1e3 / steps

    run_ref = lambda: ref.custom_kernel(data)
    run_ours = lambda: pkg.custom_kernel(data)
    rec = {"config": cfg, "compile_s": compile_s,
           "reference_us_isolated": isolated(run_ref), "ours_us_isolated": isolated(run_ours),
           "reference_us_back_to_back": back_to_back(run_ref),
           "ours_us_back_to_back": back_to_back(run_ours),
           "groups_bit_identical": f"{equal}/{prob.num_groups}", "oracle": oracle,
           "flops": prob.flops(), "algorithmic_bytes": prob.algorithmic_bytes(),
           "what": "the reference's custom_kernel (its CuTe-DSL sm_100 kernel, unmodified) vs "
                   "this library's custom_kernel on the same inputs; times are device time per "
                   "call including each API's own per-call host work"}
    rec["speedup_isolated"] = rec["reference_us_isolated"] / rec["ours_us_isolated"]
    rec["speedup_back_to_back"] = rec["reference_us_back_to_back"] / rec["ours_us_back_to_back"]
    del prob, data, flush
    torch.cuda.empty_cache()
    return rec


def run_reference_gpu(args):
    """`--impl reference_gpu`: the reference's own GPU kernel against ours, one JSON line
    with one record per configuration of `--config` (comma separated; 1 GPU, rank 0)."""
    import torch

    import submission

    if int(os.environ.get("RANK", "0")) != 0:
        return
    pkg = submission.load_package()
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    t0 = time.perf_counter()
    ref = load_reference_module()
    import_s = time.perf_counter() - t0
    recs = [reference_kernel_leg(pkg, dev, c, args.steps, args.warmup, ref)
            for c in args.config.split(",")]
    print(json.dumps({"impl": "reference_gpu", "metric": "us/call, reference kernel vs ours",
                      "unit": "us", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
                      "higher_is_better": False, "import_s": import_s, "records": recs}),
          flush=True)


def run_quantize(args):
    """The activation quantiser over the configuration's A rows, one JSON line (rank 0)."""
    import numpy as np
    import torch

    import submission

    pkg = submission.load_package()
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    if args.impl == "reference":
        from oracle import nvfp4_quant_oracle as Q
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    ms, n, k, gated, _ = pkg.workloads.config_rows(args.config, seed=0)
    rows = int(sum(ms))
    g = torch.Generator(device="cpu").manual_seed(0)
    xh = (torch.randn((rows, k), generator=g) * 2.0).to(torch.bfloat16)
    alg = rows * k * 2 + rows * k // 2 + pkg.blocked_sf_bytes(rows, k // 16)
    sg = float(xh.abs().amax().float()) / (6 * 448)
    line = {"metric": f"NVFP4 quantiser GB/s ({args.config} A rows, bf16 [{rows}, {k}])",
            "unit": "GB/s", "n_gpus": 1, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16->e2m1+e4m3", "data": "synthetic (seeded N(0, 4))",
            "config": {"workload": f"quantize:{args.config}", "rows": rows, "cols": k}}
    if args.impl == "reference":
        sample = max(1, min(rows, (1 << 22) // k))
        xs = xh[:sample].float().numpy()
        t0 = time.perf_counter()
        Q.quantize_nvfp4_blocked(xs, sg)
        dt = time.perf_counter() - t0
        v = sample * (k * 2 + k // 2 + k // 16) / dt / 1e9
        line.update({"impl": "reference", "value": v, "steps": 1, "warmup": 0,
                     "cpu_baseline": {"value": v, "unit": "GB/s", "cores": 1, "kind": "port",
                                      "sample": f"{sample} rows through the numpy oracle, {dt:.2f} s"},
                     "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0,
                             "d2h_bytes_per_step": 0}})
        print(json.dumps(line), flush=True)
        return
    x = xh.to(dev)
    packed = torch.empty((rows, k // 2), dtype=torch.uint8, device=dev)
    sf = torch.empty(pkg.blocked_sf_bytes(rows, k // 16), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev) if rows * k * 2 < L2_BYTES else None

    def timed(n_steps):
        pairs = []
        for _ in range(n_steps):
            if flush is not None:
                flush.fill_(1)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            pkg.quantize(x, sg, packed=packed, sf=sf, stream=stream)
            e1.record(stream)
            pairs.append((e0, e1))
        torch.cuda.synchronize(dev)
        return sum(a.elapsed_time(b) for a, b in pairs) / n_steps

    for _ in range(max(args.warmup, 3)):
        pkg.quantize(x, sg, packed=packed, sf=sf, stream=stream)
    ms_step = timed(args.steps)
    # End to end: bf16 rows from pinned host memory, quantise, codes and scales back.
    xp = xh.pin_memory()
    hp = torch.empty(packed.shape, dtype=torch.uint8).pin_memory()
    hs = torch.empty(sf.shape, dtype=torch.uint8).pin_memory()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    e0.record(stream)
    for _ in range(3):
        x.copy_(xp, non_blocking=True)
        pkg.quantize(x, sg, packed=packed, sf=sf, stream=stream)
        hp.copy_(packed, non_blocking=True)
        hs.copy_(sf, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = e0.elapsed_time(e1) / 3
    peaks, kind = load_peaks()
    gbs = alg / (ms_step * 1e-3) / 1e9
    sample = max(1, min(rows, (1 << 21) // k))
    from oracle import nvfp4_quant_oracle as Q
    xs = xh[:sample].float().numpy()
    t0 = time.perf_counter()
    Q.quantize_nvfp4_blocked(xs, sg)
    dt = time.perf_counter() - t0
    line.update({
        "value": gbs, "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": ms_step,
        "us_per_call": ms_step * 1e3, "gpu_launches": args.steps,
        "config": dict(line["config"], l2=("inputs smaller than L2: 256 MiB flush before every "
                                           "timed call" if flush is not None else
                                           "inputs larger than L2 (126 MB); no flush")),
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": float(peaks["hbm_gbs"]),
                     "unit": "GB/s", "frac": gbs / float(peaks["hbm_gbs"]),
                     "peak_source": f"{kind}: hbm_gbs", "traffic": None,
                     "algorithmic_bytes": alg},
        "e2e": {"value": alg / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": int(xp.numel() * 2),
                "d2h_bytes_per_step": int(hp.numel() + hs.numel())},
        "cpu_baseline": {"value": sample * (k * 2 + k // 2 + k // 16) / dt / 1e9, "unit": "GB/s",
                         "cores": 1, "kind": "port",
                         "sample": f"{sample} rows through the numpy oracle, {dt:.2f} s"},
    })
    print(json.dumps(line), flush=True)


def pcie_bandwidth(dev, s_h2d, s_d2h, nbytes: int = 256 << 20) -> dict:
    """Host<->device copy rates of pinned memory on this GPU (GB/s, best of 5): each
    direction alone, then both at once on the two streams."""
    import torch

    host_a = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    host_b = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    dev_a = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    dev_b = torch.empty(nbytes, dtype=torch.uint8, device=dev)

    def rate(fn, stream):
        best = 0.0
        for _ in range(5):
            torch.cuda.synchronize(dev)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn()
            e1.record(stream)
            torch.cuda.synchronize(dev)
            best = max(best, nbytes / (e0.elapsed_time(e1) * 1e-3) / 1e9)
        return best

    def h2d():
        with torch.cuda.stream(s_h2d):
            dev_a.copy_(host_a, non_blocking=True)

    def d2h():
        with torch.cuda.stream(s_d2h):
            host_b.copy_(dev_b, non_blocking=True)

    out = {"h2d_gbs": rate(h2d, s_h2d), "d2h_gbs": rate(d2h, s_d2h)}
    both_h2d, both_d2h = 0.0, 0.0
    for _ in range(5):
        torch.cuda.synchronize(dev)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        ev[0].record(s_h2d)
        ev[2].record(s_d2h)
        h2d()
        d2h()
        ev[1].record(s_h2d)
        ev[3].record(s_d2h)
        torch.cuda.synchronize(dev)
        both_h2d = max(both_h2d, nbytes / (ev[0].elapsed_time(ev[1]) * 1e-3) / 1e9)
        both_d2h = max(both_d2h, nbytes / (ev[2].elapsed_time(ev[3]) * 1e-3) / 1e9)
    out["h2d_concurrent_gbs"] = both_h2d
    out["d2h_concurrent_gbs"] = both_d2h
    return out


def ep_block_inputs(pkg, dev, world: int, rank: int, tokens: int):
    """Seeded inputs of the expert-parallel MoE block at cfg5's shape (256 experts, top-8,
    H 7168, I 2048) for `rank` of `world`: this rank's NVFP4 expert weights (random codes,
    scales 2^-1 / 2^0), tokens // world bf16 tokens and their uniform top-8 routing."""
    import torch

    E, topk, H, I = 256, 8, 7168, 2048
    T = tokens // world
    epr = E // world
    g = torch.Generator(device=dev).manual_seed(1000 + rank)

    def nvfp4_weights(rows, cols):
        codes = torch.randint(0, 256, (rows, cols // 2), generator=g, device=dev,
                              dtype=torch.int32).to(torch.uint8) & 0xBB
        sf_plain = torch.where(torch.rand((rows, cols // 16), generator=g, device=dev) < 0.5,
                               torch.tensor(0x38, dtype=torch.uint8, device=dev),
                               torch.tensor(0x40, dtype=torch.uint8, device=dev))
        return codes, pkg.plain_to_blocked(sf_plain)

    W = {k: [] for k in ("w_gate", "sf_gate", "w_up", "sf_up", "w_down", "sf_down")}
    for _ in range(epr):
        for name, (r, c) in (("gate", (I, H)), ("up", (I, H)), ("down", (H, I))):
            q, sf = nvfp4_weights(r, c)
            W[f"w_{name}"].append(q)
            W[f"sf_{name}"].append(sf)
    weights = pkg.moe.ExpertWeights(**W, s_gate=[2.0 ** -6] * epr, s_up=[2.0 ** -6] * epr,
                                    s_down=[2.0 ** -6] * epr)
    x = torch.randn((T, H), generator=g, device=dev).to(torch.bfloat16)
    scores = torch.rand((T, E), generator=g, device=dev)
    top = torch.topk(scores, topk, dim=1)
    ids = top.indices.to(torch.int32)
    wts = torch.softmax(top.values, dim=1)
    s_x = pkg.global_scale_for(x)
    s_h = 0.01  # fixed SiLU-output scale (values do not change the timing)
    return dict(E=E, topk=topk, H=H, I=I, T=T, epr=epr, weights=weights, x=x, ids=ids, wts=wts,
                s_x=s_x, s_h=s_h)


def ep_block_leg(pkg, dev, world: int, rank: int, steps: int, warmup: int, barrier,
                 max_over_ranks, sum_over_ranks, tokens: int = 32768) -> dict:
    """The expert-parallel MoE block (EPMoEBlock, owner-side sums) at cfg5's shape with the
    tokens and the experts split over the ranks: strong scaling of one batch. At P = 1 the
    same block runs as one rank (SingleDeviceFabric), so every N times the same code path.
    Calls back to back, events around `steps` calls, max over ranks."""
    import torch
    import torch.distributed as dist

    EP = pkg.expert_parallel
    # Every rank must set up before the timed collectives: a rank that could not makes all
    # of them skip the leg.
    try:
        inp = ep_block_inputs(pkg, dev, world, rank, tokens)
        fabric = EP.SingleDeviceFabric(1, dev).rank_view(0) if world == 1 else None
        blk = EP.EPMoEBlock(inp["weights"], inp["E"], inp["T"], inp["topk"], inp["s_x"],
                            inp["s_h"], fabric=fabric)
        err = None
    except Exception as exc:  # reported in the line, not fatal to the bench
        blk, err = None, f"{type(exc).__name__}: {exc}"[:200]
    if world > 1:
        agree = torch.tensor([0 if blk is None else 1], dtype=torch.int32, device=dev)
        dist.all_reduce(agree, op=dist.ReduceOp.MIN)
        ok = int(agree.item()) == 1
    else:
        ok = blk is not None
    if not ok:
        return {"unavailable": err or "set-up failed on another rank"}
    x, ids, wts = inp["x"], inp["ids"], inp["wts"]
    stream = torch.cuda.current_stream(dev)
    for _ in range(max(warmup, 3)):
        blk.run(x, ids, wts)
    torch.cuda.synchronize(dev)
    barrier()
    n = max(3, min(steps, 10))
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(n):
        blk.run(x, ids, wts)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1) / n)
    evs = []
    blk.run(x, ids, wts, stage_events=evs)
    torch.cuda.synchronize(dev)
    stage_us = {nm: a.elapsed_time(b) * 1e3 for (_, a), (nm, b) in zip(evs[:-1], evs[1:])}
    pairs = sum_over_ranks(float((ids >= 0).sum().item()))
    flops = 6.0 * pairs * inp["H"] * inp["I"]
    rec = {"us_per_call": ms * 1e3, "tflops": flops / (ms * 1e-3) / 1e12, "steps": n,
           "tokens_per_rank": inp["T"], "experts_per_rank": inp["epr"], "flops_total": flops,
           "scaling": "strong", "return_mode": blk.return_mode,
           "stage_us_rank0": stage_us, "exchange_error_bits": blk.check_errors(),
           "what": "expert_parallel.EPMoEBlock.run (route, quantise, NVFP4 token rows to their "
                   "experts' owners over NVLink peer stores, gated GEMM with NVFP4 output, down "
                   "GEMM, weighted owner-side sums returned to the tokens' ranks, combine; 3 "
                   "one-element NCCL barriers per call) of 32768 tokens x top-8 over 256 experts "
                   "split over the ranks, back to back, max over ranks; one GPU: the same block "
                   "as a single rank"}
    barrier()
    del blk, inp
    torch.cuda.empty_cache()
    return rec


def run_moe_ep(args, world):
    """The expert-parallel MoE block (EPMoEBlock) at cfg5's shape over `world` GPUs: the
    32768 tokens split evenly over the ranks, the 256 experts too (strong scaling of one
    batch); routed rows cross NVLink in NVFP4 and results come back to their tokens' rank."""
    import datetime

    import torch
    import torch.distributed as dist

    import submission

    pkg = submission.load_package()
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    multi = world > 1
    if multi:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))

    def barrier():
        if multi:
            barrier()

    def all_reduce(t, op=None):
        if multi:
            dist.all_reduce(t, op=op if op is not None else dist.ReduceOp.SUM)

    inp = ep_block_inputs(pkg, dev, world, rank, args.tokens)
    E, topk, H, I, T, epr = (inp[k] for k in ("E", "topk", "H", "I", "T", "epr"))
    weights, x, ids, wts, s_x, s_h = (inp[k] for k in ("weights", "x", "ids", "wts", "s_x", "s_h"))
    steps = max(1, min(args.steps, 10))
    pairs = torch.tensor([int((ids >= 0).sum().item())], dtype=torch.float64, device=dev)
    all_reduce(pairs)
    flops = 6.0 * float(pairs.item()) * H * I

    def measure(mode):
        """Eager, per-stage and CUDA-graph timings of one EPMoEBlock in `mode` (max over
        ranks), its output on this rank, and its exchange error bits."""
        # One GPU: the same block as a single rank (SingleDeviceFabric, no process group).
        fabric = None if multi else pkg.expert_parallel.SingleDeviceFabric(1, dev).rank_view(0)
        blk = pkg.expert_parallel.EPMoEBlock(weights, E, T, topk, s_x, s_h, return_mode=mode,
                                             fabric=fabric)
        for _ in range(max(args.warmup, 3)):
            blk.run(x, ids, wts)
        torch.cuda.synchronize(dev)
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            blk.run(x, ids, wts)
        e1.record()
        torch.cuda.synchronize(dev)
        t = torch.tensor([e0.elapsed_time(e1) / steps], dtype=torch.float64, device=dev)
        all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        # One instrumented call: device time between the stages (this rank).
        evs = []
        blk.run(x, ids, wts, stage_events=evs)
        torch.cuda.synchronize(dev)
        stage_us = {n: a.elapsed_time(b) * 1e3 for (_, a), (n, b) in zip(evs[:-1], evs[1:])}
        out = blk.out.clone()
        # The same call captured in a CUDA graph (NCCL barriers included) and replayed.
        graph = blk.capture(x, ids, wts)
        graph.replay()
        torch.cuda.synchronize(dev)
        barrier()
        e0.record()
        for _ in range(steps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize(dev)
        t = torch.tensor([e0.elapsed_time(e1) / steps], dtype=torch.float64, device=dev)
        all_reduce(t, op=dist.ReduceOp.MAX)
        graph_ms = float(t.item())
        del graph
        err = blk.check_errors()
        barrier()
        del blk
        torch.cuda.empty_cache()
        return {"return_mode": mode, "ms_per_step": ms, "us_per_call": ms * 1e3,
                "value": flops / (ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                "stage_us_rank0": stage_us, "exchange_error_bits": err,
                "cuda_graph": {"ms_per_step": graph_ms,
                               "value": flops / (graph_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                               "what": "EPMoEBlock.capture, one call per replay, max over ranks"}}, out

    modes = ["sums", "rows"] if args.ep_return == "both" else [args.ep_return]
    runs, outs = [], []
    for mode in modes:
        r, o = measure(mode)
        runs.append(r)
        outs.append(o)
    if len(outs) == 2:  # the two return forms differ only by the fp16 rounding of the sums
        d = (outs[0].float() - outs[1].float()).norm() / outs[1].float().norm()
        runs[1]["rel_diff_vs_sums"] = float(d.item())
    main_run = runs[0]
    ms, graph_ms, err = main_run["ms_per_step"], main_run["cuda_graph"]["ms_per_step"], \
        main_run["exchange_error_bits"]
    stage_us = main_run["stage_us_rank0"]
    tf = flops / (ms * 1e-3) / 1e12
    peaks, kind = load_peaks()
    peak = world * FP4_PER_BF16 * float(peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"]))
    barrier()
    if multi:
        dist.destroy_process_group()
    if rank != 0:
        return
    print(json.dumps({
        "metric": f"NVFP4 expert-parallel MoE block TFLOP/s (cfg5 shape: 256 experts, {args.tokens} "
                  "tokens x top-8, H 7168, I 2048)",
        "value": tf, "unit": "TFLOP/s", "n_gpus": world, "steps": steps,
        "warmup": max(args.warmup, 3), "ms_per_step": ms, "us_per_call": ms * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "e2m1xe4m3->f32->f16/bf16",
        "data": "synthetic (seeded; bf16 N(0,1) tokens, uniform top-8 routing, reference-set weights)",
        "config": {"workload": "moe-ep:cfg5", "experts": E, "tokens": args.tokens,
                   "tokens_per_rank": T, "experts_per_rank": epr, "topk": topk, "hidden": H,
                   "intermediate": I, "return_mode": main_run["return_mode"],
                   "parallelism": f"ep{world} (NVFP4 rows over NVLink peer stores; "
                   + ("each token's rows summed on each owner, one fp16 row per (token, owner) "
                      "stored back to the token's rank" if main_run["return_mode"] == "sums" else
                      "expert output rows stored back to their tokens' ranks by the down "
                      "GEMM's epilogue") + "; 3 NCCL one-element barriers per call)"},
        "api": "expert_parallel.EPMoEBlock.run",
        "gpu_launches_per_call": "route 3, quantise 1, publish 1, layout 1, dispatch 1, "
                                 + ("publish pairs 1, " if main_run["return_mode"] == "sums" else "")
                                 + "scale layout 1, segment set-up + GEMM x2, "
                                 + ("return sums 1, " if main_run["return_mode"] == "sums" else "")
                                 + "combine 1 (+3 NCCL)",
        "exchange_error_bits": err,
        "stage_us_rank0": stage_us,
        "other_return_modes": runs[1:],
        "cuda_graph": {"ms_per_step": graph_ms, "value": flops / (graph_ms * 1e-3) / 1e12,
                       "unit": "TFLOP/s", "what": "EPMoEBlock.capture, one call per replay, max "
                                                  "over ranks"},
        "roofline": {"bound": "tensor", "achieved": tf, "peak": peak, "unit": "TFLOP/s",
                     "frac": tf / peak, "peak_source": f"{kind}: {world} x 4 x bf16 (sustained)",
                     "traffic": None},
    }), flush=True)


def run_moe(args):
    """The MoE feed-forward block at cfg5's shape (256 experts, 32768 tokens x top-8,
    H = 7168, I = 2048), one JSON line (rank 0). With more than one rank: the
    expert-parallel block (run_moe_ep)."""
    import numpy as np
    import torch

    import submission

    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1 or args.ep:
        return run_moe_ep(args, world)

    pkg = submission.load_package()
    rank = int(os.environ.get("RANK", "0"))
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    E, T, topk, H, I = 256, args.tokens, 8, 7168, 2048
    g = torch.Generator(device=dev).manual_seed(rank)

    def nvfp4_weights(rows, cols):
        # e2m1 codes of {0, +-0.5, +-1, +-1.5} and scales {1, 2}: the reference generator's
        # value set (REFERENCE_IMPL.md:148-150, 190-195), whose products stay in fp16 range.
        codes = torch.randint(0, 256, (rows, cols // 2), generator=g, device=dev,
                              dtype=torch.int32).to(torch.uint8) & 0xBB
        sf_plain = torch.where(torch.rand((rows, cols // 16), generator=g, device=dev) < 0.5,
                               torch.tensor(0x38, dtype=torch.uint8, device=dev),
                               torch.tensor(0x40, dtype=torch.uint8, device=dev))
        return codes, pkg.plain_to_blocked(sf_plain)

    W = {k: [] for k in ("w_gate", "sf_gate", "w_up", "sf_up", "w_down", "sf_down")}
    for _ in range(E):
        for name, (r, c) in (("gate", (I, H)), ("up", (I, H)), ("down", (H, I))):
            q, sf = nvfp4_weights(r, c)
            W[f"w_{name}"].append(q)
            W[f"sf_{name}"].append(sf)
    # Per-expert global scales chosen so that the gate/up and down outputs stay well inside
    # fp16 (sums of 7168 products of unit-scale values).
    weights = pkg.moe.ExpertWeights(**W, s_gate=[2.0 ** -6] * E, s_up=[2.0 ** -6] * E,
                                    s_down=[2.0 ** -6] * E)
    x = torch.randn((T, H), generator=g, device=dev).to(torch.bfloat16)
    scores = torch.rand((T, E), generator=g, device=dev)
    top = torch.topk(scores, topk, dim=1)
    ids = top.indices.to(torch.int32)
    wts = torch.softmax(top.values, dim=1)
    s_x = pkg.global_scale_for(x)
    # Scale of the SiLU output: measured once from the data, then fixed (as a deployment
    # would calibrate it), so the timed calls make only the routing step's host read.
    r = pkg.moe.route(ids, E)
    a, sfa = pkg.moe.quantize_rows(x, r.rows, r.src_rows, pkg._native.ROWS_GATHER, s_x)
    h = torch.zeros((r.rows, I), dtype=torch.float16, device=dev)
    av, sfav, hv, m = pkg.moe.expert_views(r, a, sfa, h, H)
    pkg.grouped_gemm(av, weights.w_gate, sfav, weights.sf_gate, hv, [(mi, I, H) for mi in m],
                     alpha=[s_x * v for v in weights.s_gate], b2=weights.w_up,
                     sfb2=weights.sf_up, alpha2=[s_x * v for v in weights.s_up])
    s_h = pkg.global_scale_for(h)

    def step():
        return pkg.moe.moe_ffn(x, ids, wts, weights, act_scale=s_x, hidden_scale=s_h)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize(dev)
    steps = max(1, min(args.steps, 10))
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        out = step()
    e1.record()
    torch.cuda.synchronize(dev)
    ms_eager = e0.elapsed_time(e1) / steps
    # The same block with no host read (MoEBlock: routing metadata stays on the GPU, both
    # expert GEMMs are segment launches), captured once in a CUDA graph and replayed: the
    # headline number. Its output is checked against moe_ffn's.
    blk = pkg.moe.MoEBlock(weights, T, topk, act_scale=s_x, hidden_scale=s_h)
    graph = blk.capture(x, ids, wts, warmup=max(args.warmup, 3))
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize(dev)
    same = bool(torch.equal(blk.out.view(torch.int16), out.view(torch.int16)))
    e0.record()
    for _ in range(steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / steps
    # Device time between the stages of one eager MoEBlock call.
    evs = []
    blk.run(x, ids, wts, stage_events=evs)
    torch.cuda.synchronize(dev)
    block_stage_us = {n: a.elapsed_time(b) * 1e3 for (_, a), (n, b) in zip(evs[:-1], evs[1:])}
    blk_errors = blk.check_device_errors()
    del graph
    # Per-stage split of one call (events between the stages of moe_ffn).
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(8)]
    ev[0].record()
    r = pkg.moe.route(ids, E)
    ev[1].record()
    qx, sfx = pkg.quantize(x, s_x)
    ev[2].record()
    a, sfa = pkg.moe.gather_quantized(qx, sfx, r)
    ev[3].record()
    h = torch.empty((r.rows, I), dtype=torch.float16, device=dev)
    P = weights.pointers()
    t1 = pkg.moe.dispatched_table(r, a, sfa, h, P["w_gate"], P["sf_gate"], I, H,
                                  s_x * np.asarray(weights.s_gate, dtype=np.float32),
                                  P["w_up"], P["sf_up"],
                                  s_x * np.asarray(weights.s_up, dtype=np.float32))
    pkg.interface.grouped_gemm_table(t1, pkg._native.FLAG_GATED, dev)
    ev[4].record()
    a2, sfa2 = pkg.moe.quantize_rows(h, r.rows, r.src_rows, pkg._native.ROWS_MASK, s_h)
    ev[5].record()
    y = torch.empty((r.rows, H), dtype=torch.float16, device=dev)
    t2 = pkg.moe.dispatched_table(r, a2, sfa2, y, P["w_down"], P["sf_down"], H, I,
                                  s_h * np.asarray(weights.s_down, dtype=np.float32))
    pkg.interface.grouped_gemm_table(t2, 0, dev)
    ev[6].record()
    pkg.moe.combine(y, r, wts)
    ev[7].record()
    torch.cuda.synchronize(dev)
    names = ["route (incl. host read)", "quantise x (once per token)", "dispatch (gather codes + scales)",
             "gate/up GEMM + SiLU", "quantise h", "down GEMM", "combine"]
    split = {n: ev[i].elapsed_time(ev[i + 1]) * 1e3 for i, n in enumerate(names)}
    rows = int(sum(r.counts))
    flops = 6.0 * rows * H * I
    tf_eager = flops / (ms_eager * 1e-3) / 1e12
    peaks, kind = load_peaks()
    peak = FP4_PER_BF16 * float(peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"]))
    tf = flops / (ms * 1e-3) / 1e12
    if rank != 0:
        return
    print(json.dumps({
        "metric": f"NVFP4 MoE block TFLOP/s (cfg5 shape: 256 experts, {T} tokens x top-8, H 7168, I 2048)",
        "value": tf, "unit": "TFLOP/s", "n_gpus": 1, "steps": steps, "warmup": max(args.warmup, 3),
        "ms_per_step": ms, "us_per_call": ms * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "e2m1xe4m3->f32->f16/bf16",
        "data": "synthetic (seeded; bf16 N(0,1) tokens, uniform top-8 routing, reference-set weights)",
        "config": {"workload": "moe:cfg5" if T == 32768 else f"moe:cfg5-experts:{T}-tokens",
                   "experts": E, "tokens": T, "topk": topk, "hidden": H,
                   "intermediate": I, "dispatched_rows": r.rows,
                   "l2": "inputs larger than L2 (126 MB); no flush"},
        "api": "MoEBlock captured in a CUDA graph, graph.replay() (value); moe_ffn (eager)",
        "gpu_launches_per_call": "route 3, quantise 1, gather 2, segment set-up 1 + gate/up GEMM 1, quantise 1, segment set-up 1 + down GEMM 1, combine 1",
        "eager_moe_ffn": {"us_per_call": ms_eager * 1e3, "tflops": tf_eager,
                          "note": "host-sized groups: one device->host read of the routing per call"},
        "graph_output_equals_moe_ffn": same,
        "device_error_bits": blk_errors,
        "stage_us": block_stage_us,
        "stage_us_moe_ffn": split,
        "roofline": {"bound": "tensor", "achieved": tf, "peak": peak, "unit": "TFLOP/s",
                     "frac": tf / peak, "peak_source": f"{kind}: 4 x bf16 (sustained)",
                     "traffic": None},
    }), flush=True)


def main():
    args = parse_args()
    if args.op == "quantize":
        return run_quantize(args)
    if args.op == "moe":
        return run_moe(args)
    if args.config == "all" and args.impl != "reference":
        return run_all_configs(args)
    if args.impl == "reference":
        return run_reference(args)
    if args.impl == "reference_gpu":
        return run_reference_gpu(args)

    import torch
    import torch.distributed as dist

    import submission

    pkg = submission.load_package()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
        # One line per rank on stderr (stdout carries only the JSON line): the NCCL
        # communicator's size as this rank sees it.
        print(f"[bench] rank {rank} of {dist.get_world_size()} (local {local_rank}) on "
              f"{torch.cuda.get_device_name(dev)}, NCCL {torch.cuda.nccl.version()}",
              file=sys.stderr, flush=True)

    # Each rank owns its own experts (seed = rank): weak scaling, no data-path collective.
    # With --shard-experts the ranks split one configuration's experts (strong scaling).
    shard = None
    seed = rank
    strong = args.shard_experts and world > 1 and not args.experts
    if args.experts:
        start, stop = (int(x) for x in args.experts.split(":"))
        shard = slice(start, stop)
    elif strong:
        G = len(pkg.workloads.config_rows(args.config)[0])
        sh = pkg.expert_parallel.expert_shard(G, world, rank)
        shard = slice(sh.start, sh.stop)
        seed = 0  # every rank takes its slice of the same configuration
    prob = pkg.workloads.make_config(args.config, seed=seed, device=dev, experts=shard)
    stream = torch.cuda.current_stream(dev)
    sizes = prob.problem_sizes()

    # The device-resident timing runs a prepared launch: the group table is validated and
    # built once, so each step is one library call (no per-tensor Python work).
    plan = pkg.GroupedGemmPlan(prob.a, prob.b, prob.sfa, prob.sfb, prob.c, sizes,
                               alpha=prob.alpha, b2=prob.b2, sfb2=prob.sfb2, alpha2=prob.alpha2,
                               tile_n=args.tile_n, cta=args.cta, split_k=args.split_k)

    def step():
        plan.run(stream)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t)
        return float(t.item())

    # ---------------------------------------------------------------- headline configs (N = 1)
    # Isolated calls of configs 1-5, timed first, before the sustained-load measurements
    # below, so that each configuration is timed like a run of that shape alone on a warm
    # GPU (not on one held at its power limit by seconds of earlier work); the clocks
    # sampled during this record are reported with it.
    configs = None
    if rank == 0 and world == 1 and not args.no_extras:
        configs = headline_configs(pkg, dev, args.steps, args.warmup, load_peaks()[0], None,
                                   not args.no_clocks)

    # ---------------------------------------------------------------- device-resident timing
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize(dev)
    barrier()

    # Inputs smaller than L2 would be served from it on back-to-back calls: for those
    # configurations a 256 MiB buffer is rewritten before every timed call, outside the
    # events that bracket the call.
    flush_l2 = prob.input_bytes() < L2_BYTES
    flush_buf = torch.empty(256 << 20, dtype=torch.uint8, device=dev) if flush_l2 else None

    host_enqueue_us = []

    def run_timed(n: int) -> float:
        """Device time (ms) of n calls on this rank: one event pair around all of them,
        or, with the L2 flush, one pair per call with the flush between the pairs.
        The host time spent enqueueing the calls is appended to host_enqueue_us."""
        if not flush_l2:
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            t0 = time.perf_counter()
            for _ in range(n):
                step()
            host_enqueue_us.append((time.perf_counter() - t0) / n * 1e6)
            e1.record(stream)
            torch.cuda.synchronize(dev)
            return e0.elapsed_time(e1)
        pairs = []
        host = 0.0
        for _ in range(n):
            flush_buf.fill_(1)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            t0 = time.perf_counter()
            step()
            host += time.perf_counter() - t0
            e1.record(stream)
            pairs.append((e0, e1))
        host_enqueue_us.append(host / n * 1e6)
        torch.cuda.synchronize(dev)
        return sum(a.elapsed_time(b) for a, b in pairs)

    def timed(n: int) -> float:
        """Device time of n calls (ms), max over ranks."""
        barrier()
        torch.cuda.synchronize(dev)
        ms = run_timed(n)
        barrier()
        return max_over_ranks(ms)

    # Burst: right after warm-up, before the GPU reaches its power limit.
    burst_ms = timed(args.steps) / args.steps
    # Clocks are sampled every 200 ms across a load window that contains the timed
    # region: ~1 s of back-to-back calls before it and ~0.5 s after it, so that the
    # samples show the clock the timed calls ran at (the timed region itself is short).
    clocks = ClockSampler(local_rank, enabled=not args.no_clocks)

    def sustain(seconds: float) -> None:
        if args.no_clocks:
            return
        t_end = time.perf_counter() + seconds
        while time.perf_counter() < t_end:
            for _ in range(50):
                step()
            torch.cuda.synchronize(dev)

    sustain(1.0)
    barrier()
    torch.cuda.synchronize(dev)
    ms_rank = run_timed(args.steps)
    host_us = host_enqueue_us[-1]
    barrier()
    sustain(0.5)
    clk = clocks.stop()
    ms_total = max_over_ranks(ms_rank)
    ms_per_step = ms_total / args.steps
    errors = plan.check_device_errors(stream)

    # ---------------------------------------------------------------- with the output gather (N > 1)
    # The same calls followed by the NCCL all-gather that gives every rank every expert's
    # fp16 output (expert_parallel.all_gather_expert_outputs); timed the same way.
    gather = None
    if world > 1:
        rows_all = [None] * world
        dist.all_gather_object(rows_all, list(prob.m))
        rows_flat = [m for r in rows_all for m in r]

        def gather_step():
            plan.run(stream)
            pkg.expert_parallel.all_gather_expert_outputs(prob.c, rows_flat, prob.n)

        for _ in range(3):
            gather_step()
        torch.cuda.synchronize(dev)
        barrier()
        g0 = torch.cuda.Event(enable_timing=True)
        g1 = torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        for _ in range(args.steps):
            gather_step()
        g1.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
        g_ms = max_over_ranks(g0.elapsed_time(g1)) / args.steps
        gather = {"value": prob.flops() * world / (g_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                  "ms_per_step": g_ms,
                  "gather_bytes_received_per_rank": int(sum(rows_flat) * prob.n * 2
                                                        - sum(prob.m) * prob.n * 2),
                  "what": "GEMM + NCCL all-gather of every expert's fp16 output to every rank"}
    flops_rank = prob.flops()
    flops_job = flops_rank * world  # weak scaling: every rank the same amount of work
    if strong:
        t = torch.tensor([flops_rank], dtype=torch.float64, device=dev)
        dist.all_reduce(t)
        flops_job = float(t.item())
    value = flops_job / (ms_per_step * 1e-3) / 1e12

    # ---------------------------------------------------------------- CUDA graph
    # The same calls recorded back to back in one CUDA graph and replayed: no per-call host
    # work or launch gap (programmatic dependent launch edges inside the graph). No L2 flush
    # between the calls in the graph.
    graph_info = None
    if rank == 0 and world == 1:
        try:
            side = torch.cuda.Stream(dev)
            side.wait_stream(stream)
            with torch.cuda.stream(side):
                plan.run(side)
            stream.wait_stream(side)
            torch.cuda.synchronize(dev)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=side):
                for _ in range(args.steps):
                    plan.run(side)
            graph.replay()
            torch.cuda.synchronize(dev)
            q0 = torch.cuda.Event(enable_timing=True)
            q1 = torch.cuda.Event(enable_timing=True)
            q0.record(stream)
            graph.replay()
            q1.record(stream)
            torch.cuda.synchronize(dev)
            graph_ms = q0.elapsed_time(q1) / args.steps
            graph_info = {"us_per_call": graph_ms * 1e3,
                          "value": prob.flops() / (graph_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                          "what": f"{args.steps} GroupedGemmPlan.run calls captured in one CUDA "
                                  "graph, one replay timed"
                                  + ("; L2 not flushed between the calls" if flush_l2 else "")}
            del graph
        except Exception as exc:  # reported, not part of the headline
            graph_info = {"unavailable": f"{type(exc).__name__}: {exc}"[:200]}

    # ---------------------------------------------------------------- library baseline
    # The reference's own GPU arithmetic (ref_kernel: torch._scaled_mm, i.e. cuBLASLt's
    # block-scaled NVFP4 GEMM) once per group on the same device-resident inputs; gated
    # configurations run it twice per group plus silu(g) * u, as the reference's path does.
    lib_base = None
    if rank == 0 and world == 1:
        try:
            f4 = torch.float4_e2m1fn_x2
            e4 = torch.float8_e4m3fn
            ops = []
            for g in range(prob.num_groups):
                if prob.m[g] == 0:
                    continue
                a4 = prob.a[g].view(f4)
                ops.append((a4, prob.b[g].view(f4).t(), prob.sfa[g].view(e4), prob.sfb[g].view(e4),
                            None if not prob.gated else prob.b2[g].view(f4).t(),
                            None if not prob.gated else prob.sfb2[g].view(e4)))

            def lib_step():
                for a4, bt, sa, sb, b2t, sb2 in ops:
                    t1 = torch._scaled_mm(a4, bt, sa, sb, out_dtype=torch.float16)
                    if b2t is not None:
                        t2 = torch._scaled_mm(a4, b2t, sa, sb2, out_dtype=torch.float16)
                        (torch.nn.functional.silu(t1.float()) * t2.float()).half()

            for _ in range(3):
                lib_step()
            torch.cuda.synchronize(dev)
            l0 = torch.cuda.Event(enable_timing=True)
            l1 = torch.cuda.Event(enable_timing=True)
            l0.record(stream)
            for _ in range(args.steps):
                lib_step()
            l1.record(stream)
            torch.cuda.synchronize(dev)
            lib_ms = l0.elapsed_time(l1) / args.steps
            lib_base = {"us_per_call": lib_ms * 1e3,
                        "value": prob.flops() / (lib_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                        "what": "torch._scaled_mm (cuBLASLt block-scaled NVFP4) once per group"
                                + (" x2 + silu(g)*u" if prob.gated else "")
                                + ", device-resident, timed like value (no sustain window)"}
        except Exception as exc:  # the library path is a comparison, not part of the product
            lib_base = {"unavailable": f"{type(exc).__name__}: {exc}"[:200]}

    # ---------------------------------------------------------------- measured NVFP4 peak
    # The library's dense block-scaled FP4 rate on this GPU (every rank its own GPU, rank 0
    # reports), beside the 4 x bf16 figure derived from MEASURED_PEAKS.json.
    nvfp4_peak = None
    if not args.no_extras:
        try:
            nvfp4_peak = measure_nvfp4_peak(dev)
        except Exception as exc:  # a comparison figure, not part of the product
            nvfp4_peak = {"unavailable": f"{type(exc).__name__}: {exc}"[:200]}
    fp4_ok = nvfp4_peak is not None and "burst_tflops" in nvfp4_peak

    if configs is not None and fp4_ok:
        for v in configs["per_config"].values():
            if v["bound"] == "tensor":
                v["frac_of_measured_nvfp4_burst"] = v["tflops"] / nvfp4_peak["burst_tflops"]

    # ---------------------------------------------------------------- cfg5 split over the ranks
    peaks, peak_kind = load_peaks()
    sustained_key = "bf16_tflops_sustained" if "bf16_tflops_sustained" in peaks else "bf16_tflops"
    sharded = None
    if not args.no_extras:
        sharded = sharded_cfg5(pkg, dev, world, rank, args.steps, args.warmup, barrier,
                               max_over_ranks, sum_over_ranks,
                               FP4_PER_BF16 * float(peaks[sustained_key]), True)
        if fp4_ok:
            sharded["frac_of_measured_nvfp4_sustained"] = (
                sharded["tflops"] / (world * nvfp4_peak["sustained_tflops"]))

    # ---------------------------------------------------------------- EP MoE block, split over the ranks
    ep_block = None
    if not args.no_extras:
        ep_block = ep_block_leg(pkg, dev, world, rank, args.steps, args.warmup, barrier,
                                max_over_ranks, sum_over_ranks)
        if "tflops" in ep_block:
            ep_block["frac_of_per_gpu_peak"] = ep_block["tflops"] / (
                world * FP4_PER_BF16 * float(peaks[sustained_key]))

    # ---------------------------------------------------------------- the reference's kernel (N = 1)
    # The reference's own sm_100 kernel (its CuTe-DSL submission, unmodified) through its own
    # custom_kernel on this configuration, beside this library's custom_kernel.
    ref_kernel = None
    if rank == 0 and world == 1 and not args.no_extras and not prob.gated:
        try:
            ref_kernel = reference_kernel_leg(pkg, dev, args.config, args.steps, args.warmup)
        except Exception as exc:  # a comparison, not part of the product
            ref_kernel = {"unavailable": f"{type(exc).__name__}: {exc}"[:200]}

    # ---------------------------------------------------------------- end to end (host buffers)
    # Every step copies its inputs from pinned host memory, calls custom_kernel and copies
    # its fp16 outputs back. Two buffer sets: step i's H2D (copy stream) overlaps step i-1's
    # kernel and D2H (second copy stream), events order each set's reuse. `serial` is the
    # same step with all copies and the call on one stream, one step after another.
    # The same K steps as `value` (at least 4, at most 50 to bound the run's length).
    e2e_steps = args.e2e_steps or max(4, min(args.steps, 50))
    probs = [prob, pkg.workloads.make_config(args.config, seed=seed, device=dev, experts=shard)]

    def inputs_of(p):
        return p.a + p.b + p.sfa + p.sfb + (p.b2 or []) + (p.sfb2 or [])

    host_in = [t.cpu().pin_memory() for t in inputs_of(prob)]
    dev_in = [inputs_of(p) for p in probs]
    host_out = [[torch.empty(c.shape, dtype=c.dtype).pin_memory() for c in p.c] for p in probs]
    datas = [p.reference_data() for p in probs]
    scales = [p.global_scales() for p in probs]
    h2d_stream = torch.cuda.Stream(dev)
    d2h_stream = torch.cuda.Stream(dev)

    def call(i, st):
        pkg.custom_kernel(datas[i], global_scales=scales[i], tile_n=args.tile_n, stream=st,
                          cta=args.cta, split_k=args.split_k)

    def e2e_serial_step():
        for h, d in zip(host_in, dev_in[0]):
            d.copy_(h, non_blocking=True)
        call(0, stream)
        for h, c in zip(host_out[0], probs[0].c):
            h.copy_(c, non_blocking=True)

    k_done = [torch.cuda.Event(), torch.cuda.Event()]
    in_done = [torch.cuda.Event(), torch.cuda.Event()]
    out_done = [torch.cuda.Event(), torch.cuda.Event()]

    def e2e_pipelined(n):
        h2d_stream.wait_stream(stream)
        d2h_stream.wait_stream(stream)
        for i in range(n):
            b = i % 2
            with torch.cuda.stream(h2d_stream):
                h2d_stream.wait_event(k_done[b])  # the kernel two steps back read set b
                for h, d in zip(host_in, dev_in[b]):
                    d.copy_(h, non_blocking=True)
                in_done[b].record(h2d_stream)
            stream.wait_event(in_done[b])
            stream.wait_event(out_done[b])  # set b's outputs of two steps back are on the host
            call(b, stream)
            k_done[b].record(stream)
            with torch.cuda.stream(d2h_stream):
                d2h_stream.wait_event(k_done[b])
                for h, c in zip(host_out[b], probs[b].c):
                    h.copy_(c, non_blocking=True)
                out_done[b].record(d2h_stream)
        stream.wait_stream(h2d_stream)
        stream.wait_stream(d2h_stream)

    def e2e_timed(fn, n):
        torch.cuda.synchronize(dev)
        barrier()
        ev0 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        fn(n)
        ev1.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
        return max_over_ranks(ev0.elapsed_time(ev1)) / n

    e2e_pipelined(2)
    e2e_serial_step()
    e2e_ms = e2e_timed(e2e_pipelined, e2e_steps)
    e2e_serial_ms = e2e_timed(lambda n: [e2e_serial_step() for _ in range(n)], e2e_steps)
    same_out = all(torch.equal(x.view(torch.int16), y.view(torch.int16))
                   for x, y in zip(probs[0].c, probs[1].c))
    h2d = sum(t.numel() * t.element_size() for t in host_in)
    d2h = sum(t.numel() * t.element_size() for t in host_out[0])
    data = datas[0]
    scales = scales[0]
    del probs[1], dev_in, datas
    pcie = pcie_bandwidth(dev, h2d_stream, d2h_stream)
    pcie_ms = max(h2d / (pcie["h2d_concurrent_gbs"] * 1e6), d2h / (pcie["d2h_concurrent_gbs"] * 1e6))

    # The drop-in call itself on device-resident inputs: custom_kernel(data) back to back
    # (device time per call, and the host time to issue one call).
    ck_host = []
    for _ in range(3):
        pkg.custom_kernel(data, global_scales=scales, tile_n=args.tile_n, stream=stream,
                          cta=args.cta, split_k=args.split_k)
    torch.cuda.synchronize(dev)
    barrier()
    ck0 = torch.cuda.Event(enable_timing=True)
    ck1 = torch.cuda.Event(enable_timing=True)
    ck0.record(stream)
    for _ in range(args.steps):
        t0 = time.perf_counter()
        pkg.custom_kernel(data, global_scales=scales, tile_n=args.tile_n, stream=stream,
                          cta=args.cta, split_k=args.split_k)
        ck_host.append(time.perf_counter() - t0)
    ck1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    ck_ms = max_over_ranks(ck0.elapsed_time(ck1)) / args.steps

    # ---------------------------------------------------------------- CPU baseline (rank 0, N=1)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(args.config)

    if world > 1:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()
    if rank != 0:
        return

    # `value` is timed inside a sustained-load window (the clocks above describe it), so
    # its roofline uses the sustained bf16 figure; the burst timing uses the burst one.
    tensor_peak = FP4_PER_BF16 * float(peaks[sustained_key])
    burst_peak = FP4_PER_BF16 * float(peaks["bf16_tflops"])
    achieved = flops_rank / (ms_per_step * 1e-3) / 1e12
    burst_tflops = flops_rank / (burst_ms * 1e-3) / 1e12
    # Roofline: tensor-bound when the arithmetic intensity (FLOPs per algorithmic HBM
    # byte) exceeds the ridge of the measured peaks, HBM-bound otherwise.
    alg_bytes = prob.algorithmic_bytes()
    hbm_peak = float(peaks["hbm_gbs"])
    hbm_gbs = alg_bytes / (ms_per_step * 1e-3) / 1e9
    ridge = tensor_peak * 1e12 / (hbm_peak * 1e9)
    hbm_bound = flops_rank / alg_bytes < ridge
    kernel_tag = args.cta or ("single" if args.tile_n else "auto")
    traffic = load_traffic(kernel_tag, args.config)
    line = {
        "metric": f"NVFP4 grouped GEMM TFLOP/s ({args.config})",
        "value": value,
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": max(args.warmup, 3),
        "ms_per_step": ms_per_step,
        "us_per_call": ms_per_step * 1e3,
        "host_us_per_call": host_us,
        "higher_is_better": True,
        "scaling": "strong" if strong else "weak",
        "vs_baseline": None,
        "dtype": "e2m1xe4m3->f32->f16",
        "data": "synthetic (seeded; e2m1 codes uniform over 16, E4M3 scales 2^U{-4..3})",
        "config": workload_config(args, prob, world, strong),
        "gpu_launches": args.steps,  # one persistent GEMM kernel per timed call (descriptors reused)
        "api": "GroupedGemmPlan.run (value, burst); custom_kernel(data) (e2e)",
        "device_error_bits": errors,
        "e2e": {"value": flops_job / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                "ms_per_step": e2e_ms, "steps": e2e_steps,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "api": "custom_kernel(data); every step: H2D of all inputs from pinned host "
                       "memory, the call, D2H of all outputs; two buffer sets so that step i's "
                       "H2D overlaps step i-1's call and D2H (two copy streams)",
                "serial": {"value": flops_job / (e2e_serial_ms * 1e-3) / 1e12,
                           "ms_per_step": e2e_serial_ms,
                           "what": "the same step with copies and call on one stream"},
                "buffer_sets_equal_outputs": same_out,
                "pcie": dict(pcie, bound_ms_per_step=pcie_ms, frac=pcie_ms / e2e_ms,
                             what="pinned-host copies of 256 MiB alone and with the other "
                                  "direction running (two copy streams); bound_ms_per_step: "
                                  "the step's H2D and D2H bytes at the concurrent rates; frac: "
                                  "that bound over the measured e2e step")},
        "cuda_graph": graph_info,
        "custom_kernel_device_resident": {
            "us_per_call": ck_ms * 1e3, "host_us_per_call": sorted(ck_host)[len(ck_host) // 2] * 1e6,
            "what": "custom_kernel(data) back to back on device-resident inputs (the harness's "
                    "call; descriptors prepared by the first call)" +
                    ("; L2 not flushed between calls" if flush_l2 else "")},
        "burst": {"us_per_call": burst_ms * 1e3, "tflops_per_gpu": burst_tflops,
                  "frac_of_burst_peak": burst_tflops / burst_peak,
                  "hbm_frac": alg_bytes / (burst_ms * 1e-3) / 1e9 / hbm_peak,
                  "note": "timed right after warm-up, before the power limit engages"},
        "roofline": ({"bound": "hbm", "achieved": hbm_gbs, "peak": hbm_peak, "unit": "GB/s",
                      "frac": hbm_gbs / hbm_peak,
                      "peak_source": f"{peak_kind}: hbm_gbs (copy bandwidth)",
                      "traffic": traffic, "algorithmic_bytes": alg_bytes,
                      "tensor_frac": achieved / tensor_peak}
                     if hbm_bound else
                     {"bound": "tensor", "achieved": achieved, "peak": tensor_peak,
                      "unit": "TFLOP/s", "frac": achieved / tensor_peak,
                      "peak_source": f"{peak_kind}: 4 x {sustained_key} "
                                     f"({peaks[sustained_key]}; timed under sustained load)",
                      "traffic": traffic, "algorithmic_bytes": alg_bytes,
                      "hbm_frac": hbm_gbs / hbm_peak,
                      "frac_of_measured_nvfp4": (achieved / nvfp4_peak["sustained_tflops"]
                                                 if fp4_ok else None),
                      "frac_of_nominal_9pf": achieved / NOMINAL_FP4_TFLOPS,
                      "peak_note": "frac: 4 x measured bf16 (the denominator of record); "
                                   "frac_of_measured_nvfp4: cuBLASLt's dense NVFP4 rate "
                                   "measured in this run (sustained); frac_of_nominal_9pf: "
                                   "B200's nominal dense FP4 figure"}),
        "clocks": clk,
    }
    if nvfp4_peak is not None:
        line["nvfp4_peak"] = nvfp4_peak
    if sharded is not None:
        line["sharded_cfg5"] = sharded
    if ep_block is not None:
        line["ep_block"] = ep_block
    if configs is not None:
        line["geomean_us_per_call"] = configs["geomean_us_per_call"]
        line["configs"] = configs
    if ref_kernel is not None:
        line["reference_kernel"] = ref_kernel
    if gather is not None:
        line["with_gather"] = gather
    if lib_base is not None:
        line["library_baseline"] = lib_base
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
