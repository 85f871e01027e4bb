"""Benchmark of the hot path: fused causal flash-attention forward (config 3).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: causal bf16 flash-attention forward,
B=8 H=32 S=4096 D=128, scale 1/sqrt(128), fp32 accumulate, synthetic N(0,1)
inputs.  A step is one forward over the whole batch.  With N GPUs (torchrun,
one process per GPU, NCCL) the job is partitioned by (batch, head) units with
no exchange step inside the forward, so no collective runs in the timed
region.  Default `--scaling weak`: the global batch is 8*N and every rank owns
a config-3-sized block of 256 units (per-GPU work fixed); `--scaling strong`
splits the fixed config-3 job's 256 units into N contiguous shards.  Each rank
keeps its output shard in its own HBM; the optional final NCCL all-gather of
the shards is timed separately (`gather`).
Inputs (805 MB of q/k/v) exceed the 126 MB L2, so no L2 flush is needed.

`value` = algorithmic TFLOP/s of the whole job (causal counted as half of
4*B*H*S^2*D), device-timed with CUDA events, max over ranks.  `e2e` repeats
the step through the public API with pinned HOST buffers (H2D of q/k/v and
D2H of o inside the timed region).  `extra` carries the row-reduction GB/s
(config 2), GQA (config 4) and backward (config 5) numbers at N=1.
The reference arm (`--impl reference`) times the CPU oracle (the reference's
numpy f64 denotation) on bounded samples of the same workload.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

B, H, S, D = 8, 32, 4096, 128
FLOP_FULL = 4.0 * B * H * S * S * D / 2  # causal: half of 4*B*H*S^2*D
# NVLink 5 peer copy measured on this pool (per direction) and a typical NCCL
# launch-to-completion latency: the alpha-beta link model for the gather prediction
NVLINK_BPS = 770e9
NCCL_LATENCY_S = 10e-6


def _peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running."""

    REASONS = {0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x4: "sw_power_cap", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, index: int):
        self.samples, self.reasons, self.ok = [], set(), False
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:  # pragma: no cover - no NVML
            self.max_mhz = None
        self._stop = threading.Event()

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for bit, name in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.01)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        if self.ok:
            self._stop.set()
            self.t.join()

    def summary(self):
        s = sorted(self.samples)
        return {"sm_mhz": s[len(s) // 2] if s else None, "sm_max_mhz": self.max_mhz, "samples": len(s),
                "reasons": sorted(self.reasons)}


def _dist():
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    return world, rank, local


def _shard(world, rank, scaling):
    """(lo, hi) units of this rank and the global unit count."""
    from pdum_dsl_b200.partition import shard_units

    total = B * H * (world if scaling == "weak" else 1)
    sh = shard_units(total, world, rank)
    return sh.lo, sh.hi, total


def _timed(fn, steps, warmup, stream, world):
    """CUDA-event time of `steps` calls of fn (after `warmup`), max over ranks; per-call event times."""
    import torch
    import torch.distributed as dist

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    ev[0].record(stream)
    for i in range(steps):
        fn()
        ev[i + 1].record(stream)
    torch.cuda.synchronize()
    per = [ev[i].elapsed_time(ev[i + 1]) for i in range(steps)]
    total = ev[0].elapsed_time(ev[steps])
    if world > 1:
        t = torch.tensor([total], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total = float(t.item())
        dist.barrier()
    return total, per


def cpu_attention_sample(head_seq=S, rows=S, min_seconds=0.0):
    """Time the oracle (numpy f64) on whole causal heads of config 3: `rows` query rows
    at the END of a head of length head_seq (the heaviest rows), repeated over fresh
    seeded heads until at least `min_seconds` of CPU time have been spent (a bounded
    sample of the workload); returns (tflops, seconds, desc)."""
    import numpy as np

    from oracle import attention as OA

    # causal work of those rows: sum over rows of (t+1) keys, 4*D flops per (row, key)
    t_abs = np.arange(head_seq - rows, head_seq) + 1
    flops_head = 4.0 * D * float(t_abs.sum())
    heads, dt = 0, 0.0
    while heads == 0 or dt < min_seconds:
        rng = np.random.default_rng(heads)
        q = rng.standard_normal((rows, D))
        k = rng.standard_normal((head_seq, D))
        v = rng.standard_normal((head_seq, D))
        t0 = time.perf_counter()
        OA.attention_fwd(q, k, v, scale=1 / math.sqrt(D), causal=True, q_start=head_seq - rows, row_block=256)
        dt += time.perf_counter() - t0
        heads += 1
    desc = (f"{heads} causal head(s) of {rows} query rows x {head_seq} keys (D={D}) of config 3's "
            f"{B * H}, numpy f64, {dt:.1f} s")
    return flops_head * heads / dt / 1e12, dt, desc


def _cpu_threads():
    try:
        from threadpoolctl import threadpool_info

        n = max((i.get("num_threads", 1) for i in threadpool_info()), default=1)
        return int(n)
    except Exception:
        return os.cpu_count() or 1


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    vals = []
    for _ in range(args.warmup_ref):
        cpu_attention_sample(rows=256)
    t_all = 0.0
    desc = ""
    for _ in range(args.steps_ref):
        tf, dt, desc = cpu_attention_sample(min_seconds=6.0)
        vals.append(tf)
        t_all += dt
    v = sorted(vals)[len(vals) // 2]
    line = {
        "impl": "reference", "metric": "fused-attn TFLOP/s (causal flash fwd, config 3)", "value": v,
        "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps_ref, "warmup": args.warmup_ref,
        "ms_per_step": 1e3 * t_all / max(1, args.steps_ref), "higher_is_better": True, "scaling": args.scaling,
        "vs_baseline": None, "dtype": "f64", "data": "synthetic N(0,1), seeded",
        "config": {"workload": "flash-attention forward, causal, B=8 H=32 S=4096 D=128 (config 3)",
                   "sample": desc},
        "cpu_baseline": {"value": v, "unit": "TFLOP/s", "cores": _cpu_threads(), "kind": "port", "sample": desc},
        "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args):
    import torch
    import torch.distributed as dist

    from pdum_dsl_b200 import kernels
    from pdum_dsl_b200._lib import load

    load()
    world, rank, local = _dist()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    lo, hi, total_units = _shard(world, rank, args.scaling)
    units = hi - lo
    flop_job = FLOP_FULL * total_units / (B * H)  # the whole job over all ranks
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    # this rank's (batch, head) units as one (1, units, S, D) job
    q, k, v = (torch.randn((1, units, S, D), device=dev, generator=g, dtype=torch.float32).to(torch.bfloat16)
               for _ in range(3))
    o = torch.empty_like(q)
    step = lambda: kernels.flash_attention(q, k, v, causal=True, out=o)
    sampler = ClockSampler(local)
    with sampler:
        total_ms, per = _timed(step, args.steps, args.warmup, stream, world)
    kernels.check_device_errors()
    flop_rank = FLOP_FULL * units / (B * H)
    value = flop_job * args.steps / (total_ms * 1e-3) / 1e12
    peaks = _peaks()
    launch_ms = sum(per) / len(per)
    achieved = flop_rank / (launch_ms * 1e-3) / 1e12

    gather = None
    if world > 1 and (B * H) % world == 0:
        # the north star's final NCCL gather of the output shards, timed on its own
        full = torch.empty((world * units, S, D), dtype=o.dtype, device=dev)
        g_ms, _ = _timed(lambda: dist.all_gather_into_tensor(full, o.reshape(units, S, D)), 5, 2, stream, world)
        nbytes = o.numel() * o.element_size()
        from pdum_dsl_b200.partition import alpha_beta_seconds, gather_bytes

        moved = gather_bytes(nbytes * world, world)  # what placement.traffic charges the merge
        gather = {"ms": g_ms / 5, "bytes_in_per_rank": moved,
                  "GB/s_in_per_rank": moved / (g_ms / 5 * 1e-3) / 1e9,
                  "predicted_ms": 1e3 * alpha_beta_seconds(moved, NVLINK_BPS, NCCL_LATENCY_S),
                  "model": "placement.traffic all-gather ((p-1)/p x output bytes), alpha-beta at "
                           f"{NVLINK_BPS / 1e9:.0f} GB/s per direction + {NCCL_LATENCY_S * 1e6:.0f} us",
                  "note": "all_gather_into_tensor of o shards over NCCL; outside `value`"}
        del full
    if args.kernel_only:
        if rank == 0:
            print(json.dumps({"workload": [B, H, S, D], "n_gpus": world, "gather": gather, "value": value, "unit": "TFLOP/s", "launch_ms": launch_ms,
                              "achieved": achieved, "clocks": sampler.summary()}), flush=True)
        return
    # ---- e2e: the same step through the public API with pinned host buffers
    qh, kh, vh = (x.cpu().pin_memory() for x in (q, k, v))
    oh = torch.empty(o.shape, dtype=o.dtype, pin_memory=True)

    from pdum_dsl_b200.host import flash_attention_host

    def e2e_step():  # the host-buffer entry point: chunked, copies overlapped with compute
        flash_attention_host(qh, kh, vh, oh, causal=True)

    e2e_steps = max(1, min(args.steps, 10))
    e2e_ms, _ = _timed(e2e_step, e2e_steps, 1, stream, world)
    e2e_val = flop_job * e2e_steps / (e2e_ms * 1e-3) / 1e12
    h2d = 3 * q.numel() * q.element_size() * world
    d2h = o.numel() * o.element_size() * world

    extra = {}
    cpu_base = None
    if world == 1 and not args.no_extra:
        extra = secondary(args, dev, stream, peaks)
    elif world > 1 and not args.no_extra:
        del qh, kh, vh, oh
        torch.cuda.empty_cache()
        gq = _gqa_sharded(world, rank, dev, stream)
        if gq is not None:
            extra["gqa_fwd_sharded"] = gq
    if rank == 0 and world == 1 and not args.no_cpu:
        tf, dt, desc = cpu_attention_sample(min_seconds=10.0)
        cpu_base = {"value": tf, "unit": "TFLOP/s", "cores": _cpu_threads(), "kind": "port", "sample": desc,
                    "seconds": round(dt, 2)}
    if world > 1:
        dist.barrier()
    if rank == 0:
        line = {
            "metric": "fused-attn TFLOP/s (causal flash fwd, config 3)", "value": value, "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms / args.steps,
            "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic N(0,1) (torch.randn, seeded), bf16",
            "config": {"workload": "flash-attention forward, causal, B=8 H=32 S=4096 D=128, scale 1/sqrt(128) "
                                   "(config 3)", "global_batch": B * total_units // (B * H), "heads": H, "seq_len": S, "head_dim": D,
                       "parallelism": f"batch x head shards over {world} GPU(s), {args.scaling} scaling",
                       "l2": "inputs 805 MB > 126 MB L2 (no flush)"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": achieved / peaks["bf16_tflops"], "peak_source": peaks["source"] + " (burst)",
                         "frac_sustained": achieved / peaks["bf16_tflops_sustained"]
                         if peaks.get("bf16_tflops_sustained") else None,
                         # ncu dram read+write of one launch at B=2 (the full ncu capture of this kernel),
                         # scaled by the 4x units of a config-3 launch; algorithmic bytes are 1073.7 MB
                         "traffic": 4 * (202.89e6 + 45.39e6) * units / (B * H) if (B, H, S, D) == (8, 32, 4096, 128)
                         else None, "traffic_unit": "bytes per launch",
                         "kernel": "flash_fwd_sm100_kernel<128>",
                         "launch_ms": launch_ms},
            "clocks": sampler.summary(),
            "e2e": {"value": e2e_val, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "steps": e2e_steps},
            "gpu_launches": args.steps,
            "cpu_baseline": cpu_base,
            "extra": extra,
            "gather": gather,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def secondary(args, dev, stream, peaks, parts=("rows", "gqa", "bwd", "gemm")):
    """Config 2 (row reductions), 4 (GQA) and 5 (backward) at N=1."""
    import torch

    from pdum_dsl_b200 import kernels

    out = {}
    g = torch.Generator(device=dev).manual_seed(7)
    if "rows" in parts:
        _rows(out, kernels, dev, stream, peaks, g)
    if "gqa" in parts:
        _gqa(out, kernels, dev, stream, g)
    if "bwd" in parts:
        _bwd(out, kernels, dev, stream, g)
    if "gemm" in parts:
        _gemm(out, kernels, dev, stream, g, peaks)
    return out


def _gemm(out, kernels, dev, stream, g, peaks):
    """Contraction-epilogue template (bf16 tcgen05 path): relu(A B^T + bias), 8192^3."""
    import torch

    M = N = K = 8192
    a = torch.randn((1, M, K), device=dev, generator=g).to(torch.bfloat16)
    b = torch.randn((1, N, K), device=dev, generator=g).to(torch.bfloat16)
    bias = torch.randn((1, 1, N), device=dev, generator=g)
    c = torch.empty((1, M, N), dtype=torch.bfloat16, device=dev)
    ep = [("add", bias, False), ("maximum", 0.0, False)]
    ms, per = _timed(lambda: kernels.contract(a, b, epilogue=ep, out=c), 10, 3, stream, 1)
    tf = 2.0 * M * N * K / (sum(per) / len(per) * 1e-3) / 1e12
    out["contract_bf16"] = {"TFLOP/s": tf, "frac_peak": tf / peaks["bf16_tflops"], "ms": sum(per) / len(per),
                            "config": "relu(A B^T + bias), M=N=K=8192, bf16 in/out, fp32 accumulate"}


def _rows(out, kernels, dev, stream, peaks, g):
    import torch

    x = torch.randn(8192, 4096, device=dev, generator=g)
    y = torch.empty_like(x)
    gam = 1 + 0.1 * torch.randn(4096, device=dev, generator=g)
    bet = 0.1 * torch.randn(4096, device=dev, generator=g)
    nbytes = 2 * x.numel() * 4
    for name, fn in (("row_softmax", lambda: kernels.row_softmax(x, out=y)),
                     ("layernorm", lambda: kernels.layernorm(x, gam, bet, 1e-5, out=y))):
        ms, per = _timed(fn, 50, 5, stream, 1)
        gbs = nbytes / (sum(per) / len(per) * 1e-3) / 1e9
        out[name] = {"GB/s": gbs, "frac_hbm": gbs / peaks["hbm_gbs"], "us_per_call": 1e3 * sum(per) / len(per),
                     "bytes_per_call": nbytes, "config": "X 8192x4096 f32 (config 2)"}


def _gqa(out, kernels, dev, stream, g):
    import torch

    # config 4: GQA fwd, B4 Hq64 Hkv8 S8192 D128 causal
    Bq, Hq, Hk, Sq = 4, 64, 8, 8192
    q = torch.randn((Bq, Hq, Sq, D), device=dev, generator=g).to(torch.bfloat16)
    k = torch.randn((Bq, Hk, Sq, D), device=dev, generator=g).to(torch.bfloat16)
    v = torch.randn((Bq, Hk, Sq, D), device=dev, generator=g).to(torch.bfloat16)
    o = torch.empty_like(q)
    ms, per = _timed(lambda: kernels.flash_attention(q, k, v, causal=True, out=o), 5, 2, stream, 1)
    fl = 4.0 * Bq * Hq * Sq * Sq * D / 2
    out["gqa_fwd"] = {"TFLOP/s": fl / (sum(per) / len(per) * 1e-3) / 1e12, "ms": sum(per) / len(per),
                      "config": "B4 Hq64 Hkv8 S8192 D128 causal (config 4)"}


def _gqa_sharded(world, rank, dev, stream):
    """Config 4 over `world` GPUs: the KV groups split by the placement rule
    (b, w, gl) with w bound to the GPU level, each rank computing its block of
    KV heads of every batch, then the NCCL all-gather of the output shards.
    Strong scaling (the problem is fixed); device time, max over ranks."""
    import torch
    import torch.distributed as dist

    from pdum_dsl_b200 import kernels
    from pdum_dsl_b200.partition import Placement, alpha_beta_seconds, gather_bytes

    Bq, Hq, Hk, Sq = 4, 64, 8, 8192
    if Hk % world:
        return None
    pl = Placement("g", "gpu", world, Hk // world)
    r = Hq // Hk
    g = torch.Generator(device=dev).manual_seed(4321 + rank)
    # this rank's shard only: query heads of its KV groups, and those K/V heads
    q = torch.randn((Bq, pl.local * r, Sq, D), device=dev, generator=g).to(torch.bfloat16)
    k = torch.randn((Bq, pl.local, Sq, D), device=dev, generator=g).to(torch.bfloat16)
    v = torch.randn((Bq, pl.local, Sq, D), device=dev, generator=g).to(torch.bfloat16)
    o = torch.empty_like(q)
    ms, _ = _timed(lambda: kernels.flash_attention(q, k, v, causal=True, out=o), 5, 2, stream, world)
    fl = 4.0 * Bq * Hq * Sq * Sq * D / 2
    full = torch.empty((world, *o.shape), dtype=o.dtype, device=dev)
    g_ms, _ = _timed(lambda: dist.all_gather_into_tensor(full.reshape(-1, Sq, D), o.reshape(-1, Sq, D)), 5, 2,
                     stream, world)
    moved = gather_bytes(o.numel() * o.element_size() * world, world)
    del full
    return {"TFLOP/s": fl / (ms / 5 * 1e-3) / 1e12, "ms": ms / 5, "n_gpus": world,
            "partition": f"KV groups over {world} GPUs (placement g -> (w, gl), {pl.local} KV heads per GPU)",
            "gather": {"ms": g_ms / 5, "bytes_in_per_rank": moved, "GB/s_in_per_rank": moved / (g_ms / 5 * 1e-3) / 1e9,
                       "predicted_ms": 1e3 * alpha_beta_seconds(moved, NVLINK_BPS, NCCL_LATENCY_S)},
            "config": "B4 Hq64 Hkv8 S8192 D128 causal (config 4), strong scaling"}


def _bwd(out, kernels, dev, stream, g):
    import torch

    # config 5: backward, B4 H16 S2048 D64 causal
    Bb, Hb, Sb, Db = 4, 16, 2048, 64
    q, k, v, do = (torch.randn((Bb, Hb, Sb, Db), device=dev, generator=g).to(torch.bfloat16) for _ in range(4))
    try:
        o, lse = kernels.flash_attention(q, k, v, causal=True, return_lse=True)
        ms, per = _timed(lambda: kernels.flash_attention_backward(q, k, v, o, do, lse, causal=True), 20, 3, stream, 1)
        fl = 2.5 * 4.0 * Bb * Hb * Sb * Sb * Db / 2
        out["flash_bwd"] = {"TFLOP/s": fl / (sum(per) / len(per) * 1e-3) / 1e12, "ms": sum(per) / len(per),
                            "config": "B4 H16 S2048 D64 causal (config 5), 2.5x fwd FLOP convention"}
    except Exception as e:  # the backward is reported, not required, for the headline line
        out["flash_bwd"] = {"error": str(e)[:200]}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--scaling", choices=("weak", "strong"), default="weak")
    ap.add_argument("--no-extra", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--shape", default=None,
                    help="B,H,S,D override of the flash workload (profiling a smaller case); implies --kernel-only")
    ap.add_argument("--kernel-only", action="store_true", help="time only the flash forward (no e2e/extra/cpu)")
    ap.add_argument("--only", choices=("rows", "gqa", "bwd", "gemm"), default=None,
                    help="run only one secondary workload (config 2, 4 or 5) and print it (profiling)")
    args = ap.parse_args()
    if args.only:
        import torch

        from pdum_dsl_b200._lib import load

        load()
        dev = torch.device("cuda", 0)
        print(json.dumps(secondary(args, dev, torch.cuda.current_stream(dev), _peaks(), (args.only,))), flush=True)
        return
    if args.shape:
        global B, H, S, D, FLOP_FULL
        B, H, S, D = (int(x) for x in args.shape.split(","))
        FLOP_FULL = 4.0 * B * H * S * S * D / 2
        args.kernel_only = True
    if args.kernel_only:
        args.no_extra = args.no_cpu = True
    args.warmup = max(args.warmup, 3)
    args.steps_ref = max(1, min(args.steps, 5))
    args.warmup_ref = 1
    if args.impl == "reference":
        run_reference(args)
    else:
        try:
            run_ours(args)
        finally:
            import torch.distributed as dist

            if dist.is_available() and dist.is_initialized():
                dist.destroy_process_group()


if __name__ == "__main__":
    main()
