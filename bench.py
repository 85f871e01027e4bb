"""Benchmark of the hot path: fused causal flash-attention forward (config 3).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: causal bf16 flash-attention forward,
B=8 H=32 S=4096 D=128, scale 1/sqrt(128), fp32 accumulate, synthetic N(0,1)
inputs (each (batch, head) unit drawn from its own seeded generator, so every
N sees the same job).  A step is one forward over this rank's units.  With N
GPUs (torchrun, one process per GPU, NCCL) the fixed config-3 job's 256
(batch, head) units are split N ways (`--scaling strong`, the default; the
north star's 1/2/4/8-GPU figures are quoted on this fixed job) with no
exchange inside the forward; `--scaling weak` gives every rank a full
config-3 job instead.
Inputs (805 MB of q/k/v at N=1) exceed the 126 MB L2, so no L2 flush is needed.

`value` = algorithmic TFLOP/s of the whole job (causal counted as half of
4*B*H*S^2*D), device-timed with CUDA events, max over ranks.  At N>1,
`gather_inclusive` times the forward together with the final NCCL all-gather
of the output (the slabs' gathers overlapped with the next slab's compute).
`e2e` repeats the step through the drop-in runner `compile_tile(region,
dtype="bf16")` with pinned HOST buffers (H2D of q/k/v and D2H of o inside
the timed region).  `extra` (N=1) carries config 2 (row reductions), 4 (GQA)
and 5 (backward) with roofline fractions and CPU baselines, and `bars`
times torch's SDPA and the reference's own Triton flash column on config 3.
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


GATHER_SLABS = 4  # slabs of the overlapped final gather (N > 1)
GATHER_SM_MARGIN = 16  # SMs the forward leaves to NCCL's all-gather kernels while they overlap


def _shard(world, rank, scaling):
    """This rank's units (a list of (lo, hi) global unit ranges) and the global unit
    count.  Strong scaling: the slab-interleaved partition of the fixed job, so the
    final all-gather of each slab lands in place (partition.chunked_shards)."""
    from pdum_dsl_b200.partition import chunked_shards, shard_units

    if scaling == "weak" or world == 1:
        total = B * H * (world if scaling == "weak" else 1)
        sh = shard_units(total, world, rank)
        return [(sh.lo, sh.hi)], total
    total = B * H
    slabs = GATHER_SLABS if total % (GATHER_SLABS * world) == 0 else 1
    return [(x.lo, x.hi) for x in chunked_shards(total, world, rank, slabs)], total


def _unit_inputs(ranges, dev, seed_base=1234):
    """q, k, v of the given global units as (1, units, S, D) bf16: unit u of tensor i
    is N(0,1) from its own generator seeded (seed_base, i, u), so a unit's data is
    the same whichever rank draws it."""
    import torch

    units = sum(hi - lo for lo, hi in ranges)
    out = []
    for i in range(3):
        t = torch.empty((1, units, S, D), dtype=torch.bfloat16, device=dev)
        j = 0
        for lo, hi in ranges:
            for u in range(lo, hi):
                g = torch.Generator(device=dev).manual_seed(seed_base + 100003 * i + u)
                t[0, j] = torch.randn((S, D), device=dev, generator=g, dtype=torch.float32).to(torch.bfloat16)
                j += 1
        out.append(t)
    return out


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


def _dsl_on_path():
    """The reference DSL (pdum.dsl / pdum.tl) the drop-in runner plans against: an
    installed copy, or the importable copy kept in baseline/_ref."""
    for pkg in ("dsl", "tensorlib"):
        src = REPO / "baseline" / "_ref" / "packages" / pkg / "src"
        if src.is_dir() and str(src) not in sys.path:
            sys.path.insert(0, str(src))


def _region(units):
    """The attention region of a (1, units, S, D) job, spelled as the DSL spells it."""
    from pdum_dsl_b200.regions import attention_region

    return attention_region(B=1, H=units, T=S, D=D, causal=True, scale=1 / math.sqrt(D))


def _e2e(q, k, v, o, flop_job, world, stream, steps):
    """The same step through the drop-in runner (compile_tile(region, dtype="bf16"))
    with pinned host buffers: H2D of q/k/v, the kernel, D2H of o every step."""
    import torch

    qh, kh, vh = (x.cpu().pin_memory() for x in (q, k, v))
    oh = torch.empty(o.shape, dtype=o.dtype, pin_memory=True)
    api = "compile_tile(attention_region(...), dtype='bf16')(values, out=host) [pinned host buffers]"
    try:
        _dsl_on_path()
        from pdum_dsl_b200.tile import compile_tile

        run = compile_tile(_region(q.shape[1]), dtype="bf16")
        step = lambda: run([qh, kh, vh], out=oh)  # noqa: E731
    except Exception as e:  # the DSL is not importable on this host: the host-buffer entry point
        from pdum_dsl_b200.host import flash_attention_host

        api = f"host.flash_attention_host (compile_tile unavailable: {type(e).__name__})"
        step = lambda: flash_attention_host(qh, kh, vh, oh, causal=True)  # noqa: E731
    n = max(1, min(steps, 10))
    ms, _ = _timed(step, n, 1, stream, world)
    h2d = 3 * q.numel() * q.element_size() * world
    d2h = o.numel() * o.element_size() * world
    return {"value": flop_job * n / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "steps": n, "api": api}


def _gather_inclusive(q, k, v, ranges, world, stream, flop_job):
    """Forward + the final NCCL all-gather of the output, one step = every slab's
    kernel and its all_gather_into_tensor, each slab's gather overlapping the next
    slab's kernel (partition.gather_overlapped); device time, max over ranks."""
    import torch
    import torch.distributed as dist

    from pdum_dsl_b200 import kernels
    from pdum_dsl_b200.partition import alpha_beta_seconds, gather_bytes, gather_overlapped

    dev = q.device
    full = torch.empty((B * H, S, D), dtype=q.dtype, device=dev)
    slab = (B * H) // len(ranges)
    ins, outs, j = [], [], 0
    o = torch.empty_like(q)
    for c, (lo, hi) in enumerate(ranges):
        n = hi - lo
        ins.append((q[:, j:j + n], k[:, j:j + n], v[:, j:j + n], o[:, j:j + n]))
        outs.append(full[c * slab:(c + 1) * slab])
        j += n
    comm = torch.cuda.Stream(dev)

    # the forward leaves SMs to NCCL so the gather of slab c runs while slab c + 1 computes
    # (the persistent kernel otherwise holds every SM until it retires)
    def attend(qs, ks, vs, os_):
        return kernels.flash_attention(qs, ks, vs, causal=True, out=os_, sm_margin=GATHER_SM_MARGIN)

    step = lambda: gather_overlapped(attend, ins, outs, comm_stream=comm)  # noqa: E731
    ms, _ = _timed(step, 5, 2, stream, world)
    # the plain gather alone (no compute), for the link figure
    flat = o.reshape(-1, S, D)
    g_ms, _ = _timed(lambda: dist.all_gather_into_tensor(full, flat), 5, 2, stream, world) if len(ranges) == 1 \
        else _timed(lambda: [dist.all_gather_into_tensor(outs[c], ins[c][3].reshape(-1, S, D))
                             for c in range(len(ranges))], 5, 2, stream, world)
    moved = gather_bytes(full.numel() * full.element_size(), world)
    peer = _peer_gather(ins, ranges, full, stream, world, flop_job, moved)
    return {"value": flop_job * 5 / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms": ms / 5, "slabs": len(ranges),
            "gather_alone_ms": g_ms / 5, "bytes_in_per_rank": moved,
            "GB/s_in_per_rank": moved / (g_ms / 5 * 1e-3) / 1e9,
            "predicted_gather_ms": 1e3 * alpha_beta_seconds(moved, NVLINK_BPS, NCCL_LATENCY_S),
            "model": "placement.traffic all-gather ((p-1)/p x output bytes), alpha-beta at "
                     f"{NVLINK_BPS / 1e9:.0f} GB/s per direction + {NCCL_LATENCY_S * 1e6:.0f} us",
            "sm_margin": GATHER_SM_MARGIN,
            "note": "forward + all_gather_into_tensor per slab on a side stream (NCCL, no multicast loads); "
                    "the forward leaves sm_margin SMs to NCCL so the gathers overlap the next slab",
            "copy_engine": peer}


def _peer_gather(ins, ranges, full_nccl, stream, world, flop_job, moved):
    """The same step with the gather done by copy engines into peer-mapped symmetric
    memory (partition.PeerGather): each slab's kernel writes into the global output
    and its rows are pushed to every peer under the next slab's kernel; the forward
    keeps every SM. Checked bit-equal against the NCCL-gathered output."""
    import torch

    from pdum_dsl_b200 import kernels
    from pdum_dsl_b200.partition import PeerGather, peer_gather_overlapped

    try:
        pg = PeerGather(tuple(full_nccl.shape), full_nccl.dtype, full_nccl.device)
    except Exception as e:  # symmetric memory unavailable on this box / build
        return {"unavailable": f"{type(e).__name__}: {e}"[:200]}

    def attend(qs, ks, vs, _o, out):
        return kernels.flash_attention(qs, ks, vs, causal=True, out=out.unsqueeze(0))

    step = lambda: peer_gather_overlapped(attend, ins, ranges, pg)  # noqa: E731
    ms, _ = _timed(step, 5, 2, stream, world)
    def push_all():  # the gather alone (no compute), for the link figure
        for lo, hi in ranges:
            pg.push(lo, hi)
        pg.finish()

    g_ms, _ = _timed(push_all, 5, 2, stream, world)
    torch.cuda.synchronize()
    same = bool(torch.equal(pg.full, full_nccl))
    return {"value": flop_job * 5 / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms": ms / 5,
            "gather_alone_ms": g_ms / 5, "GB/s_in_per_rank": moved / (g_ms / 5 * 1e-3) / 1e9,
            "matches_nccl_gather": same, "sm_margin": 0,
            "note": "forward writing into symmetric memory + one cudaMemcpyAsync per peer and slab on side "
                    "streams (copy engines over NVLink, no SMs, no multicast), closed by a one-word NCCL all-reduce"}


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
    ranges, total_units = _shard(world, rank, args.scaling)
    units = sum(hi - lo for lo, hi in ranges)
    flop_job = FLOP_FULL * total_units / (B * H)  # the whole job over all ranks
    q, k, v = _unit_inputs(ranges, dev)
    o = torch.empty_like(q)
    step = lambda: kernels.flash_attention(q, k, v, causal=True, out=o)  # noqa: E731
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
    if world > 1 and args.scaling == "strong" and (B * H) % world == 0:
        gather = _gather_inclusive(q, k, v, ranges, world, stream, flop_job)
    if args.kernel_only:
        if rank == 0:
            print(json.dumps({"workload": [B, H, S, D], "n_gpus": world, "gather_inclusive": gather, "value": value,
                              "unit": "TFLOP/s", "launch_ms": launch_ms, "achieved": achieved,
                              "clocks": sampler.summary()}), flush=True)
        return
    e2e = _e2e(q, k, v, o, flop_job, world, stream, args.steps)

    extra, bars = {}, None
    cpu_base = None
    if world == 1 and not args.no_extra:
        extra = secondary(args, dev, stream, peaks)
    elif world > 1 and not args.no_extra:
        torch.cuda.empty_cache()
        gq = _gqa_sharded(world, rank, dev, stream)
        if gq is not None:
            extra["gqa_fwd_sharded"] = gq
    if world == 1 and not args.no_bars:
        bars = _bars(q, k, v, o, stream, value)
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
            "data": "synthetic N(0,1) (per-unit seeded torch generators), bf16",
            "config": {"workload": "flash-attention forward, causal, B=8 H=32 S=4096 D=128, scale 1/sqrt(128) "
                                   "(config 3)", "global_batch": B * total_units // (B * H), "heads": H, "seq_len": S,
                       "head_dim": D,
                       "parallelism": f"batch x head shards over {world} GPU(s), {args.scaling} scaling"
                                      + (f", {len(ranges)} slab(s) per rank" if world > 1 else ""),
                       "l2": "inputs 805 MB > 126 MB L2 (no flush)"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": achieved / peaks["bf16_tflops"], "peak_source": peaks["source"] + " (burst)",
                         "frac_sustained": achieved / peaks["bf16_tflops_sustained"]
                         if peaks.get("bf16_tflops_sustained") else None,
                         # ncu dram read+write of one launch at B=2 (the full ncu capture of this kernel),
                         # scaled by the units of this launch; algorithmic bytes are 1073.7 MB at config 3
                         "traffic": 4 * (202.89e6 + 45.39e6) * units / (B * H) if (S, D) == (4096, 128)
                         else None, "traffic_unit": "bytes per launch",
                         "kernel": "flash_fwd_sm100_kernel<128>",
                         "launch_ms": launch_ms},
            "clocks": sampler.summary(),
            "e2e": e2e,
            "gpu_launches": args.steps,
            "cpu_baseline": cpu_base,
            "gather_inclusive": gather,
            "bars": bars,
            "extra": extra,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def _bars(q, k, v, o, stream, ours):
    """Labelled bars on the same box and workload: torch's SDPA (the baseline call of
    conformance/torch_zoo.py:99-100, here with the config's scale) and the reference's
    own hand-written Triton flash column (conformance/triton_zoo.py:46-79: single
    head, f32, IEEE dot, 32 x 32 blocks, one launch per head), timed on a sample of
    config-3 heads and scaled to TFLOP/s."""
    import torch
    import torch.nn.functional as F

    out = {}
    sc = 1 / math.sqrt(D)
    try:
        ms, _ = _timed(lambda: F.scaled_dot_product_attention(q, k, v, is_causal=True, scale=sc), 10, 3, stream, 1)
        tf = FLOP_FULL * q.shape[1] / (B * H) / (ms / 10 * 1e-3) / 1e12
        out["torch_sdpa"] = {"TFLOP/s": tf, "ms": ms / 10, "ours_over_bar": ours / tf,
                             "call": "F.scaled_dot_product_attention(q, k, v, is_causal=True, scale=1/sqrt(D)), bf16"}
    except Exception as e:  # pragma: no cover - reported, not required
        out["torch_sdpa"] = {"error": str(e)[:200]}
    try:
        sys.path.insert(0, str(REPO / "baseline" / "_ref"))
        from conformance import triton_zoo as TZ  # the reference's own code, unchanged
        import triton

        heads = 4
        qf, kf, vf = (x[0, :heads].float().contiguous() for x in (q, k, v))
        qf = (qf * sc).contiguous()  # the column takes unscaled scores
        of = torch.empty_like(qf)

        def run():
            for h in range(heads):
                TZ._flash_kernel[(triton.cdiv(S, 32),)](qf[h], kf[h], vf[h], of[h], S, D, 32, 32)

        ms, _ = _timed(run, 3, 1, stream, 1)
        tf = FLOP_FULL * heads / (B * H) / (ms / 3 * 1e-3) / 1e12
        out["reference_triton_flash"] = {
            "TFLOP/s": tf, "ms_per_head": ms / 3 / heads, "ours_over_bar": ours / tf,
            "call": "conformance/triton_zoo.py _flash_kernel (f32, input_precision='ieee', BT=BS=32), "
                    f"{heads} config-3 heads, q pre-scaled by 1/sqrt(D)"}
    except Exception as e:
        out["reference_triton_flash"] = {"error": f"{type(e).__name__}: {str(e)[:200]}"}
    return out


def secondary(args, dev, stream, peaks, parts=("rows", "gqa", "bwd", "gemm")):
    """Config 2 (row reductions), 4 (GQA) and 5 (backward) at N=1."""
    import torch

    from pdum_dsl_b200 import kernels

    out = {}
    g = torch.Generator(device=dev).manual_seed(7)
    cpu = not args.no_cpu
    if "rows" in parts:
        _rows(out, kernels, dev, stream, peaks, g, cpu=cpu)
    if "gqa" in parts:
        _gqa(out, kernels, dev, stream, g, peaks, cpu=cpu)
    if "bwd" in parts:
        _bwd(out, kernels, dev, stream, g, peaks, cpu=cpu)
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


def _cpu_seconds(fn, min_seconds):
    """Repeat fn until min_seconds of wall time; returns (seconds per call, calls)."""
    n, dt = 0, 0.0
    while n == 0 or dt < min_seconds:
        t0 = time.perf_counter()
        fn()
        dt += time.perf_counter() - t0
        n += 1
    return dt / n, n


def _rows(out, kernels, dev, stream, peaks, g, cpu=True):
    """Config 2: X 8192 x 4096 ~ N(0,1), gamma ~ N(1, 0.1), beta ~ N(0, 0.1), eps 1e-5."""
    import torch

    x = torch.randn(8192, 4096, device=dev, generator=g)
    y = torch.empty_like(x)
    gam = 1 + 0.1 * torch.randn(4096, device=dev, generator=g)
    bet = 0.1 * torch.randn(4096, device=dev, generator=g)
    nbytes = 2 * x.numel() * 4
    xh = x.double().cpu().numpy() if cpu else None
    gh, bh = gam.double().cpu().numpy(), bet.double().cpu().numpy()
    from oracle import rowops as OR

    for name, fn, cfn in (("row_softmax", lambda: kernels.row_softmax(x, out=y), lambda: OR.softmax(xh)),
                          ("layernorm", lambda: kernels.layernorm(x, gam, bet, 1e-5, out=y),
                           lambda: OR.layernorm(xh, gh, bh, eps=1e-5))):
        ms, per = _timed(fn, 50, 5, stream, 1)
        gbs = nbytes / (sum(per) / len(per) * 1e-3) / 1e9
        out[name] = {"GB/s": gbs, "frac_hbm": gbs / peaks["hbm_gbs"], "peak_source": peaks["source"] + " copy",
                     "us_per_call": 1e3 * sum(per) / len(per),
                     "bytes_per_call": nbytes, "config": "X 8192x4096 f32 (config 2)"}
        if cpu:  # the reference's numpy denotation of the whole config on the host cores
            sec, n = _cpu_seconds(cfn, 3.0)
            out[name]["cpu_baseline"] = {"GB/s": nbytes / sec / 1e9, "seconds_per_call": sec, "calls": n,
                                         "cores": _cpu_threads(), "kind": "port",
                                         "sample": "the whole 8192 x 4096 config, numpy f64"}


def _gqa(out, kernels, dev, stream, g, peaks=None, cpu=True):
    import torch

    # config 4: GQA fwd, B4 Hq64 Hkv8 S8192 D128 causal
    Bq, Hq, Hk, Sq = 4, 64, 8, 8192
    q = torch.randn((Bq, Hq, Sq, D), device=dev, generator=g).to(torch.bfloat16)
    k = torch.randn((Bq, Hk, Sq, D), device=dev, generator=g).to(torch.bfloat16)
    v = torch.randn((Bq, Hk, Sq, D), device=dev, generator=g).to(torch.bfloat16)
    o = torch.empty_like(q)
    ms, per = _timed(lambda: kernels.flash_attention(q, k, v, causal=True, out=o), 5, 2, stream, 1)
    fl = 4.0 * Bq * Hq * Sq * Sq * D / 2
    tf = fl / (sum(per) / len(per) * 1e-3) / 1e12
    out["gqa_fwd"] = {"TFLOP/s": tf, "ms": sum(per) / len(per),
                      "config": "B4 Hq64 Hkv8 S8192 D128 causal (config 4)"}
    if peaks:
        out["gqa_fwd"]["roofline"] = {"bound": "tensor", "frac": tf / peaks["bf16_tflops"],
                                      "peak": peaks["bf16_tflops"], "peak_source": peaks["source"] + " (burst)"}
    if cpu:
        from oracle import attention as OA

        qh = q[0, 0].double().cpu().numpy()
        kh, vh = k[0, 0].double().cpu().numpy(), v[0, 0].double().cpu().numpy()
        sec, n = _cpu_seconds(lambda: OA.attention_fwd(qh, kh, vh, scale=1 / math.sqrt(D), causal=True,
                                                       row_block=1024), 5.0)
        out["gqa_fwd"]["cpu_baseline"] = {"TFLOP/s": 4.0 * Sq * Sq * D / 2 / sec / 1e12, "cores": _cpu_threads(),
                                          "kind": "port", "sample": f"{n} causal query head(s) of 8192 x 8192, "
                                                                    "D=128, numpy f64"}


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


def _bwd(out, kernels, dev, stream, g, peaks=None, cpu=True):
    """Config 5 (B4 H16 S2048 D64 causal) and the same job at D=128."""
    import torch

    for name, Db in (("flash_bwd", 64), ("flash_bwd_d128", 128)):
        Bb, Hb, Sb = 4, 16, 2048
        q, k, v, do = (torch.randn((Bb, Hb, Sb, Db), device=dev, generator=g).to(torch.bfloat16) for _ in range(4))
        try:
            o, lse = kernels.flash_attention(q, k, v, causal=True, return_lse=True)
            ms, per = _timed(lambda: kernels.flash_attention_backward(q, k, v, o, do, lse, causal=True), 20, 3,
                             stream, 1)
            fl = 2.5 * 4.0 * Bb * Hb * Sb * Sb * Db / 2
            tf = fl / (sum(per) / len(per) * 1e-3) / 1e12
            out[name] = {"TFLOP/s": tf, "ms": sum(per) / len(per),
                         "config": f"B4 H16 S2048 D{Db} causal ({'config 5' if Db == 64 else 'config 5 at D=128'}), "
                                   "2.5x fwd FLOP convention"}
            if peaks:
                out[name]["roofline"] = {"bound": "tensor", "frac": tf / peaks["bf16_tflops"],
                                         "peak": peaks["bf16_tflops"], "peak_source": peaks["source"] + " (burst)"}
            try:  # the same backward through torch's SDPA (its fused backward kernels), as a labelled bar
                import math

                import torch.nn.functional as F

                qg, kg, vg = (x.detach().requires_grad_() for x in (q, k, v))
                og = F.scaled_dot_product_attention(qg, kg, vg, is_causal=True, scale=1 / math.sqrt(Db))
                _, per_b = _timed(lambda: torch.autograd.grad(og, (qg, kg, vg), do, retain_graph=True), 20, 3,
                                  stream, 1)
                tf_b = fl / (sum(per_b) / len(per_b) * 1e-3) / 1e12
                out[name]["bar_torch_sdpa_bwd"] = {
                    "TFLOP/s": tf_b, "ours_over_bar": tf / tf_b,
                    "call": "torch.autograd.grad of F.scaled_dot_product_attention(is_causal=True), bf16"}
                del qg, kg, vg, og
            except Exception as e:
                out[name]["bar_torch_sdpa_bwd"] = {"error": str(e)[:200]}
            if cpu and Db == 64:
                from oracle import attention as OA

                hs = [x[0, 0].double().cpu().numpy() for x in (q, k, v, do)]
                sec, n = _cpu_seconds(lambda: OA.attention_bwd(*hs, scale=1 / 8, causal=True), 3.0)
                out[name]["cpu_baseline"] = {"TFLOP/s": 2.5 * 4.0 * Sb * Sb * Db / 2 / sec / 1e12,
                                             "cores": _cpu_threads(), "kind": "port",
                                             "sample": f"{n} causal head(s) of 2048 x 2048, D=64, numpy f64 "
                                                       "(closed-form adjoint)"}
        except Exception as e:  # the backward is reported, not required, for the headline line
            out[name] = {"error": str(e)[:200]}
        del q, k, v, do


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--scaling", choices=("weak", "strong"), default="strong")
    ap.add_argument("--no-bars", action="store_true", help="skip the SDPA / reference-Triton bars")
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
