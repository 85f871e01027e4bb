"""Single-kernel workloads for profiling (ncu) and quick timing.

    python -m pdum_dsl_b200.profile_cases CASE [--reps N]

Each case sets up device inputs once, runs its kernel ``reps`` times (default
3) and synchronises, so ``ncu -k regex:<kernel> -s <warm-up launches> -c <n>``
can capture one launch of a known workload.  Inputs exceed the 126 MB L2
where the kernel streams from HBM, so DRAM counters mean something; every
case stays within a few GB of device memory.  The printed line gives the
CUDA-event time per launch (not to be read under a profiler).
"""

from __future__ import annotations

import argparse
import json
import math
import sys


def _time(fn, reps):
    import torch

    fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps


def case_fwd(B, H, S, D, causal=True):
    import torch

    from . import kernels

    g = torch.Generator(device="cuda").manual_seed(0)
    q, k, v = (torch.randn((B, H, S, D), device="cuda", generator=g).to(torch.bfloat16) for _ in range(3))
    o = torch.empty_like(q)
    flop = 4.0 * B * H * S * S * D / (2 if causal else 1)
    return (lambda: kernels.flash_attention(q, k, v, causal=causal, out=o)), {"TFLOP": flop / 1e12}


def case_bwd(B, H, S, D):
    import torch

    from . import kernels

    g = torch.Generator(device="cuda").manual_seed(0)
    q, k, v, do = (torch.randn((B, H, S, D), device="cuda", generator=g).to(torch.bfloat16) for _ in range(4))
    o, lse = kernels.flash_attention(q, k, v, causal=True, return_lse=True)
    flop = 2.5 * 4.0 * B * H * S * S * D / 2
    return (lambda: kernels.flash_attention_backward(q, k, v, o, do, lse, causal=True)), {"TFLOP": flop / 1e12}


def case_f32_flash():
    import torch

    from . import kernels

    g = torch.Generator(device="cuda").manual_seed(0)
    q, k, v = (torch.randn((1, 4, 256, 64), device="cuda", generator=g) for _ in range(3))
    return (lambda: kernels.flash_attention(q, k, v, scale=0.125, causal=False)), {"TFLOP": 4.0 * 4 * 256 * 256 * 64 / 1e12}


def case_contract_single(M=128, N=8192, K=8192):
    import torch

    from . import kernels

    g = torch.Generator(device="cuda").manual_seed(0)
    a = torch.randn((1, M, K), device="cuda", generator=g).to(torch.bfloat16)
    b = torch.randn((1, N, K), device="cuda", generator=g).to(torch.bfloat16)
    c = torch.empty((1, M, N), dtype=torch.bfloat16, device="cuda")
    return (lambda: kernels.contract(a, b, out=c)), {"TFLOP": 2.0 * M * N * K / 1e12,
                                                    "bytes": 2 * (M * K + N * K + M * N)}


def case_pointwise(n=8192):
    import torch

    from . import kernels

    x = torch.randn((1, n, n), device="cuda")
    y = torch.empty_like(x)
    prog = [("mul", 0.5, False), ("exp", None, False), ("add", 1.0, False)]
    return (lambda: kernels.pointwise(x, prog, out=y)), {"bytes": 8 * n * n}


def case_rows(kind):
    """Config 2: X 8192 x 4096 f32 (gamma / beta for the layernorm)."""
    import torch

    from . import kernels

    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn((8192, 4096), device="cuda", generator=g)
    y = torch.empty_like(x)
    gam = 1 + 0.1 * torch.randn(4096, device="cuda", generator=g)
    bet = 0.1 * torch.randn(4096, device="cuda", generator=g)
    if kind == "softmax":
        return (lambda: kernels.row_softmax(x, out=y)), {"bytes": 2 * x.numel() * 4}
    return (lambda: kernels.layernorm(x, gam, bet, 1e-5, out=y)), {"bytes": 2 * x.numel() * 4}


def case_score_program(T=2048, E=64):
    """The den-gradient carve of the attention joint (a row-sum score program)."""
    import torch

    try:
        from pdum.tl.autodiff import grad
    except ImportError:
        raise SystemExit("score_program needs the reference DSL (pdum.dsl / pdum.tl) importable") from None
    from pdum.tl.partition import plan_model
    from pdum.tl.zoo.tiles import flash_tile

    from .score_program import ScoreProgramSpec
    from .tile import compile_tile

    f = flash_tile(T=T, E=E, OD=E, SI=32)
    out = f.naive.body[-1].args[0]
    names = {id(p): f"p{i}" for i, p in enumerate(f.naive.params)}
    names[id(out)] = "out"
    plan = plan_model(grad(f.naive, "out", seed="dO", names=names).region)
    for c in plan.carves:
        if c.root is None or c.group.kernel is not None and c.group.template == "flash":
            continue
        try:
            run = compile_tile(c.kernel)
        except Exception:
            continue
        if isinstance(run.spec, ScoreProgramSpec) and run.spec.passes[0].mode == "row_sum":
            break
    else:
        raise SystemExit("no row-sum score program among the carves")
    g = torch.Generator(device="cuda").manual_seed(0)
    ins = [torch.randn(tuple(d.stop - d.start for d in p.type.dims), device="cuda", generator=g)
           for p in c.kernel.params]
    return (lambda: run.run_t(*ins)), {"source": run.source}


CASES = {
    "fwd_config3": lambda: case_fwd(8, 32, 4096, 128),
    "fwd_b2": lambda: case_fwd(2, 32, 4096, 128),
    "fwd_d64": lambda: case_fwd(8, 32, 4096, 64),
    "fwd_d64_b4": lambda: case_fwd(4, 32, 4096, 64),
    "fwd_d256": lambda: case_fwd(2, 16, 4096, 256),
    "bwd_config5": lambda: case_bwd(4, 16, 2048, 64),
    "bwd_d128": lambda: case_bwd(4, 16, 2048, 128),
    "f32_flash_config1": case_f32_flash,
    "contract_single": case_contract_single,
    "pointwise": case_pointwise,
    "score_program": case_score_program,
    "rowsoftmax_config2": lambda: case_rows("softmax"),
    "layernorm_config2": lambda: case_rows("layernorm"),
}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=sorted(CASES))
    ap.add_argument("--reps", type=int, default=3)
    a = ap.parse_args(argv)
    import torch  # noqa: F401

    from ._lib import load

    load()
    fn, meta = CASES[a.case]()
    ms = _time(fn, a.reps)
    rec = {"case": a.case, "ms": ms, **meta}
    if "TFLOP" in meta:
        rec["TFLOP/s"] = meta["TFLOP"] / (ms * 1e-3)
    if "bytes" in meta:
        rec["GB/s"] = meta["bytes"] / (ms * 1e-3) / 1e9
    print(json.dumps(rec), flush=True)


if __name__ == "__main__":
    sys.exit(main())
