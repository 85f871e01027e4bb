"""Generate the golden fixtures with the REFERENCE's own evaluator.

Run in an environment where the reference DSL is importable (a shimmed copy
made by ``python oracle/make_ref_shim.py``):

    python tests/golden/make_golden.py

Every case builds an ordinary DSL Region (``pdum_dsl_b200.regions`` spells
them as the reference zoo does, or the zoo makers themselves), draws inputs
with ``np.random.default_rng(seed).standard_normal``, rounds them to the
device dtype (f32 or bf16, so the device kernels and the evaluator see the
same values), evaluates with ``pdum.tl.dialect.run_region``
(dialect.py:1349) in f64, and stores seeds + outputs in ``<case>.npz``.
Inputs are regenerated from the seeds by ``tests/golden/__init__.py``; a
checksum of each input is stored to prove the regeneration.
"""

from __future__ import annotations

import json
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))

from oracle.make_ref_shim import ensure_importable  # noqa: E402
from tests.golden import draw, input_checksum  # noqa: E402


def _run(region, arrays, names_list):
    from pdum.tl.dialect import run_region
    from pdum.tl.tensor import Tensor

    vals = [Tensor.from_numpy(a, n) for a, n in zip(arrays, names_list)]
    out = run_region(region, vals)
    outs = out if isinstance(out, tuple) else (out,)
    return [o.to_numpy(order=o.names) if hasattr(o, "names") else np.asarray(o) for o in outs], [
        tuple(o.names) if hasattr(o, "names") else () for o in outs
    ]


def _param_names(region):
    return [tuple(d.name for d in p.type.dims) for p in region.params]


def _param_shapes(region):
    return [tuple(d.stop - d.start for d in p.type.dims) for p in region.params]


def save(case, *, region_kw, inputs_spec, outputs, out_names, meta=None):
    arrays = {f"out{i}": o for i, o in enumerate(outputs)}
    spec = {"region": region_kw, "inputs": inputs_spec, "out_names": out_names, **(meta or {})}
    np.savez_compressed(HERE / f"{case}.npz", spec=np.array(json.dumps(spec)), **arrays)
    print(f"{case}: {[o.shape for o in outputs]}", flush=True)


def attention_case(case, *, dtype, seeds, **kw):
    from pdum_dsl_b200.regions import attention_region

    region = attention_region(**kw)
    shapes, names = _param_shapes(region), _param_names(region)
    arrays = [draw(seed, shp, dtype) for seed, shp in zip(seeds, shapes)]
    t0 = time.time()
    outs, onames = _run(region, arrays, names)
    spec = [{"seed": s, "shape": list(shp), "names": list(n), "dtype": dtype, "scale": 1.0,
             "checksum": input_checksum(a)} for s, shp, n, a in zip(seeds, shapes, names, arrays)]
    save(case, region_kw=kw, inputs_spec=spec, outputs=outs, out_names=[list(n) for n in onames],
         meta={"run_region_s": round(time.time() - t0, 3)})


def masked_case(case, *, dtype, seeds, zoo_sliding=None, **kw):
    """General closed masks: the reference zoo's sliding_attention (zoo/attention.py:84-103)
    or a region spelled with a window / block mask."""
    from pdum_dsl_b200.regions import attention_region

    if zoo_sliding is not None:
        from pdum.tl.zoo.attention import sliding_attention

        region = sliding_attention(**zoo_sliding).region
        rkw = {"zoo": "sliding_attention", **zoo_sliding}
    else:
        region = attention_region(**kw)
        rkw = kw
    shapes, names = _param_shapes(region), _param_names(region)
    arrays = [draw(seed, shp, dtype) for seed, shp in zip(seeds, shapes)]
    t0 = time.time()
    outs, onames = _run(region, arrays, names)
    spec = [{"seed": s, "shape": list(shp), "names": list(n), "dtype": dtype, "scale": 1.0,
             "checksum": input_checksum(a)} for s, shp, n, a in zip(seeds, shapes, names, arrays)]
    save(case, region_kw=rkw, inputs_spec=spec, outputs=outs, out_names=[list(n) for n in onames],
         meta={"run_region_s": round(time.time() - t0, 3)})


def mask_cases():
    masked_case("sliding_zoo_f32", dtype="f32", seeds=(601, 602, 603),
                zoo_sliding=dict(T=300, E=64, OD=64, W=70))
    masked_case("sliding_zoo_bf16", dtype="bf16", seeds=(604, 605, 606),
                zoo_sliding=dict(T=384, E=64, OD=64, W=130))
    masked_case("sliding_bf16_riders", dtype="bf16", seeds=(611, 612, 613), B=1, H=2, T=300, D=128,
                causal=True, window=100, scale=1 / np.sqrt(128))
    masked_case("block_bf16_d128", dtype="bf16", seeds=(621, 622, 623), H=2, T=384, D=128, causal=False,
                block=128, scale=1 / np.sqrt(128))
    masked_case("block_causal_f32", dtype="f32", seeds=(631, 632, 633), T=200, D=32, causal=True, block=50,
                scale=0.2)


def row_case(case, kind, R, C, dtype, seeds, eps=1e-5):
    from pdum_dsl_b200.regions import layernorm_region, row_softmax_region

    if kind == "softmax":
        region = row_softmax_region(R, C)
        specs = [(seeds[0], (R, C), ("r", "c"), 1.0, 0.0)]
    else:
        region = layernorm_region(R, C, eps)
        specs = [(seeds[0], (R, C), ("r", "c"), 1.0, 0.0), (seeds[1], (C,), ("c",), 0.1, 1.0),
                 (seeds[2], (C,), ("c",), 0.1, 0.0)]
    arrays = [draw(s, shp, dtype, scale=sc, shift=sh) for s, shp, _, sc, sh in specs]
    outs, onames = _run(region, arrays, [n for _, _, n, _, _ in specs])
    spec = [{"seed": s, "shape": list(shp), "names": list(n), "dtype": dtype, "scale": sc, "shift": sh,
             "checksum": input_checksum(a)} for (s, shp, n, sc, sh), a in zip(specs, arrays)]
    save(case, region_kw={"kind": kind, "R": R, "C": C, "eps": eps}, inputs_spec=spec, outputs=outs,
         out_names=[list(n) for n in onames])


def flash_tile_case():
    """The reference's own tile flagship (zoo/tiles.py:143) and its planned kernel."""
    from pdum.tl.dialect import run_region
    from pdum.tl.fusion import plan_region
    from pdum.tl.zoo.tiles import flash_tile

    f = flash_tile()
    (g,) = plan_region(f.naive).groups
    vals = list(f.inputs.values())
    naive = run_region(f.naive, vals)
    tile = run_region(g.kernel, vals)
    ins = {k: v.to_numpy() for k, v in f.inputs.items()}
    np.savez_compressed(HERE / "flash_tile_default.npz", q=ins["q"], k=ins["k"], v=ins["v"],
                        naive=naive.to_numpy(order=("t", "o")), tile=tile.to_numpy(order=("t", "o")),
                        oracle=f.oracle(f.numpy_inputs()))
    print("flash_tile_default", flush=True)


def joint_case(case, T, E, OD, seed):
    """autodiff.grad of the naive flash region (the test_partition.py:124-193 joint)."""
    from pdum.tl.autodiff import grad
    from pdum.tl.zoo.tiles import flash_tile

    f = flash_tile(T=T, E=E, OD=OD, SI=2)
    out = f.naive.body[-1].args[0]
    names = {id(p): f"p{i}" for i, p in enumerate(f.naive.params)}
    names[id(out)] = "out"
    rg = grad(f.naive, "out", seed="dO", names=names)
    shapes, pnames = _param_shapes(rg.region), _param_names(rg.region)
    # q is drawn at 1/sqrt(E) so the unscaled region's scores have unit variance (the regime of the
    # scaled configs); the region itself is the reference's, unchanged
    scales = [1.0 / np.sqrt(E) if i == 0 else 1.0 for i in range(len(shapes))]
    arrays = [draw(seed + i, shp, "bf16", scale=sc) for i, (shp, sc) in enumerate(zip(shapes, scales))]
    outs, onames = _run(rg.region, arrays, pnames)
    spec = [{"seed": seed + i, "shape": list(shp), "names": list(n), "dtype": "bf16", "scale": sc,
             "checksum": input_checksum(a)} for i, (shp, n, a, sc) in enumerate(zip(shapes, pnames, arrays, scales))]
    save(case, region_kw={"T": T, "E": E, "OD": OD, "causal": True, "scale": None}, inputs_spec=spec,
         outputs=outs, out_names=[list(n) for n in onames], meta={"outputs": list(rg.outputs)})


def main():
    if not ensure_importable():
        raise SystemExit("reference DSL not importable: run `python oracle/make_ref_shim.py` first")
    if "--masks-only" in sys.argv:  # just the general-mask cases
        mask_cases()
        return
    flash_tile_case()
    attention_case("cfg1_flash_f32", dtype="f32", seeds=(101, 102, 103), B=1, H=4, T=256, D=64,
                   causal=False, scale=1 / 8)
    attention_case("causal_bf16_ragged", dtype="bf16", seeds=(201, 202, 203), B=1, H=2, T=200, D=64,
                   causal=True, scale=1 / 8, artifacts=True)
    attention_case("causal_bf16_d128", dtype="bf16", seeds=(211, 212, 213), B=1, H=1, T=384, D=128,
                   causal=True, scale=1 / np.sqrt(128))
    attention_case("noncausal_bf16_kv_ragged", dtype="bf16", seeds=(221, 222, 223), B=2, H=1, T=130, S=300,
                   D=64, causal=False, scale=0.125)
    attention_case("gqa_bf16", dtype="bf16", seeds=(301, 302, 303), B=1, H=2, T=130, D=64, causal=True,
                   scale=1 / 8, group=2)
    attention_case("causal_f32_small", dtype="f32", seeds=(311, 312, 313), T=40, D=24, causal=True,
                   scale=None)
    row_case("rowsoftmax_16x4096", "softmax", 16, 4096, "f32", (401,))
    row_case("rowsoftmax_37x1001", "softmax", 37, 1001, "f32", (402,))
    row_case("layernorm_16x4096", "layernorm", 16, 4096, "f32", (411, 412, 413))
    row_case("layernorm_37x1001", "layernorm", 37, 1001, "f32", (414, 415, 416))
    joint_case("flash_joint_bwd", T=64, E=16, OD=16, seed=501)
    joint_case("flash_joint_bwd_d64", T=200, E=64, OD=64, seed=511)
    mask_cases()


if __name__ == "__main__":
    main()
