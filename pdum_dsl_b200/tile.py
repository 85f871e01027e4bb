"""``compile_tile``: the reference lowering's call convention, on sm_100a kernels.

Mirrors ``conformance/triton_tile.py:662-698``:

    run = compile_tile(region, launch=(), prune=())
    out = run(values)            # values: numpy arrays, positional per region param,
                                 # each in its param's type-dim order
    run.source, run.grid         # what runs, and how many programs (CTAs) it launches

``region`` is a plan group's ``kernel`` (the tile region the reference's
fusion templates emit) or the naive region itself; ``recognize`` decides
which fixed kernel of ``libpdb_sm100.so`` executes it.  Outputs are
allocated by the runner (destination passing), returned as float32 numpy
arrays in the yield's dim order -- a tuple ``(out, m, den)`` for the flash
artifact variant, as the reference returns.  ``run`` synchronises.

Differences from the Triton column, by design:
* nothing is generated or JIT-compiled -- the kernels are prebuilt sm_100a;
* ``dtype="bf16"`` runs the tcgen05 tensor-core path (bf16 operands, fp32
  accumulate); the default ``"f32"`` is the IEEE CUDA-core path, matching the
  reference column's refusal of tf32 (triton_tile.py:684-690);
* ``run_t(*tensors)`` is the zero-copy device-tensor path (no host copies);
* unsupported regions raise ``Untranslatable`` at compile time -- there is no
  fallback to the reference evaluator or to any other backend.
"""

from __future__ import annotations

import math

import numpy as np

from .recognize import AttentionSpec, ContractSpec, MapSpec, RowSpec, Untranslatable, recognize
from .score_program import ScoreProgramSpec, match_score_program, run_score_program

# the executor fingerprint (the reference's Pair seat is keyed the same way, triton_tile.py:54)
B200_FP = ("tile_sm100a", "pdb")


def _prod(xs):
    return math.prod(xs) if xs else 1


def _run_contract(spec: ContractSpec, tensors, dtype):
    """Device tensors -> c in the yield's dim order, through pdb_contract."""
    import torch

    from . import kernels

    def sizes(t, dims, names):
        return [t.shape[dims.index(n)] for n in names]

    def operand(t, pro, dims, kept):
        t = t.float() if t.dtype != torch.float32 else t
        if pro:  # unary prologue chain, materialised once by the map-chain kernel
            flat = kernels.pointwise(t.contiguous().reshape(1, 1, -1), [(f, None, False) for f in pro])
            t = flat.reshape(t.shape)
        v = t.permute(*[dims.index(n) for n in spec.batch + kept + spec.k])
        return v.reshape(_prod(sizes(t, dims, spec.batch)), _prod(sizes(t, dims, kept)),
                         _prod(sizes(t, dims, spec.k)))

    a, b = tensors[spec.a], tensors[spec.b]
    A = operand(a, spec.a_pro, spec.a_dims, spec.m)
    Bm = operand(b, spec.b_pro, spec.b_dims, spec.n)
    if dtype == "bf16":
        A, Bm = A.to(torch.bfloat16).contiguous(), Bm.to(torch.bfloat16).contiguous()
    bs = sizes(a, spec.a_dims, spec.batch)
    ms = sizes(a, spec.a_dims, spec.m)
    ns = sizes(b, spec.b_dims, spec.n)
    full_names = spec.batch + spec.m + spec.n
    full = bs + ms + ns
    epi = []
    for f, leaf, swap in spec.epilogue:
        if leaf is None:
            epi.append((f, None, False))
        elif leaf.param is None:
            epi.append((f, leaf.const, swap))
        else:
            t = tensors[leaf.param].float()
            v = t.permute(*[leaf.dims.index(n) for n in full_names if n in leaf.dims])
            shape = [full[i] if n in leaf.dims else 1 for i, n in enumerate(full_names)]
            v = v.reshape(shape).expand(full).reshape(A.shape[0], A.shape[1], Bm.shape[1])
            epi.append((f, v, swap))
    alpha = 1.0 / _prod(sizes(a, spec.a_dims, spec.k)) if spec.mean else 1.0
    c = kernels.contract(A, Bm, epilogue=epi, alpha=alpha)
    c = c.reshape(full)
    return c.permute(*[full_names.index(n) for n in spec.out_dims])


def _run_map(spec: MapSpec, tensors):
    """Device tensors -> the chain's output in the yield's dim order (pdb_pointwise_f32)."""
    from . import kernels

    x = tensors[spec.x].float().permute(*[spec.x_dims.index(n) for n in spec.out_dims])
    full = list(x.shape)
    flat = x.reshape(1, 1, -1)
    prog = []
    for f, leaf, swap in spec.steps:
        if leaf is None:
            prog.append((f, None, False))
        elif leaf.param is None:
            prog.append((f, leaf.const, swap))
        else:
            t = tensors[leaf.param].float()
            v = t.permute(*[leaf.dims.index(n) for n in spec.out_dims if n in leaf.dims])
            v = v.reshape([full[i] if n in leaf.dims else 1 for i, n in enumerate(spec.out_dims)]).expand(full)
            prog.append((f, v.reshape(1, 1, -1), swap))
    return kernels.pointwise(flat, prog).reshape(full)


def _check_launch(spec, launch, prune, region):
    """launch: (output dim, tile) pairs (launch.py:95); prune: (scan dim, lo, hi) affine
    bounds (fusion.py:659-690).  The kernels tile internally (128/256-row programs) and
    visit only live key tiles, so these artifacts are validated and recorded, not obeyed."""
    out_dims = spec.out_dims
    if isinstance(spec, AttentionSpec):
        carried = {spec.s, spec.e}
    elif isinstance(spec, MapSpec):
        carried = set()
    elif isinstance(spec, ScoreProgramSpec):
        carried = {ps.cols for ps in spec.passes if ps.mode != "tile"}
    elif isinstance(spec, ContractSpec):
        carried = set(spec.k)
    else:
        carried = {spec.dim}
    for name, tile in launch:
        if name not in out_dims:
            raise Untranslatable(f"launch dim {name!r} is not an output dim")
        if name in carried:
            raise Untranslatable(f"launch dim {name!r} is carried/reduced -- not griddable")
        if int(tile) <= 0:
            raise Untranslatable(f"launch tile for {name!r} must be positive")
    for entry in prune:
        if not isinstance(spec, AttentionSpec) or not (spec.causal or spec.mask is not None):
            raise Untranslatable("prune bounds only apply to a masked flash template")
        if entry[0] != "so":
            raise Untranslatable(f"prune dim {entry[0]!r} is not the flash scan dim")


def _extent(region, i, name):
    d = next(d for d in region.params[i].type.dims if d.name == name)
    return d.stop - d.start


class _Runner:
    def __init__(self, region, spec, dtype, launch, prune):
        self.region, self.spec, self.dtype = region, spec, dtype
        self.launch, self.prune = tuple(launch), tuple(prune)
        self.checked = False
        if isinstance(spec, AttentionSpec):
            T = _extent(region, spec.q, spec.t)
            heads = 1
            for n in spec.riders:
                heads *= _extent(region, spec.k, n)
            if spec.group:
                heads *= _extent(region, spec.q, spec.group)
            rows = 256 if dtype == "bf16" else 64
            self.grid = heads * -(-T // rows)
            self.source = (f"pdb_flash_fwd dtype={dtype} causal={spec.causal} mask={spec.mask} scale={spec.scale} "
                           f"riders={spec.riders} group={spec.group} artifacts={spec.artifacts} "
                           f"kernel={'flash_fwd_sm100_kernel (tcgen05/TMEM, TMA)' if dtype == 'bf16' else 'flash_f32_kernel (IEEE FMA)'}")
        elif isinstance(spec, MapSpec):
            n = _prod([d.stop - d.start for d in region.params[spec.x].type.dims])
            self.grid = -(-n // 256)
            self.source = f"pdb_pointwise_f32 steps={[e[0] for e in spec.steps]}"
        elif isinstance(spec, ContractSpec):
            def ext(i, names):
                return _prod([next(d.stop - d.start for d in region.params[i].type.dims if d.name == n)
                              for n in names])
            Bt, M, N = ext(spec.a, spec.batch), ext(spec.a, spec.m), ext(spec.b, spec.n)
            if dtype == "bf16":
                self.grid = Bt * -(-M // 128) * -(-N // 128)
                kern = "contract_bf16_kernel (tcgen05/TMEM, TMA)"
            else:
                self.grid = Bt * -(-M // 64) * -(-N // 64)
                kern = "contract_f32_kernel (IEEE FMA)"
            self.source = (f"pdb_contract dtype={dtype} batch={spec.batch} m={spec.m} n={spec.n} k={spec.k} "
                           f"prologue=({spec.a_pro}, {spec.b_pro}) epilogue={[e[0] for e in spec.epilogue]} "
                           f"kernel={kern}")
        elif isinstance(spec, ScoreProgramSpec):
            self.grid = sum(-(-(spec.extents[ps.rows][1] - spec.extents[ps.rows][0]) // 64) for ps in spec.passes)
            self.source = spec.source
        else:
            R = 1
            for d in region.params[spec.x].type.dims:
                if d.name != spec.dim:
                    R *= d.stop - d.start
            self.grid = R
            self.source = f"pdb_{'rowsoftmax' if spec.kind == 'softmax' else 'layernorm'}_f32 dim={spec.dim}"

    # ---------------------------------------------------------------- device path
    def run_t(self, *tensors, out=None):
        """Device tensors (CUDA, in param type-dim order) -> device tensor(s), no copies."""
        from . import kernels

        spec = self.spec
        if isinstance(spec, ContractSpec):
            return _run_contract(spec, tensors, self.dtype)
        if isinstance(spec, MapSpec):
            return _run_map(spec, tensors)
        if isinstance(spec, ScoreProgramSpec):
            return run_score_program(spec, tensors)
        if isinstance(spec, RowSpec):
            x = tensors[spec.x]
            perm = [spec.x_dims.index(n) for n in spec.x_dims if n != spec.dim] + [spec.x_dims.index(spec.dim)]
            xv = x.permute(*perm)
            lead = xv.shape[:-1]
            x2 = xv.reshape(-1, xv.shape[-1])
            if spec.kind == "softmax":
                y = kernels.row_softmax(x2)
            else:
                g = tensors[spec.gamma] if spec.gamma is not None else None
                b = tensors[spec.beta] if spec.beta is not None else None
                y = kernels.layernorm(x2, g, b, eps=spec.eps)
            ynames = tuple(n for n in spec.x_dims if n != spec.dim) + (spec.dim,)
            y = y.view(*lead, y.shape[-1])
            return y.permute(*[ynames.index(n) for n in spec.out_dims])
        return self._attention(tensors)

    def _attention(self, tensors):
        import torch

        from . import kernels

        spec = self.spec
        q, k, v = tensors[spec.q], tensors[spec.k], tensors[spec.v]
        rid = list(spec.riders)
        qg = [spec.group] if spec.group else []
        qv = q.permute(*[spec.q_dims.index(n) for n in rid + qg + [spec.t, spec.e]])
        kv = k.permute(*[spec.k_dims.index(n) for n in rid + [spec.s, spec.e]])
        vv = v.permute(*[spec.v_dims.index(n) for n in rid + [spec.s, spec.o]])
        lead = list(kv.shape[:-2])
        while len(lead) < 2:  # (batch, heads) with missing riders as 1
            lead.insert(0, 1)
        Bn, HK = lead[0], lead[1]
        G = qv.shape[len(rid)] if spec.group else 1
        T, D = qv.shape[-2], qv.shape[-1]
        S, DV = vv.shape[-2], vv.shape[-1]
        q4 = qv.reshape(Bn, HK * G, T, D)
        k4 = kv.reshape(Bn, HK, S, D)
        v4 = vv.reshape(Bn, HK, S, DV)
        dt = torch.bfloat16 if self.dtype == "bf16" else torch.float32
        q4, k4, v4 = (x if x.dtype == dt else x.to(dt) for x in (q4, k4, v4))
        scale = 1.0 if spec.scale is None else spec.scale
        res = kernels.flash_attention(q4, k4, v4, scale=scale, causal=spec.causal, q_start=spec.t_start,
                                      return_artifacts=spec.artifacts, key_intervals=spec.mask)
        o = res[0] if spec.artifacts else res
        # back to the yield's dim order: (riders..., [group], t, o)
        onames = tuple(rid + qg + [spec.t, spec.o])
        o = o.reshape(*qv.shape[:-2], T, DV)
        o = o.permute(*[onames.index(n) for n in spec.out_dims])
        if not spec.artifacts:
            return o
        snames = tuple(rid + qg + [spec.t])
        stats = []
        for st in res[1:3]:
            st = st.reshape(*qv.shape[:-2], T)
            stats.append(st.permute(*[snames.index(n) for n in spec.stat_dims]))
        return (o, *stats)

    # ------------------------------------------------------------------ host path
    def _attention_host(self, values, out):
        """Attention on host values through the pipelined host entry point: the
        (batch, KV-head) units are chunked so host-to-device copies, the kernel and
        device-to-host copies overlap (host.flash_attention_host)."""
        import torch

        from .host import flash_attention_host

        spec = self.spec
        rid = list(spec.riders)
        qg = [spec.group] if spec.group else []
        ts = [v if isinstance(v, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(v)) for v in values]
        q = ts[spec.q].permute(*[spec.q_dims.index(n) for n in rid + qg + [spec.t, spec.e]])
        k = ts[spec.k].permute(*[spec.k_dims.index(n) for n in rid + [spec.s, spec.e]])
        v = ts[spec.v].permute(*[spec.v_dims.index(n) for n in rid + [spec.s, spec.o]])
        lead = list(k.shape[:-2])
        while len(lead) < 2:
            lead.insert(0, 1)
        Bn, HK = lead
        G = q.shape[len(rid)] if spec.group else 1
        T, D = q.shape[-2:]
        S, DV = v.shape[-2:]
        q4 = q.reshape(Bn, HK * G, T, D).contiguous()
        k4 = k.reshape(Bn, HK, S, D).contiguous()
        v4 = v.reshape(Bn, HK, S, DV).contiguous()
        onames = tuple(rid + qg + [spec.t, spec.o])
        perm = [onames.index(n) for n in spec.out_dims]
        oshape = tuple(list(q.shape[:-2]) + [T, DV])
        if out is None:
            o4 = torch.empty((Bn, HK * G, T, DV), dtype=q4.dtype)
        else:  # the caller's host buffer, in the yield's dim order
            inv = [spec.out_dims.index(n) for n in onames]
            o4 = out.permute(*inv).reshape(Bn, HK * G, T, DV)
            if o4.data_ptr() != out.data_ptr() or not o4.is_contiguous():
                raise ValueError("out must be a contiguous host tensor in the yield's dim order")
        cdt = torch.bfloat16 if self.dtype == "bf16" else torch.float32
        flash_attention_host(q4, k4, v4, o4, scale=1.0 if spec.scale is None else spec.scale, causal=spec.causal,
                             compute_dtype=cdt, q_start=spec.t_start, key_intervals=spec.mask)
        if out is not None:
            return out
        return o4.reshape(oshape).permute(*perm).float().numpy()

    def __call__(self, values, out=None):
        """values: host arrays (numpy, or CPU torch tensors -- pinned for full copy
        speed), positional per region param in type-dim order.  ``out`` (optional,
        attention only) is a host tensor in the yield's dim order that receives
        the result instead of a freshly allocated array."""
        import torch

        if not torch.cuda.is_available():
            raise RuntimeError("compile_tile runners execute on a CUDA device (sm_100a); none is available")
        if isinstance(self.spec, AttentionSpec) and not self.spec.artifacts:
            res = self._attention_host(values, out)
            if not self.checked:
                from .kernels import check_device_errors

                check_device_errors()
                self.checked = True
            return res
        if out is not None:
            raise ValueError("out= is taken by the attention runner only")
        values = [v.numpy() if isinstance(v, torch.Tensor) else v for v in values]
        dt = torch.bfloat16 if self.dtype == "bf16" else torch.float32
        ins = []
        for i, v in enumerate(values):
            t = torch.as_tensor(np.ascontiguousarray(v), dtype=torch.float32).cuda()
            if isinstance(self.spec, AttentionSpec) and i in (self.spec.q, self.spec.k, self.spec.v):
                t = t.to(dt)
            ins.append(t)
        out = self.run_t(*ins)
        torch.cuda.synchronize()
        if not self.checked:  # bounded device waits report through the error flag
            from .kernels import check_device_errors

            check_device_errors()
            self.checked = True
        if isinstance(out, tuple):
            return tuple(o.float().cpu().numpy() for o in out)
        return out.float().cpu().numpy()


def compile_tile(region, launch: tuple = (), prune: tuple = (), *, dtype: str = "f32"):
    """Region -> runner over the prebuilt sm_100a kernels (see the module docstring)."""
    if dtype not in ("f32", "bf16"):
        raise ValueError("dtype must be 'f32' or 'bf16'")
    try:
        spec = recognize(region)
    except Untranslatable as first:
        try:
            spec = match_score_program(region)
        except Untranslatable as e:
            raise Untranslatable(f"{first}; score-space program: {e}") from None
    if isinstance(spec, ScoreProgramSpec) and dtype != "f32":
        raise Untranslatable("score-space programs are f32")
    if isinstance(spec, MapSpec) and dtype != "f32":
        raise Untranslatable("the map-chain kernel is f32")
    if isinstance(spec, RowSpec) and dtype != "f32":
        raise Untranslatable("row-reduction kernels are f32")
    if isinstance(spec, ContractSpec) and dtype == "bf16":
        kx = _prod([next(d.stop - d.start for d in region.params[spec.a].type.dims if d.name == n) for n in spec.k])
        if kx % 8:
            raise Untranslatable("bf16 contraction needs the contracted extent to be a multiple of 8 (16-byte rows)")
    if isinstance(spec, AttentionSpec) and dtype == "bf16":
        D = _extent(region, spec.q, spec.e)
        DV = _extent(region, spec.v, spec.o)
        if any(x % 8 or x > 256 for x in (D, DV)):
            raise Untranslatable(f"bf16 flash needs head dims that are multiples of 8 up to 256, got {D}, {DV} "
                                 "(rows of 16-byte multiples for the tensor maps)")
    if isinstance(spec, AttentionSpec) and (_extent(region, spec.q, spec.e) > 256 or
                                            _extent(region, spec.v, spec.o) > 256):
        raise Untranslatable("flash head dims above 256 are not built")
    _check_launch(spec, launch, prune, region)
    runner = _Runner(region, spec, dtype, launch, prune)

    def run(values, out=None):
        return runner(values, out=out)

    run.run_t = runner.run_t
    run.source = runner.source
    run.grid = runner.grid
    run.spec = spec
    run.checked = False
    return run


def flops(region) -> float:
    """Algorithmic FLOPs of an attention region (causal counted as half)."""
    spec = recognize(region)
    if not isinstance(spec, AttentionSpec):
        return 0.0
    T = _extent(region, spec.q, spec.t)
    S = _extent(region, spec.k, spec.s)
    D = _extent(region, spec.q, spec.e)
    DV = _extent(region, spec.v, spec.o)
    heads = math.prod(_extent(region, spec.k, n) for n in spec.riders)
    if spec.group:
        heads *= _extent(region, spec.q, spec.group)
    f = 2.0 * heads * T * S * (D + DV)
    if spec.mask is not None:  # the visible (row, key) pairs of a general closed mask
        return 2.0 * heads * float(np.sum(spec.mask.hi.astype(np.int64) - spec.mask.lo)) * (D + DV)
    return f / 2 if spec.causal else f
