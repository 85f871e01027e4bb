"""Lowering of the attention backward that the DSL's autodiff derives.

``autodiff.grad(region, "out", seed="dO", names=...)`` (``pdum/tl/autodiff.py:
102-150``) returns a ``RegionGrad`` whose joint region takes the forward's
params plus the seed ``dO`` (last) and yields ``(out, *grads)``; the
reference executes it carve by carve after ``plan_model`` (``pdum/tl/
partition.py:586-607``; ``packages/tensorlib/tests/test_partition.py:124-193``).
``compile_grad(rg)`` reads the joint's forward output as attention (the same
recogniser as ``compile_tile``) and runs the whole joint as one forward
(for the logsumexp) plus the fused backward of ``include/pdb.h``
(``pdb_flash_bwd``).  The grads are returned in the joint's yield order and
dim order (e.g. ``dv`` as ``(o, s)``, as the joint yields it).
"""

from __future__ import annotations

import numpy as np

from .recognize import AttentionSpec, Untranslatable, match_naive_attention, names_of

_WRAPS = ("tl.with_charts", "tl.strip_charts", "tl.simplify", "tl.with_labels", "tl.bind")


def _unwrap(n):
    while n.op in _WRAPS:
        n = n.args[0]
    return n


class _GradRunner:
    def __init__(self, rg, dtype):
        region = rg.region
        yld = region.body[-1].args[0]
        if yld.op != "core.tuple" or len(yld.args) < 2:
            raise Untranslatable("joint region does not yield (out, *grads)")
        if rg.outputs[0] != "out" and len(rg.outputs) != len(yld.args):
            raise Untranslatable("RegionGrad outputs do not match the joint's yield")
        self.spec: AttentionSpec = match_naive_attention(region, _unwrap(yld.args[0]))
        if self.spec.artifacts:
            raise Untranslatable("artifact-yielding forward inside a joint is not lowered")
        if self.spec.mask is not None:
            raise Untranslatable("the fused backward takes causal or unmasked attention; a general mask's "
                                 "joint runs carve by carve (plan_model + execute_model_plan)")
        for i, d in ((self.spec.q, self.spec.e), (self.spec.v, self.spec.o)):
            x = next(t.stop - t.start for t in region.params[i].type.dims if t.name == d)
            if x % 8 or x > 128:
                raise Untranslatable(f"the bf16 backward takes head dims that are multiples of 8 up to 128, got {x}")
        self.n_params = len(region.params)
        self.do_index = self.n_params - 1  # the seed is passed last (RegionGrad docstring)
        pnames = {rg.names[id(p)]: i for i, p in enumerate(region.params) if id(p) in rg.names}
        by_grad = {g: pname for pname, g in rg.grads.items() if g is not None}
        self.slots = []  # per grad output: (which of q/k/v, yield dim order)
        role = {self.spec.q: "q", self.spec.k: "k", self.spec.v: "v"}
        for gname, node in zip(rg.outputs[1:], yld.args[1:]):
            pname = by_grad.get(gname)
            if pname is None or pname not in pnames or pnames[pname] not in role:
                raise Untranslatable(f"grad {gname!r} is not the gradient of q, k or v")
            self.slots.append((role[pnames[pname]], names_of(node)))
        self.out_dims = names_of(yld.args[0])
        self.dtype = dtype

    def __call__(self, values):
        import torch

        from . import kernels

        spec = self.spec
        dt = torch.bfloat16 if self.dtype == "bf16" else torch.float32
        ins = [torch.as_tensor(np.ascontiguousarray(v), dtype=torch.float32).cuda() for v in values]
        # (riders..., [group], row, feature) views as the forward runner builds them
        rid = list(spec.riders)
        qg = [spec.group] if spec.group else []
        q = ins[spec.q].permute(*[spec.q_dims.index(n) for n in rid + qg + [spec.t, spec.e]])
        k = ins[spec.k].permute(*[spec.k_dims.index(n) for n in rid + [spec.s, spec.e]])
        v = ins[spec.v].permute(*[spec.v_dims.index(n) for n in rid + [spec.s, spec.o]])
        o_dims_internal = tuple(rid + qg + [spec.t, spec.o])
        do = ins[self.do_index].permute(*[self.out_dims.index(n) for n in o_dims_internal])
        lead = list(k.shape[:-2])
        while len(lead) < 2:
            lead.insert(0, 1)
        Bn, HK = lead
        G = q.shape[len(rid)] if spec.group else 1
        T, D = q.shape[-2:]
        S, DV = v.shape[-2:]
        q4 = q.reshape(Bn, HK * G, T, D).to(dt).contiguous()
        k4 = k.reshape(Bn, HK, S, D).to(dt).contiguous()
        v4 = v.reshape(Bn, HK, S, DV).to(dt).contiguous()
        do4 = do.reshape(Bn, HK * G, T, DV).to(dt).contiguous()
        scale = 1.0 if spec.scale is None else spec.scale
        o4, lse = kernels.flash_attention(q4, k4, v4, scale=scale, causal=spec.causal, q_start=spec.t_start,
                                          return_lse=True)
        dq, dk, dv = kernels.flash_attention_backward(q4, k4, v4, o4, do4, lse, scale=scale, causal=spec.causal,
                                                      q_start=spec.t_start)
        torch.cuda.synchronize()
        outs = []
        o = o4.reshape(*q.shape[:-2], T, DV)
        outs.append(o.permute(*[o_dims_internal.index(n) for n in self.out_dims]))
        internal = {"q": (dq.reshape(q.shape), tuple(rid + qg + [spec.t, spec.e])),
                    "k": (dk.reshape(k.shape), tuple(rid + [spec.s, spec.e])),
                    "v": (dv.reshape(v.shape), tuple(rid + [spec.s, spec.o]))}
        for role, dims in self.slots:
            t, names = internal[role]
            outs.append(t.permute(*[names.index(n) for n in dims]))
        return tuple(x.float().cpu().numpy() for x in outs)


def compile_grad(rg, *, dtype: str = "bf16"):
    """RegionGrad of an attention region -> run(values) -> (out, *grads).

    ``values``: numpy arrays positional per joint param (the forward's params,
    then the seed ``dO``), each in its param's type-dim order.  The backward
    kernels are bf16 (fp32 accumulate), head dims multiples of 8 up to 128."""
    if dtype != "bf16":
        raise Untranslatable("the attention backward kernels are bf16")
    runner = _GradRunner(rg, dtype)

    def run(values):
        return runner(values)

    run.spec = runner.spec
    run.source = f"pdb_flash_fwd + pdb_flash_bwd (bf16 tcgen05) causal={runner.spec.causal}"
    return run
