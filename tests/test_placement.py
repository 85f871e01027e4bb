"""The partition read off a placed region (mesh placement integration).

A rider dim bound to a machine level in the reference's global-view spelling
(``pdum/tl/zoo/megatron.py``) gives the shards; the reference's own traffic pass
(``pdum/tl/placement.py:116-181``) prices the final merge, and ``gather_bytes`` /
``alpha_beta_seconds`` must restate it exactly.  The world-size-2 gloo runs check
that the placement-driven shards gather back to the full attention."""

import os
import socket

import numpy as np
import pytest

from pdum_dsl_b200.partition import Placement, alpha_beta_seconds, gather_bytes


def _ins(region, seed=0):
    from pdum.tl.tensor import Tensor

    rng = np.random.default_rng(seed)
    out = []
    for p in region.params:
        dims = p.type.layout.dims
        out.append(Tensor.from_numpy(rng.standard_normal(tuple(d.size for d in dims)), tuple(d.name for d in dims)))
    return out


@pytest.mark.parametrize("bind,group,world", [("h", None, 2), ("h", None, 4), ("b", None, 2), ("g", 2, 2)])
def test_placement_read_off_the_region(dsl, bind, group, world):
    from pdum_dsl_b200.partition import placement_of
    from pdum_dsl_b200.regions import placed_attention_region

    B, H = 4, 4
    r = placed_attention_region(B, H, 6, 3, world=world, bind=bind, group=group)
    pl = placement_of(r)
    extent = {"b": B, "h": H, "g": H}[bind]
    assert pl == Placement(bind, "gpu", world, extent // world)


@pytest.mark.parametrize("bind,group", [("h", None), ("b", None), ("g", 2)])
def test_reference_traffic_prices_the_gather_as_we_do(dsl, bind, group):
    """placement.traffic charges (p-1)/p of the merged output at the declared 8-byte
    interior item; our gather moves the same elements at the device's item size."""
    from pdum.tl.dialect import region_names
    from pdum.tl.placement import mesh, traffic

    from pdum_dsl_b200.regions import placed_attention_region

    B, H, T, D, W = 2, 4, 6, 3, 2
    r = placed_attention_region(B, H, T, D, world=W, bind=bind, group=group)
    rep = traffic(r, None, mesh(W), names=region_names(r, ("q", "k", "v")))
    assert [(c.kind, c.level) for c in rep.collectives] == [("all_gather", "gpu")]
    hq = H * (group or 1)
    elems = B * hq * T * D
    assert rep.collectives[0].bytes == gather_bytes(elems * 8, W)
    assert gather_bytes(elems * 2, W) * 4 == rep.collectives[0].bytes  # bf16 on the device
    machine = mesh(W, link_bandwidth=770e9, link_latency=10e-6)
    assert rep.time(machine) == pytest.approx(alpha_beta_seconds(rep.collectives[0].bytes, 770e9, 10e-6))


def test_placement_keeps_the_denotation(dsl):
    """Placement is metadata: the placed region evaluates to the unplaced one."""
    from pdum.tl.dialect import run_region

    from pdum_dsl_b200.regions import attention_region, placed_attention_region

    placed = placed_attention_region(2, 4, 5, 3, world=2, bind="h", scale=0.5)
    plain = attention_region(B=2, H=4, T=5, D=3, scale=0.5)
    pin = _ins(placed)
    qin = []
    from pdum.tl.tensor import Tensor

    for t, p in zip(pin, plain.params):
        names = tuple(d.name for d in p.type.layout.dims)
        arr = t.to_numpy()
        qin.append(Tensor.from_numpy(arr.reshape(tuple(d.size for d in p.type.layout.dims)), names))
    a = run_region(placed, pin)
    b = run_region(plain, qin)
    np.testing.assert_array_equal(a.to_numpy(order=("b", "h", "t", "o")), b.to_numpy(order=("b", "h", "t", "o")))


def test_sequence_and_replicating_bindings_are_refused(dsl):
    from pdum.dsl.ir import Region
    from pdum.dsl.ops import CORE_OPS
    from pdum.tl.dialect import TL_OPS, tensor_type_of_layout
    from pdum.tl.tensor import Tensor

    from pdum_dsl_b200.partition import placement_of
    from pdum_dsl_b200.regions import attention_region

    with pytest.raises(ValueError, match="binds no dim"):
        placement_of(attention_region(B=2, H=2, T=4, D=3))
    from pdum.dsl.ir import Builder

    b = Builder({**CORE_OPS, **TL_OPS})
    lay = Tensor.from_numpy(np.zeros((2, 2, 3)), ("w", "tl", "e")).bind(w="gpu").layout
    p0 = b.param(0, tensor_type_of_layout(lay))
    region = Region(params=(p0,), body=(b.emit("core.yield", p0),))
    with pytest.raises(ValueError, match="rider"):
        placement_of(region)


def _worker(rank, world, port, q, k, v, want, pl, errs):
    import torch
    import torch.distributed as dist

    from oracle import attention as OA
    from pdum_dsl_b200.partition import sharded_attention

    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)

        def attend(qs, ks, vs):
            g = qs.shape[1] // ks.shape[1]
            o, *_ = OA.attention_fwd(qs.numpy(), np.repeat(ks.numpy(), g, axis=1), np.repeat(vs.numpy(), g, axis=1),
                                     scale=0.25, causal=True)
            return torch.from_numpy(o)

        full = sharded_attention(torch.from_numpy(q), torch.from_numpy(k), torch.from_numpy(v), world=world,
                                 rank=rank, attend=attend, gather=True, placement=pl)
        np.testing.assert_allclose(full.numpy(), want, rtol=1e-12, atol=1e-12)
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported to the parent
        errs.put(f"rank {rank}: {e!r}")


@pytest.mark.parametrize("pl,hq,hkv", [(Placement("h", "gpu", 2, 2), 4, 4), (Placement("b", "gpu", 2, 1), 4, 4),
                                       (Placement("g", "gpu", 2, 1), 4, 2)])
def test_gloo_world2_placed_shards_gather_the_full_output(pl, hq, hkv):
    import torch.multiprocessing as mp

    from oracle import attention as OA

    rng = np.random.default_rng(1)
    q = rng.standard_normal((2, hq, 9, 8))
    k = rng.standard_normal((2, hkv, 9, 8))
    v = rng.standard_normal((2, hkv, 9, 8))
    want, *_ = OA.attention_fwd(q, k, v, scale=0.25, causal=True)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    errs = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, k, v, want, pl, errs)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert errs.empty(), errs.get()
