"""Batch x head / KV-group partitioning: host logic, and a world-size-2 gloo run on CPU."""

import os
import socket

import numpy as np
import pytest

from pdum_dsl_b200.partition import attention_units, gather_bytes, local_slices, shard_units


@pytest.mark.parametrize("n,world", [(256, 1), (256, 2), (256, 8), (32, 8), (7, 3), (3, 8)])
def test_shards_cover_every_unit_once(n, world):
    seen = []
    for r in range(world):
        s = shard_units(n, world, r)
        seen += list(range(s.lo, s.hi))
        assert abs(s.units - n / world) < 1
    assert seen == list(range(n))


def test_gqa_units_are_kv_groups_and_runs_split_at_batch():
    n, r = attention_units(4, 64, 8)
    assert (n, r) == (32, 8)
    s = shard_units(n, 3, 1)  # units 10..21
    runs = local_slices(s, 4, 8)
    assert runs == [(1, 2, 8), (2, 0, 5)]
    assert sum(h1 - h0 for _, h0, h1 in runs) == s.units
    assert gather_bytes(256, 8) == 224


def _worker(rank, world, port, q, k, v, want, errs):
    import torch
    import torch.distributed as dist

    from oracle import attention as OA
    from pdum_dsl_b200.partition import sharded_attention

    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)

        def attend(qs, ks, vs):  # CPU stand-in for the kernel: the oracle, per unit
            g = qs.shape[1] // ks.shape[1]
            o, *_ = OA.attention_fwd(qs.numpy(), np.repeat(ks.numpy(), g, axis=1), np.repeat(vs.numpy(), g, axis=1),
                                     scale=0.25, causal=True)
            return torch.from_numpy(o)

        full = sharded_attention(torch.from_numpy(q), torch.from_numpy(k), torch.from_numpy(v), world=world,
                                 rank=rank, attend=attend, gather=True)
        np.testing.assert_allclose(full.numpy(), want, rtol=1e-12, atol=1e-12)
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported to the parent
        errs.put(f"rank {rank}: {e!r}")


def test_gloo_world2_sharded_gqa_gathers_the_full_output():
    import torch.multiprocessing as mp

    from oracle import attention as OA

    rng = np.random.default_rng(0)
    q = rng.standard_normal((2, 4, 9, 8))
    k = rng.standard_normal((2, 2, 9, 8))
    v = rng.standard_normal((2, 2, 9, 8))
    want, *_ = OA.attention_fwd(q, k, v, scale=0.25, causal=True)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    errs = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, k, v, want, errs)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert errs.empty(), errs.get()


@pytest.mark.parametrize("n,world,chunks", [(256, 8, 2), (256, 2, 4), (32, 4, 2), (8, 1, 8)])
def test_chunked_shards_interleave_slabs(n, world, chunks):
    from pdum_dsl_b200.partition import chunked_shards

    owner = {}
    for r in range(world):
        for c, s in enumerate(chunked_shards(n, world, r, chunks)):
            for u in range(s.lo, s.hi):
                owner[u] = (c, r)
    assert sorted(owner) == list(range(n))
    slab = n // chunks
    for u, (c, r) in owner.items():  # slab-major, then rank-major: what a rank-major all-gather writes
        assert u // slab == c and (u % slab) // (slab // world) == r


def _overlap_worker(rank, world, port, q, k, v, want, errs):
    import torch
    import torch.distributed as dist

    from oracle import attention as OA
    from pdum_dsl_b200.partition import chunked_shards, gather_overlapped

    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        chunks = 2
        B, H, T, D = q.shape
        qf, kf, vf = (torch.from_numpy(x.reshape(B * H, T, D)) for x in (q, k, v))
        shards = chunked_shards(B * H, world, rank, chunks)
        full = torch.empty((B * H, T, D), dtype=torch.float64)
        slab = B * H // chunks

        def attend(qs, ks, vs):
            o, *_ = OA.attention_fwd(qs.numpy(), ks.numpy(), vs.numpy(), scale=0.25, causal=True)
            return torch.from_numpy(o)

        gather_overlapped(attend, [(qf[s.lo:s.hi], kf[s.lo:s.hi], vf[s.lo:s.hi]) for s in shards],
                          [full[c * slab:(c + 1) * slab] for c in range(chunks)])
        np.testing.assert_allclose(full.numpy().reshape(want.shape), want, rtol=1e-12, atol=1e-12)
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported to the parent
        errs.put(f"rank {rank}: {e!r}")


def test_gloo_world2_overlapped_slab_gather_rebuilds_the_output():
    import torch.multiprocessing as mp

    from oracle import attention as OA

    rng = np.random.default_rng(1)
    q, k, v = (rng.standard_normal((2, 4, 9, 8)) for _ in range(3))
    want, *_ = OA.attention_fwd(q, k, v, scale=0.25, causal=True)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    errs = ctx.Queue()
    procs = [ctx.Process(target=_overlap_worker, args=(r, 2, port, q, k, v, want, errs)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert errs.empty(), errs.get()
