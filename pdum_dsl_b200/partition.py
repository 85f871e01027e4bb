"""Batch x head (or KV-group) partitioning of attention over the GPUs of one box.

The reference prices sharding analytically: named dims bound to mesh levels,
a merge of a bound dim implies an all-gather of (p-1)/p of its bytes
(``pdum/tl/placement.py:116-178``), and head groups bind to the GPU level in
``pdum/tl/zoo/megatron.py:7-14,45-50``.  Attention has no reduction over the
(batch, head) riders, so the partition here is exact and communication-free
inside the computation:

* MHA: the B*H (batch, head) units are split into contiguous blocks, one per
  rank;
* GQA: the units are (batch, KV head) groups, so every query head of a group
  stays with its K/V and K/V are never replicated;
* the only exchange is the optional final gather of the output shards over
  NCCL (``all_gather``), priced exactly as ``placement.traffic`` prices a merge.

Sequence is never split (the reference refuses split-K over the carried s dim,
``docs/design/340_grid-launch.md:162-171``).

A partition can also be read off a placed region instead of the fixed rule:
``placement_of`` finds the rider dim the region binds to a machine level (the
global-view spelling ``(w, <rider>l)`` with ``w`` bound, ``zoo/megatron.py``),
``sharded_attention(..., placement=...)`` gives each rank its index along that
dim, and ``gather_bytes`` / ``alpha_beta_seconds`` restate what
``placement.traffic`` and ``TrafficReport.time`` charge for the final merge
(``tl/placement.py:91-101,170-181``), so the measured NCCL gather can be set
beside the model's prediction.
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class Shard:
    rank: int
    world: int
    lo: int  # first unit (inclusive)
    hi: int  # last unit (exclusive)

    @property
    def units(self) -> int:
        return self.hi - self.lo


def shard_units(n_units: int, world: int, rank: int) -> Shard:
    """Contiguous, balanced block of units for `rank` (sizes differ by at most one)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    lo = n_units * rank // world
    hi = n_units * (rank + 1) // world
    return Shard(rank, world, lo, hi)


def attention_units(batch: int, heads_q: int, heads_kv: int) -> tuple[int, int]:
    """(number of units, query heads per unit): KV groups when heads_q > heads_kv."""
    if heads_q % heads_kv:
        raise ValueError("heads_q must be a multiple of heads_kv")
    return batch * heads_kv, heads_q // heads_kv


def gather_bytes(out_bytes: int, world: int) -> int:
    """Bytes each rank receives in the final all-gather: (p-1)/p of the output
    (the merge cost of placement.traffic, placement.py:166-178)."""
    return out_bytes * (world - 1) // world


def alpha_beta_seconds(nbytes: int, bandwidth: float, latency: float = 0.0) -> float:
    """The reference's alpha-beta estimate of one collective: latency + bytes over
    the link bandwidth (``TrafficReport.time``, placement.py:91-101)."""
    return latency + (nbytes / bandwidth if bandwidth else 0.0)


@dataclass(frozen=True)
class Placement:
    dim: str    # the rider dim split over the mesh: "b", "h", or "g" (GQA KV groups)
    level: str  # machine level the mesh dim is bound to
    world: int  # extent of the bound mesh dim = number of devices
    local: int  # extent of `dim` held by each device


_NOT_RIDERS = ("t", "s", "e", "o", "r")


def placement_of(region) -> Placement:
    """The partition a placed attention region declares.

    Exactly one dim may be bound to a machine level, the same one in every
    param; it must be immediately followed by the per-device part of a rider
    dim (``<rider>l``).  Binding a sequence / feature dim (or ``r``, which
    would replicate K/V) is refused: that placement implies a cross-device
    reduction or a split-K the reference does not model."""
    bound = set()
    locs = set()
    for prm in region.params:
        dims = prm.type.layout.dims
        for i, d in enumerate(dims):
            if d.level is None:
                continue
            if i + 1 >= len(dims):
                raise ValueError(f"bound dim {d.name!r} has no per-device part after it")
            nxt = dims[i + 1]
            rider = nxt.name[:-1] if nxt.name.endswith("l") else None
            if rider is None or rider in _NOT_RIDERS:
                raise ValueError(f"bound dim {d.name!r} must split a batch / head rider, found {nxt.name!r}")
            bound.add((d.name, d.level, d.size))
            locs.add((rider, nxt.size))
    if not bound:
        raise ValueError("region binds no dim to a machine level")
    if len(bound) != 1 or len(locs) != 1:
        raise ValueError(f"expected one bound rider shared by every param, found {sorted(bound)} / {sorted(locs)}")
    (_, level, world), = bound
    (rider, local), = locs
    if len(region.params) != sum(1 for p in region.params if any(d.level for d in p.type.layout.dims)):
        raise ValueError("every param must carry the bound dim (K/V would otherwise be replicated)")
    return Placement(rider, level, world, local)


def local_slices(shard: Shard, batch: int, heads_kv: int):
    """Units -> list of (b, hk_lo, hk_hi) runs covered by this shard."""
    runs = []
    u = shard.lo
    while u < shard.hi:
        b, hk = divmod(u, heads_kv)
        end = min(shard.hi, (b + 1) * heads_kv)
        runs.append((b, hk, hk + (end - u)))
        u = end
    return runs


def _placed_attention(q, k, v, pl: Placement, *, world, rank, attend, gather, group):
    import torch

    if pl.world != world:
        raise ValueError(f"placement is over {pl.world} devices, running on {world}")
    B, Hq = q.shape[:2]
    Hkv = k.shape[1]
    r = Hq // Hkv
    lo, hi = rank * pl.local, (rank + 1) * pl.local
    if pl.dim == "b":
        if B != world * pl.local:
            raise ValueError(f"b={B} does not match placement {pl}")
        qs, ks, vs = q[lo:hi], k[lo:hi], v[lo:hi]
    elif pl.dim in ("h", "g"):
        if Hkv != world * pl.local or (pl.dim == "h" and r != 1):
            raise ValueError(f"heads {Hq}/{Hkv} do not match placement {pl}")
        qs, ks, vs = q[:, lo * r:hi * r], k[:, lo:hi], v[:, lo:hi]
    else:
        raise ValueError(f"cannot place attention on {pl.dim!r}")
    o = attend(qs, ks, vs)
    if not gather:
        return o
    import torch.distributed as dist

    T, Dv = o.shape[2], o.shape[3]
    full = torch.empty((world, *o.shape), dtype=o.dtype, device=o.device)
    dist.all_gather_into_tensor(full.reshape(-1, T, Dv), o.contiguous().reshape(-1, T, Dv), group=group)
    if pl.dim == "b":
        return full.reshape(B, Hq, T, Dv)
    return full.permute(1, 0, 2, 3, 4).reshape(B, Hq, T, Dv)  # (w, b, hl, t, o) -> (b, h, t, o)


def sharded_attention(q, k, v, *, world: int, rank: int, attend, gather: bool = False, group=None,
                      placement: Placement | None = None):
    """Run ``attend(q_s, k_s, v_s)`` on this rank's units; optionally all-gather.

    q (B, Hq, T, D), k/v (B, Hkv, S, D) hold the FULL problem (or at least this
    rank's units).  The shard's units are flattened to one (1, units*r, T, D)
    job so a single kernel launch covers them.  Returns this rank's output
    shard, or with ``gather`` the full (B, Hq, T, Dv) output on every rank
    (``torch.distributed.all_gather_into_tensor``; ``group`` as in torch).

    With ``placement`` (from ``placement_of`` on a placed region) rank ``i``
    takes index ``i`` of the bound mesh dim instead: its block of batches, of
    heads of every batch, or of KV groups of every batch; the gathered output
    is put back in (b, h, t, o) order."""
    import torch

    if placement is not None:
        return _placed_attention(q, k, v, placement, world=world, rank=rank, attend=attend, gather=gather,
                                 group=group)

    B, Hq, T, D = q.shape
    Hkv = k.shape[1]
    n, r = attention_units(B, Hq, Hkv)
    sh = shard_units(n, world, rank)
    qs, ks, vs = [], [], []
    for b, h0, h1 in local_slices(sh, B, Hkv):
        qs.append(q[b, h0 * r:h1 * r])
        ks.append(k[b, h0:h1])
        vs.append(v[b, h0:h1])
    qj = torch.cat(qs)[None] if qs else q[:0, :0]
    kj = torch.cat(ks)[None] if ks else k[:0, :0]
    vj = torch.cat(vs)[None] if vs else v[:0, :0]
    o = attend(qj, kj, vj) if sh.units else torch.empty((1, 0, T, v.shape[3]), dtype=q.dtype, device=q.device)
    if not gather:
        return o
    import torch.distributed as dist

    per = [shard_units(n, world, i).units for i in range(world)]
    if len(set(per)) != 1:
        raise ValueError("gather needs equal shards: choose world dividing the unit count")
    full = torch.empty((world * per[0] * r, T, v.shape[3]), dtype=o.dtype, device=o.device)
    dist.all_gather_into_tensor(full, o.reshape(per[0] * r, T, v.shape[3]).contiguous(), group=group)
    return full.reshape(B, Hq, T, v.shape[3])


def chunked_shards(n_units: int, world: int, rank: int, chunks: int) -> list[Shard]:
    """The partition for a final gather that overlaps the computation.

    The units are cut into ``chunks`` consecutive slabs and every slab is split
    evenly over the ranks: rank r owns block r of each slab.  The all-gather of
    one slab's outputs (``all_gather_into_tensor``, rank-major) then lands
    exactly on that slab of the global output -- no reordering copy -- while
    the next slab computes.  Requires chunks * world to divide the unit count."""
    if n_units % (chunks * world):
        raise ValueError(f"{n_units} units do not split into {chunks} slabs x {world} ranks")
    per = n_units // (chunks * world)
    return [Shard(rank, world, c * per * world + rank * per, c * per * world + (rank + 1) * per)
            for c in range(chunks)]


def gather_overlapped(attend, slabs_in, slabs_out, *, group=None, comm_stream=None):
    """For each slab: ``attend(*slabs_in[c])`` -> this rank's block of outputs, then
    ``all_gather_into_tensor(slabs_out[c], block)`` -- on ``comm_stream`` (CUDA)
    once that block's kernel has completed, so the gather of slab c runs under
    the computation of slab c + 1.  ``slabs_out[c]`` is the global output of the
    slab (world x block, rank-major).  Returns the per-slab blocks."""
    import torch
    import torch.distributed as dist

    blocks = []
    cur = torch.cuda.current_stream() if comm_stream is not None else None
    for ins, out in zip(slabs_in, slabs_out):
        blk = attend(*ins)
        blocks.append(blk)
        flat = blk.reshape(out.shape[0] // dist.get_world_size(group), *out.shape[1:])
        if comm_stream is None:
            dist.all_gather_into_tensor(out, flat.contiguous(), group=group)
            continue
        done = torch.cuda.Event()
        done.record(cur)
        comm_stream.wait_event(done)
        with torch.cuda.stream(comm_stream):
            dist.all_gather_into_tensor(out, flat, group=group)
            flat.record_stream(comm_stream)
    if comm_stream is not None:
        cur.wait_stream(comm_stream)
    return blocks


class PeerGather:
    """The final gather by copy engines over NVLink, without NCCL kernels.

    The global output lives in symmetric memory (``torch.distributed._symmetric_memory``):
    every rank's buffer is mapped into every other rank's address space. When a
    block of rows of the output is final on this rank, ``push(lo, hi)`` copies it
    into the same rows of every peer's buffer, one ``cudaMemcpyAsync`` per peer on
    its own side stream (copy engines: no SMs taken from the forward, which
    keeps all of them); ``finish()`` joins the side streams and runs a one-word
    NCCL all-reduce on the current stream, which completes on a rank only once
    every rank has reached it, i.e. once every push into this rank's buffer has
    completed. The all-gather is the one of ``placement.traffic`` (each rank
    receives (p-1)/p of the output); only the transport differs from
    ``all_gather_into_tensor``. Loads of peer memory: none (the copies write to
    the peers); no multicast.
    """

    def __init__(self, shape, dtype, device, group=None):
        import torch
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem

        grp = group if group is not None else dist.group.WORLD
        self.rank = dist.get_rank(grp)
        self.world = dist.get_world_size(grp)
        self.group = grp
        self.full = symm_mem.empty(tuple(shape), dtype=dtype, device=device)
        self._hdl = symm_mem.rendezvous(self.full, grp.group_name)
        self.peers = [self._hdl.get_buffer(p, tuple(shape), dtype) for p in range(self.world) if p != self.rank]
        self.streams = [torch.cuda.Stream(device) for _ in self.peers]
        self._flag = torch.zeros(1, device=device)

    def push(self, lo: int, hi: int) -> None:
        """Copy rows [lo, hi) of this rank's buffer to every peer, after the work
        already queued on the current stream."""
        import torch

        cur = torch.cuda.current_stream(self.full.device)
        src = self.full[lo:hi]
        for s, peer in zip(self.streams, self.peers):
            s.wait_stream(cur)
            with torch.cuda.stream(s):
                peer[lo:hi].copy_(src, non_blocking=True)

    def finish(self) -> None:
        """Every rank's pushes into every buffer are complete once this returns on
        the current stream (stream-ordered; the host does not wait)."""
        import torch
        import torch.distributed as dist

        cur = torch.cuda.current_stream(self.full.device)
        for s in self.streams:
            cur.wait_stream(s)
        dist.all_reduce(self._flag, group=self.group)


def peer_gather_overlapped(attend, slabs_in, slab_rows, pg: PeerGather):
    """For each slab: ``attend(*slabs_in[c], out)`` writes this rank's block of the
    slab straight into ``pg.full[slab_rows[c]]``, then ``pg.push`` sends it to
    every peer while the next slab computes; ``pg.finish`` closes the step."""
    for ins, (lo, hi) in zip(slabs_in, slab_rows):
        attend(*ins, pg.full[lo:hi])
        pg.push(lo, hi)
    pg.finish()
    return pg.full
