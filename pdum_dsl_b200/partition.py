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


def sharded_attention(q, k, v, *, world: int, rank: int, attend, gather: bool = False, group=None):
    """Run ``attend(q_s, k_s, v_s)`` on this rank's units; optionally all-gather.

    q (B, Hq, T, D), k/v (B, Hkv, S, D) hold the FULL problem (or at least this
    rank's units).  The shard's units are flattened to one (1, units*r, T, D)
    job so a single kernel launch covers them.  Returns this rank's output
    shard, or with ``gather`` the full (B, Hq, T, Dv) output on every rank
    (``torch.distributed.all_gather_into_tensor``; ``group`` as in torch)."""
    import torch

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
