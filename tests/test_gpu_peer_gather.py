"""The copy-engine final gather (partition.PeerGather) on two GPUs of one box.

Two ranks (one process per GPU, NCCL) run the slab-interleaved forward of a small
causal job, writing into symmetric memory and pushing each slab to the peer; the
gathered output must equal, bit for bit, the same units computed whole on one GPU.
Needs two GPUs: on a one-GPU box the test is skipped.
"""

import os
import socket

import pytest

pytestmark = pytest.mark.gpu

B, H, S, D = 1, 16, 512, 128


def _inputs(dev):
    import torch

    g = torch.Generator(device="cpu").manual_seed(7)
    return [torch.randn(1, B * H, S, D, generator=g).to(torch.bfloat16).to(dev) for _ in range(3)]


def _rank(rank, world, port, result):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        from pdum_dsl_b200 import kernels
        from pdum_dsl_b200.partition import PeerGather, chunked_shards, peer_gather_overlapped

        q, k, v = _inputs(dev)
        ranges = [(x.lo, x.hi) for x in chunked_shards(B * H, world, rank, 2)]
        ins = [(q[:, lo:hi], k[:, lo:hi], v[:, lo:hi], None) for lo, hi in ranges]
        pg = PeerGather((B * H, S, D), torch.bfloat16, dev)

        def attend(qs, ks, vs, _o, out):
            return kernels.flash_attention(qs, ks, vs, causal=True, out=out.unsqueeze(0))

        for _ in range(2):  # twice: the second step overwrites the first step's rows
            full = peer_gather_overlapped(attend, ins, ranges, pg)
        torch.cuda.synchronize()
        whole = kernels.flash_attention(q, k, v, causal=True)[0]
        kernels.check_device_errors()
        result[rank] = bool(torch.equal(full, whole))
    finally:
        dist.destroy_process_group()


def test_peer_gather_matches_whole_job(cuda):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        result = mgr.dict()
        procs = [ctx.Process(target=_rank, args=(r, 2, port, result)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=300)
        for p in procs:  # a rank stuck past the limit is ended here (its process only)
            if p.is_alive():
                p.kill()
                p.join()
        codes = [p.exitcode for p in procs]
        assert codes == [0, 0], f"rank exit codes {codes}"
        assert dict(result) == {0: True, 1: True}
