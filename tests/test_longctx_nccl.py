"""Sequence-sharded prefill over NCCL, one process per GPU (needs two or more GPUs; skipped
otherwise): each rank's slice of the result must equal the same slice of one pass of the
matcher over the whole sequence."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

SPEC_POOL = 1 << 16


def _rank(rank, world, port, q, peer):
    import datetime

    import torch.distributed as dist

    from latest_exact_match_attention_b200 import prefill_match, synth
    from latest_exact_match_attention_b200.longctx import TorchComm, sharded_prefill
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0",
                      LEMA_SHARD_PEER=peer)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    ok = False
    try:
        spec = synth.CodeSpec(bits=32, pool=SPEC_POOL, alpha=1.05, fresh=0.05)
        H, T = 4, world * (1 << 21)
        L = T // world
        qc, kc, v = synth.long_code_shard(H, 0, T, spec, seed=3, device="cuda")
        src1, out1 = prefill_match(qc, kc, v)
        sl = slice(rank * L, (rank + 1) * L)
        comm = TorchComm()
        src, out = sharded_prefill(qc[:, sl], kc[:, sl], v[:, sl], comm, seg_len=4096)
        # twice: the second call reuses the mapped peer values
        src2, out2 = sharded_prefill(qc[:, sl], kc[:, sl], v[:, sl], comm, seg_len=4096)
        torch.cuda.synchronize()
        comm.close()
        ok = bool(torch.equal(src, src1[:, sl]) and torch.equal(out.view(torch.int16),
                                                                  out1[:, sl].view(torch.int16)))
        ok = ok and bool(torch.equal(src2, src) and torch.equal(out2.view(torch.int16), out.view(torch.int16)))
        crossed = bool(((src >= 0) & (src < rank * L)).any()) if rank else True
        ok = ok and crossed
        dist.barrier()
    finally:
        q.put((rank, ok))
        dist.destroy_process_group()


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("peer", ["1", "0"])
def test_nccl_two_ranks_equal_one_pass(peer):
    # peer=1: rank 1's gather reads rank 0's value rows over NVLink (CUDA IPC); 0: the rows
    # are requested and exchanged by all-to-all
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q, peer)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
    assert all(res.values()), res
    assert all(p.exitcode == 0 for p in procs)
