"""The sequence-sharded protocol across real processes, on the CPU: two gloo ranks run
latest_exact_match_attention_b200.longctx.sharded_prefill through TorchComm (the same code a
multi-GPU NCCL run takes), with the per-rank device work replaced by a plain restatement, and
their concatenated result must equal the oracle's single pass over the whole sequence.

This pins the host logic: shard offsets, the last-occurrence exchange, the deduplicated row
requests routed to their owners and the rows coming back in request order."""
import ctypes
import os
import socket
import threading

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import oracle


class PlainOps:
    """What CudaOps computes, in numpy, for small shards (test-only)."""

    status = None

    @staticmethod
    def segment_match(qc, kc, seg_len):
        H, L = qc.shape
        n = H * (L // seg_len)
        q = qc.numpy().view(np.uint32).reshape(n, seg_len)
        k = kc.numpy().view(np.uint32).reshape(n, seg_len)
        src = oracle.latest_prev_match(q, k).astype(np.int32).reshape(H, L)
        ltc = np.zeros((n, seg_len), np.uint32)
        ltp = np.zeros((n, seg_len), np.int32)
        ltn = np.zeros(n, np.int32)
        for s in range(n):
            u, first_rev = np.unique(k[s][::-1], return_index=True)
            ltn[s] = len(u)
            ltc[s, : len(u)] = u
            ltp[s, : len(u)] = seg_len - 1 - first_rev
        return (torch.from_numpy(src), torch.from_numpy(ltc.view(np.int32)), torch.from_numpy(ltp),
                torch.from_numpy(ltn))

    @staticmethod
    def sweep(qc, src, lt, seg_len, base, want_table=True):
        ltc, ltp, ltn = (t.numpy() for t in lt)
        ltc = ltc.view(np.uint32)
        H, L = qc.shape
        n_seg = L // seg_len
        q = qc.numpy().view(np.uint32)
        s = src.numpy()
        rows = []
        for h in range(H):
            table = {}
            for g in range(n_seg):
                g0 = base + g * seg_len
                for i in range(g * seg_len, (g + 1) * seg_len):
                    s[h, i] = g0 + s[h, i] if s[h, i] >= 0 else table.get(int(q[h, i]), -1)
                st = h * n_seg + g
                for e in range(ltn[st]):
                    table[int(ltc[st, e])] = g0 + int(ltp[st, e])
            rows += [(h, c - (1 << 32) if c >= 1 << 31 else c, p) for c, p in table.items()]
        return torch.tensor(rows, dtype=torch.int32).reshape(-1, 3)

    @staticmethod
    def resolve(qc, src, earlier):
        H, L = qc.shape
        best = {}
        if not earlier:
            return
        for h, c, p in torch.cat(list(earlier)).tolist():
            key = (h, c)
            best[key] = max(best.get(key, -1), p)
        q, s = qc.numpy(), src.numpy()
        for h in range(H):
            for i in range(L):
                if s[h, i] < 0:
                    s[h, i] = best.get((h, int(q[h, i])), -1)

    @staticmethod
    def rows(vflat, idx):
        return vflat.index_select(0, idx)

    @staticmethod
    def gather(src, base, v, remote_rows, remote_idx):
        H, L = src.shape
        out = torch.zeros_like(v)
        vb = v.view(H, L, -1).view(torch.uint8)
        ob = out.view(H, L, -1).view(torch.uint8)
        for h in range(H):
            for i in range(L):
                s = int(src[h, i])
                if s >= base:
                    ob[h, i] = vb[h, s - base]
                elif s >= 0:
                    ob[h, i] = remote_rows[int(remote_idx[h, i])]
        return out

    @staticmethod
    def check():
        pass


class PeerPlainOps(PlainOps):
    """PlainOps plus the peer gather, restated: a position before this shard is read from its
    owner rank's [H, L, d] values (owner = s // L, row s - owner * L) through the address the
    comm hands out -- what lema_shard_gather_peer does on the GPU (test-only)."""

    @staticmethod
    def gather_peer(src, base, v, peers):
        H, L = src.shape
        d = v.shape[-1]
        n = H * L * d
        views = [np.ctypeslib.as_array((ctypes.c_float * n).from_address(a)).reshape(H, L, d) if a else None
                 for a in peers]
        out = np.zeros((H, L, d), np.float32)
        s = src.numpy()
        for h in range(H):
            for i in range(L):
                if s[h, i] >= 0:
                    owner = int(s[h, i]) // L
                    out[h, i] = views[owner][h, int(s[h, i]) - owner * L]
        return torch.from_numpy(out)


def inputs(H, T):
    rng = np.random.default_rng(5)
    kc = rng.integers(0, 40, size=(H, T)).astype(np.uint32) * np.uint32(2654435761)  # wraps
    qc = rng.integers(0, 44, size=(H, T)).astype(np.uint32) * np.uint32(2654435761)
    v = rng.standard_normal((H, T, 4)).astype(np.float32)
    return qc.astype(np.uint32), kc.astype(np.uint32), v


def _rank(rank, world, port, H, T, seg, q, peer_ops=False):
    import torch.distributed as dist

    from latest_exact_match_attention_b200.longctx import TorchComm, sharded_prefill
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        qc, kc, v = inputs(H, T)
        L = T // world
        sl = slice(rank * L, (rank + 1) * L)
        src, out = sharded_prefill(torch.from_numpy(qc[:, sl].view(np.int32).copy()),
                                   torch.from_numpy(kc[:, sl].view(np.int32).copy()),
                                   torch.from_numpy(v[:, sl].copy()), TorchComm(),
                                   PeerPlainOps() if peer_ops else PlainOps(), seg)
        q.put((rank, src.numpy(), out.numpy()))
    finally:
        dist.destroy_process_group()


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("peer_ops", [False, True])
@pytest.mark.parametrize("world", [2, 3])
def test_two_gloo_ranks_match_one_pass(world, peer_ops):
    # peer_ops: the ops can read peers' memory, but over gloo TorchComm.peer_values answers
    # None on every rank (no collective is left unmatched) and the rows travel by all-to-all
    H, T, seg = 3, 2 * 6 * 64, 64
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, H, T, seg, q, peer_ops)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict()
    for _ in range(world):
        r, s, o = q.get(timeout=120)
        got[r] = (s, o)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    src = np.concatenate([got[r][0] for r in range(world)], 1)
    out = np.concatenate([got[r][1] for r in range(world)], 1)
    qc, kc, v = inputs(H, T)
    ref = oracle.latest_prev_match(qc, kc)
    assert np.array_equal(src, ref)
    assert np.array_equal(out, oracle.gather(ref, v))
    L = T // world
    assert (ref[:, L:] < L).any() and (ref[:, L:] >= 0).any()   # matches cross the boundary


@pytest.mark.parametrize("world", [2, 3, 4])
def test_peer_rows_with_thread_ranks(world):
    """The peer path's host protocol: ranks as threads (ThreadComm hands every rank the others'
    value addresses), the gather reading earlier shards' rows in place, the release barrier
    after it; the concatenated result equals the oracle's single pass."""
    from latest_exact_match_attention_b200.longctx import ThreadComm, _Board, sharded_prefill
    H, T, seg = 3, world * 6 * 64, 64
    qc, kc, v = inputs(H, T)
    L = T // world
    board = _Board(world)
    res, errs = [None] * world, []
    vs = [torch.from_numpy(v[:, r * L:(r + 1) * L].copy()) for r in range(world)]   # kept alive

    def run(r):
        try:
            sl = slice(r * L, (r + 1) * L)
            res[r] = sharded_prefill(torch.from_numpy(qc[:, sl].view(np.int32).copy()),
                                     torch.from_numpy(kc[:, sl].view(np.int32).copy()), vs[r],
                                     ThreadComm(board, r), PeerPlainOps(), seg)
        except BaseException as e:  # noqa: BLE001 -- re-raised below
            errs.append(e)
            board.barrier.abort()

    threads = [threading.Thread(target=run, args=(r,)) for r in range(world)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=120)
    assert not errs, errs
    src = np.concatenate([res[r][0].numpy() for r in range(world)], 1)
    out = np.concatenate([res[r][1].numpy() for r in range(world)], 1)
    ref = oracle.latest_prev_match(qc, kc)
    assert np.array_equal(src, ref)
    assert np.array_equal(out, oracle.gather(ref, v))
    assert (ref[:, L:] < L).any() and (ref[:, L:] >= 0).any()
