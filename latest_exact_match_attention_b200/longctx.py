"""The exact op over one sequence too long for one pass or one GPU, sharded by sequence.

Config 5 of the benchmark: one sequence of 2^26 positions, 16 heads, 32-bit codes, 128-byte
value rows -- about 287 GB resident, so at least two B200s. Rank r of W owns positions
[r * L, (r + 1) * L) of every head ([H, L] codes, [H, L, d_v] values) and computes, for
those positions, exactly what one `latest_prev_match` + gather over the whole sequence gives
(code/lema/attention.py:100-158): src as global positions, and the value rows.

Per rank (kernels in csrc/shard.cu, K2 in csrc/prefill_match.cu):

    1. segment match     K2 on segments of `seg_len` positions, each with its last-occurrence
                         table (LT: distinct key codes and their last positions)
    2. sweep             per head, segments in order against a device hash: in-segment
                         misses look up earlier segments; the hash ends as the shard's LT
    3. exchange          all-gather of the shards' LTs, each re-hashed by its owner into a
                         table sized for it (8 bytes per slot, load <= 0.5)
    4. resolve           queries still unmatched probe the earlier shards' tables, newest
                         first (reads only: no rank re-inserts the others' entries)
    5. fetch             rows at earlier shards' positions: requests (deduplicated) and rows
                         by all-to-all, landing in this GPU's memory before any kernel reads
    6. gather            one kernel: own rows, fetched rows, or zeros

Where every rank can map every other rank's values (one node: CUDA IPC over NVLink; ranks as
threads of one process: the same memory), steps 5 and 6 are one kernel instead: the gather
reads an earlier shard's row where it lies, with plain loads of the peer GPU's memory, and a
collective after it keeps every rank's values in place until the last read. A single rank
takes that kernel too: all its sources are its own, so there are no requests to build.

Only steps 3 and 5 talk to other ranks, and nothing waits for another rank before step 3.
The collectives go through a `Comm`: `TorchComm` (torch.distributed: NCCL on the GPU, gloo
in the CPU tests), `ThreadComm` (ranks as threads of one process, for running the same code
over virtual shards on one GPU), `SingleComm`. The per-rank device work goes through an ops
object (`CudaOps` here; the CPU tests plug in a restatement).
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

from . import _lib
from ._lib import LEMA_STATUS_PROBE_LIMIT, LEMA_STATUS_TABLE_FULL, LemaError, call, ptr, require_cuda

__all__ = ["sharded_prefill", "emulated_sharded_prefill", "CudaOps", "TorchComm", "ThreadComm",
           "SingleComm"]


# ---------------------------------------------------------------------------- comms
class SingleComm:
    rank, world = 0, 1

    def peer_values(self, t):
        return [t.data_ptr()]

    def after_peer_reads(self, device):
        pass

    def all_gather(self, t):
        return [t]

    def all_to_all(self, parts):
        return list(parts)


class TorchComm:
    """Collectives over a torch.distributed process group (every rank calls every method in
    the same order). Variable-length data: counts first, then padded / split transfers."""

    def __init__(self, group=None):
        import torch.distributed as dist
        self.dist, self.group = dist, group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self._mapped: dict[int, tuple[bytes, int, int]] = {}  # rank -> (handle, offset, address)

    def peer_values(self, t: torch.Tensor) -> list[int] | None:
        """Every earlier rank's `t` mapped into this process (CUDA IPC), then this rank's own,
        in rank order (0 for the later ranks, never read), or None on every rank when any rank
        cannot (not NCCL, not CUDA, more than 16 ranks, a failed
        export or import). A collective: every rank calls it."""
        ok = t.is_cuda and self.world <= 16 and self.dist.get_backend(self.group) == "nccl"
        if not ok:
            return None        # the same on every rank: backend, world size and environment
        rec = torch.zeros(80, dtype=torch.uint8)
        handle = (ctypes.c_ubyte * 64)()
        off = ctypes.c_int64(0)
        if _lib.lib().lema_ipc_export(ctypes.c_void_p(t.data_ptr()), handle, ctypes.byref(off)) == 0:
            rec[:64] = torch.tensor(list(handle), dtype=torch.uint8)
            rec[64:72] = torch.tensor([off.value], dtype=torch.int64).view(torch.uint8)
            rec[72] = 1
        recs = torch.empty(self.world * 80, dtype=torch.uint8, device=t.device)
        self.dist.all_gather_into_tensor(recs, rec.to(t.device), group=self.group)
        recs = recs.cpu().view(self.world, 80)
        ptrs, good = [], bool(recs[:, 72].all())
        for r in range(self.world):
            if r >= self.rank or not good:   # only the earlier ranks' rows are ever read
                ptrs.append(t.data_ptr() if r == self.rank else 0)
                continue
            h = bytes(recs[r, :64].tolist())
            o = int(recs[r, 64:72].view(torch.int64))
            got = self._mapped.get(r)
            if got is not None and got[:2] == (h, o):
                ptrs.append(got[2])
                continue
            if got is not None:   # the rank's values moved since the last call: drop that map
                _lib.lib().lema_ipc_close(ctypes.c_void_p(got[2]), got[1])
                del self._mapped[r]
            addr = ctypes.c_void_p(0)
            if _lib.lib().lema_ipc_import(h, o, ctypes.byref(addr)) != 0:
                good = False
                ptrs.append(0)
                continue
            self._mapped[r] = (h, o, addr.value)
            ptrs.append(addr.value)
        flag = torch.tensor([1 if good else 0], dtype=torch.int32, device=t.device)
        self.dist.all_reduce(flag, op=self.dist.ReduceOp.MIN, group=self.group)
        return ptrs if int(flag.item()) == 1 else None

    def after_peer_reads(self, device):
        """Stream-ordered: no rank's later work on its values runs before every rank's gather."""
        self.dist.all_reduce(torch.zeros(1, dtype=torch.int32, device=device), group=self.group)

    def close(self):
        """Unmap the other ranks' values (the maps also end with the process)."""
        for _, o, a in self._mapped.values():
            _lib.lib().lema_ipc_close(ctypes.c_void_p(a), o)
        self._mapped.clear()

    def _counts(self, n: int, device) -> list[int]:
        c = torch.tensor([n], dtype=torch.int64, device=device)
        out = torch.empty(self.world, dtype=torch.int64, device=device)
        self.dist.all_gather_into_tensor(out, c, group=self.group)
        return [int(x) for x in out.cpu()]

    def all_gather(self, t: torch.Tensor) -> list[torch.Tensor]:
        """t [n, ...] -> the tensors of every rank, in rank order."""
        counts = self._counts(t.shape[0], t.device)
        m = max(counts)
        pad = torch.zeros((m,) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        pad[: t.shape[0]] = t
        out = torch.empty((self.world * m,) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        self.dist.all_gather_into_tensor(out, pad, group=self.group)
        return [out[r * m: r * m + counts[r]] for r in range(self.world)]

    def all_to_all(self, parts: list[torch.Tensor]) -> list[torch.Tensor]:
        """parts[d] goes to rank d; returns what every rank sent here, in rank order."""
        dev = parts[0].device
        send_n = torch.tensor([p.shape[0] for p in parts], dtype=torch.int64, device=dev)
        recv_n = torch.empty_like(send_n)
        self.dist.all_to_all_single(recv_n, send_n, group=self.group)
        rn = [int(x) for x in recv_n.cpu()]
        tail = tuple(parts[0].shape[1:])
        send = torch.cat(parts) if parts else torch.empty((0,) + tail, dtype=parts[0].dtype, device=dev)
        recv = torch.empty((sum(rn),) + tail, dtype=send.dtype, device=dev)
        self.dist.all_to_all_single(recv, send, output_split_sizes=rn,
                                    input_split_sizes=[p.shape[0] for p in parts], group=self.group)
        return list(recv.split(rn))


class _Board:
    def __init__(self, world):
        self.world = world
        self.slots = [None] * world
        self.barrier = threading.Barrier(world)


class ThreadComm:
    """Ranks as threads of one process sharing one board; for emulating W shards on one GPU
    with the code path the distributed run takes."""

    def __init__(self, board: _Board, rank: int):
        self.board, self.rank, self.world = board, rank, board.world

    def _swap(self, obj):
        b = self.board
        b.barrier.wait()
        b.slots[self.rank] = obj
        b.barrier.wait()
        got = list(b.slots)
        b.barrier.wait()
        return got

    def all_gather(self, t):
        return self._swap(t)

    def all_to_all(self, parts):
        got = self._swap(list(parts))
        return [got[r][self.rank] for r in range(self.world)]

    def peer_values(self, t):
        return self._swap(t.data_ptr())          # one process: every rank's memory as it is

    def after_peer_reads(self, device):
        self.board.barrier.wait()                # every rank's gather is enqueued (one stream)


# ---------------------------------------------------------------------------- device ops
class CudaOps:
    """The per-rank device work, on this library's kernels."""

    def __init__(self, device, rows_per_head: int | None = None):
        self.device = device
        self.vrows = rows_per_head
        self.status = torch.zeros(1, dtype=torch.int32, device=device)

    def _stream(self):
        return torch.cuda.current_stream(self.device).cuda_stream

    def segment_match(self, qc, kc, seg_len):
        """-> src [H, L] (index within the segment or -1), lt_code/lt_pos [H * n_seg, seg_len],
        lt_count [H * n_seg]."""
        H, L = qc.shape
        n = H * (L // seg_len)
        src = torch.empty((H, L), dtype=torch.int32, device=self.device)
        ltc = torch.empty((n, seg_len), dtype=torch.int32, device=self.device)
        ltp = torch.empty((n, seg_len), dtype=torch.int32, device=self.device)
        ltn = torch.empty(n, dtype=torch.int32, device=self.device)
        wsb = int(_lib.lib().lema_segment_workspace_bytes(n, seg_len, 4))
        ws = torch.empty(wsb, dtype=torch.uint8, device=self.device) if wsb else None
        call("lema_segment_match", ptr(qc), ptr(kc), 4, n, seg_len, ptr(src), ptr(ltc), ptr(ltp),
             ptr(ltn), ptr(ws), wsb, ptr(self.status), self._stream())
        return src, ltc, ltp, ltn

    def rows_per_head(self, H: int, n_seg: int) -> int:
        """Independent sweep rows per head (rows_per_head, default 1). More rows sweep in
        parallel, but merging their tables into the shard's table costs more than that saves
        at config 5's sizes (measured at 2^25 x 16 positions: 1 row 45.7 ms, 2 rows 49.4 ms,
        4 rows 58.0 ms for the whole sweep phase)."""
        if self.vrows is not None:
            return self.vrows
        return 1

    def sweep(self, qc, src, lt, seg_len, base, want_table=True):
        """Segments in order, each head as V rows swept in parallel (a row's remaining misses then
        probe its head's earlier rows); returns the shard's LT re-hashed into a compact table,
        [H * slots] int64, for the other ranks."""
        ltc, ltp, ltn = lt
        H, L = qc.shape
        n_seg = L // seg_len
        V = self.rows_per_head(H, n_seg)
        R, Lr = H * V, L // V
        # distinct codes per row <= the sum of its segments' distinct codes, and <= its length
        per_row = torch.minimum(ltn.view(R, n_seg // V).sum(1, dtype=torch.int64),
                                torch.tensor(Lr, device=self.device)).tolist()
        slots = int(_lib.lib().lema_lt_table_slots(max(per_row)))
        table = torch.zeros((R, slots), dtype=torch.int64, device=self.device)
        call("lema_shard_sweep", ptr(table), R, slots, ptr(qc), ptr(src), Lr, seg_len, ptr(ltc),
             ptr(ltp), ptr(ltn), base, V, ptr(self.status), self._stream())
        call("lema_lt_resolve_rows", ptr(table), R, slots, V, ptr(qc), ptr(src), Lr, self._stream())
        if not want_table:                                   # a single rank: nobody asks
            return None
        cap = sum(per_row)
        ent = torch.empty((3, cap), dtype=torch.int32, device=self.device)
        cnt = torch.empty(1, dtype=torch.int32, device=self.device)
        call("lema_lt_extract", ptr(table), R, slots, base, ptr(ent[0]), ptr(ent[1]), ptr(ent[2]),
             ptr(cnt), cap, ptr(self.status), self._stream())
        del table
        if V > 1:
            ent[0].div_(V, rounding_mode="floor")            # row -> head
        # the shard's LT re-hashed into a table sized for it (what the other ranks receive)
        m = int(cnt.item())
        per_head = torch.bincount(ent[0, :m].long(), minlength=H)
        cslots = int(_lib.lib().lema_lt_table_slots(int(per_head.max()) if m else 1))
        compact = torch.zeros((H, cslots), dtype=torch.int64, device=self.device)
        call("lema_lt_insert", ptr(compact), H, cslots, ptr(ent[0]), ptr(ent[1]), ptr(ent[2]), m,
             ptr(self.status), self._stream())
        return compact.view(-1)

    def resolve(self, qc, src, earlier):
        """Queries with src == -1 probe the earlier shards' tables (a list, rank order; each
        [H * slots] int64), newest first."""
        if not earlier:
            return
        H, L = qc.shape
        tabs = [t.contiguous() for t in earlier]
        ptrs = torch.tensor([t.data_ptr() for t in tabs], dtype=torch.int64, device=self.device)
        slots = torch.tensor([t.numel() // H for t in tabs], dtype=torch.int64, device=self.device)
        call("lema_lt_resolve_tables", ptr(ptrs), ptr(slots), len(tabs), H, ptr(qc), ptr(src), L,
             self._stream())

    @staticmethod
    def rows(vflat, idx):
        return vflat.index_select(0, idx)

    def gather(self, src, base, v, remote_rows, remote_idx):
        H, L = src.shape
        vb = v[0, 0].numel() * v.element_size()
        out = torch.empty_like(v)
        call("lema_shard_gather", ptr(src), base, ptr(v), ptr(remote_rows), ptr(remote_idx), vb,
             ptr(out), H, L, ptr(self.status), self._stream())
        return out

    def gather_peer(self, src, base, v, peers):
        """The gather reading earlier shards' rows in place: peers[k] = rank k's values."""
        H, L = src.shape
        vb = v[0, 0].numel() * v.element_size()
        out = torch.empty_like(v)
        arr = (ctypes.c_void_p * len(peers))(*peers)
        call("lema_shard_gather_peer", ptr(src), base, arr, len(peers), vb, ptr(out), H, L,
             ptr(self.status), self._stream())
        return out

    def check(self):
        s = int(self.status.item())
        if s:
            self.status.zero_()
            what = "a hash table filled up" if s & LEMA_STATUS_TABLE_FULL else (
                "an internal bound ran out" if s & LEMA_STATUS_PROBE_LIMIT else f"status {s:#x}")
            raise LemaError(f"sharded prefill: {what}")


# ---------------------------------------------------------------------------- the protocol
def sharded_prefill(qc: torch.Tensor, kc: torch.Tensor, v: torch.Tensor, comm=None, ops=None,
                    seg_len: int = 4096, marks: list | None = None):
    """This rank's part of the exact op over one sharded sequence.

    qc, kc: [H, L] int32 (uint32 codes) of positions [rank * L, (rank + 1) * L); v: [H, L, d_v].
    Every rank passes the same H, L and seg_len (L a multiple of seg_len). Returns
    (src [H, L] int32 global positions or -1, out [H, L, d_v]). `marks`, if a list, receives
    (phase name, CUDA event recorded after it) for timing the phases."""
    comm = comm or SingleComm()
    if ops is None:
        ops = CudaOps(require_cuda(qc, kc, v))
    H, L = qc.shape
    if kc.shape != (H, L) or v.shape[:2] != (H, L):
        raise ValueError(f"shapes qc {tuple(qc.shape)}, kc {tuple(kc.shape)}, v {tuple(v.shape)}")
    if qc.dtype != torch.int32 or kc.dtype != torch.int32:
        raise ValueError("codes must be int32 (uint32 bit patterns)")
    if L % seg_len:
        raise ValueError(f"L = {L} is not a multiple of seg_len = {seg_len}")
    if comm.world * L >= 2 ** 31 - 1:
        raise ValueError("the sequence must stay below 2^31 - 1 positions")
    qc, kc, v = qc.contiguous(), kc.contiguous(), v.contiguous()
    base = comm.rank * L
    # the same decision on every rank: same comm and ops types and environment, then a
    # collective answer; LEMA_SHARD_PEER=0 keeps the request + all-to-all path (same results)
    peers = None
    if hasattr(ops, "gather_peer") and os.environ.get("LEMA_SHARD_PEER", "1")[:1] != "0":
        if comm.world == 1:
            peers = [v.data_ptr()]      # one rank: every source is its own (no requests to build)
        elif hasattr(comm, "peer_values"):
            peers = comm.peer_values(v)

    # 1-2: local work, no rank waits for another
    src, ltc, ltp, ltn = ops.segment_match(qc, kc, seg_len)
    _mark(marks, "segment_match")
    mine = ops.sweep(qc, src, (ltc, ltp, ltn), seg_len, base, want_table=comm.world > 1)
    del ltc, ltp, ltn
    _mark(marks, "sweep")
    # 3-4: the shards' last-occurrence tables
    tables = comm.all_gather(mine) if comm.world > 1 else [None]
    _mark(marks, "lt_all_gather")
    earlier = list(tables[: comm.rank])
    ops.resolve(qc, src, earlier)
    del tables, earlier
    _mark(marks, "resolve")

    if peers is not None:
        # 5-6: rows of earlier shards read in place (peer memory), own rows, zeros
        out = ops.gather_peer(src, base, v, peers)
        _mark(marks, "gather")
        if comm.world > 1:
            comm.after_peer_reads(src.device)
            _mark(marks, "release")
        ops.check()
        return src, out

    # 5: rows at earlier shards' positions, requested once each, in groups of heads
    vflat = v.view(H * L, -1).view(torch.uint8)           # rows as bytes, for transport
    remote_idx = torch.full((H, L), -1, dtype=torch.int32, device=src.device)
    want, where = [], []
    n_before = 0
    hg = max(1, min(H, (1 << 26) // max(L, 1)))           # heads per group: <= 64 M positions
    for h0 in range(0, H, hg):
        h1 = min(H, h0 + hg)
        s = src[h0:h1].reshape(-1)
        q = ((s >= 0) & (s < base)).nonzero().squeeze(1)   # flat index within the group
        p = s[q].long()
        owner = p // L
        key = owner * (H * L) + (q // L + h0) * L + (p - owner * L)  # owner-major, owner's row
        uniq, inv = torch.unique(key, return_inverse=True)
        want.append(uniq)
        where.append((h0, h1, q, inv + n_before))
        n_before += uniq.numel()
    uniq = torch.cat(want) if want else torch.empty(0, dtype=torch.int64, device=src.device)
    order = torch.sort(uniq // (H * L), stable=True)                # group by owner
    pos_of = torch.empty_like(order.indices)
    pos_of[order.indices] = torch.arange(order.indices.numel(), device=src.device)
    for h0, h1, q, j in where:
        remote_idx[h0:h1].view(-1)[q] = pos_of[j].to(torch.int32)
    req = uniq[order.indices]
    counts = torch.bincount(order.values, minlength=comm.world).tolist()
    send = list((req % (H * L)).split(counts))
    _mark(marks, "requests")
    asked = comm.all_to_all(send)                          # rows the other ranks want from me
    reply = [ops.rows(vflat, a) for a in asked]
    got = comm.all_to_all(reply)
    remote_rows = torch.cat(got) if got else vflat[:0]
    _mark(marks, "row_all_to_all")

    # 6
    out = ops.gather(src, base, v, remote_rows, remote_idx)
    _mark(marks, "gather")
    ops.check()
    return src, out


def _mark(marks, name):
    if marks is not None:
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        marks.append((name, e))


def emulated_sharded_prefill(qc: torch.Tensor, kc: torch.Tensor, v: torch.Tensor, n_shards: int,
                             seg_len: int = 4096):
    """The sharded computation over [H, T] inputs on ONE device: n_shards ranks as threads,
    each with its slice, through the same protocol a multi-GPU run takes. Returns the shards'
    (src, out) concatenated along the sequence."""
    H, T = qc.shape
    if T % n_shards:
        raise ValueError(f"T = {T} does not split into {n_shards} shards")
    L = T // n_shards
    board = _Board(n_shards)
    results: list = [None] * n_shards
    errors: list = []
    dev = qc.device

    def run(r):
        try:
            with torch.cuda.device(dev):
                sl = slice(r * L, (r + 1) * L)
                results[r] = sharded_prefill(qc[:, sl], kc[:, sl], v[:, sl], ThreadComm(board, r),
                                             CudaOps(dev), seg_len)
        except BaseException as e:  # noqa: BLE001 -- re-raised in the caller
            errors.append(e)
            board.barrier.abort()

    threads = [threading.Thread(target=run, args=(r,)) for r in range(n_shards)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    if errors:
        raise errors[0]
    return (torch.cat([s for s, _ in results], 1), torch.cat([o for _, o in results], 1))
