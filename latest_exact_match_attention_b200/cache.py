"""Inference store on the B200: the LEMA cache of code/lema/cache.py, moved into HBM.

At inference a LEMA head is a dictionary {code -> value of the latest position that emitted
that code as its key}; a position looks its query up, then inserts its key. The reference
runs that dictionary as one C++ hash table in host RAM (code/lema/cache.py:129-201,
code/lema/csrc/store.cpp) and moves codes and values across PCIe once per layer. Here the
same table -- one open-addressing table for every (layer, stream, head) partition, keyed by
(group, code), presized and never grown -- lives in device memory and the exchange is a
kernel (K3 in liblema_b200.so), so a decode step has no host phase and captures into a
single CUDA graph.

The classes and their methods mirror the reference's:

    HashStore    code/lema/cache.py:129-201   the table, counts, load, exchange
    Staging      code/lema/cache.py:205-222   one exchange's buffers (device-side here)
    Buffers      code/lema/cache.py:230-245   staging per size + the codes hook
    LayerStore   code/lema/cache.py:248-302   a layer's view: stage / host / fetch / exchange
    LemaCache    code/lema/cache.py:305-378   provisioning, layer views, counts / load

`stage`, `host` and `fetch` keep their meaning and order, but all three are device work:
`stage` applies the codes hook and lays the codes and values out item-major, `host`
launches the exchange kernel, `fetch` copies the retrieved rows out. Codes may be int64
(the reference's uint64 bit patterns) or int32 (uint32 bit patterns, d_qk <= 32).

A full table is reported by the kernel through a device status word; `exchange` checks it
(one synchronisation, as the reference's host exchange synchronises anyway) and raises the
reference's RuntimeError. Under a CUDA graph call `LemaCache.check()` after replays instead.
"""
from __future__ import annotations

import math

import numpy as np
import torch

from . import _lib
from ._lib import LEMA_STATUS_PROBE_LIMIT, LEMA_STATUS_TABLE_FULL, LemaError, call, ptr, stream_handle
from .attention import code_bytes_of

EMPTY = 0   # state word of a free slot: a zero-filled table is an empty table

# The store copies value rows and never interprets them; the dtype only fixes the row size.
_CARRIER = {torch.float32: torch.float32, torch.float16: torch.float16,
            torch.bfloat16: torch.bfloat16}
_NP_TO_TORCH = {np.dtype(np.float32): torch.float32, np.dtype(np.float16): torch.float16,
                np.dtype(np.uint16): torch.bfloat16}   # uint16 = the reference's bf16 carrier

FULL_MESSAGE = ("hash table full: the store is presized and never grows -- provision more "
                "capacity")


def _as_torch_dtype(dtype) -> torch.dtype:
    if isinstance(dtype, torch.dtype):
        if dtype not in _CARRIER:
            raise ValueError(f"store dtype must be float16, float32 or bfloat16, got {dtype}")
        return dtype
    try:
        return _NP_TO_TORCH[np.dtype(dtype)]
    except (TypeError, KeyError):
        raise ValueError(f"store dtype must be float16, float32, or uint16 (the carrier for "
                         f"bfloat16), got {dtype}") from None


class HashStore:
    """ONE open-addressing table in device memory for every (layer, stream, head) partition;
    an entry's key is the pair (group, code). Capacity is exact slots (any count, not a power
    of two), provisioned once; the table never grows and an overfull exchange raises.

    Slot = [code u64 | state u64 | value row] with the row padded to 16 bytes
    (`lema_store_slot_bytes`), so `nbytes()` is cap * slot bytes.
    """

    def __init__(self, d_v: int, groups: int, dtype=torch.bfloat16, capacity: int = 256,
                 device=None, segments: int = 1):
        self.dtype = _as_torch_dtype(dtype)
        self.d_v, self.groups = d_v, groups
        self.vbytes = d_v * torch.empty((), dtype=self.dtype).element_size()
        if self.vbytes % 8:
            raise ValueError(f"value row of {self.vbytes} bytes breaks slot alignment "
                             f"(d_v * itemsize must be a multiple of 8)")
        self.device = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        if self.device.type != "cuda":
            raise LemaError("the B200 store lives in device memory; device must be CUDA")
        self.stride = int(_lib.lib().lema_store_slot_bytes(self.vbytes))
        self.cap = max(16, int(capacity))
        self.table = torch.zeros((self.cap, self.stride), dtype=torch.uint8, device=self.device)
        self.counts = torch.zeros(groups, dtype=torch.int64, device=self.device)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._ws = None
        # segments > 1: each run of groups/segments groups (a layer, for LemaCache) has its
        # home slots in its own 1/segments of the table; results are the same either way
        segments = max(1, min(int(segments), groups, self.cap))
        self.seg_groups = -(-groups // segments) if segments > 1 else 0
        self.seg_slots = self.cap // segments if segments > 1 else 0

    def __len__(self):
        return int(self.counts.sum())

    def nbytes(self) -> int:
        return self.table.numel()

    def load(self) -> float:
        """Fraction of slots occupied."""
        return len(self) / self.cap

    def reserve(self, n: int, T: int, code_bytes: int = 8) -> None:
        """Allocate the exchange workspace for n items in chunks of T ahead of time (before a
        CUDA graph capture, say)."""
        self._workspace(n, T, code_bytes)

    def _workspace(self, n: int, T: int, code_bytes: int):
        need = int(_lib.lib().lema_store_workspace_bytes(n, T, code_bytes))
        if need == 0:
            return None
        if self._ws is None or self._ws.numel() < need:
            if torch.cuda.is_current_stream_capturing():
                raise LemaError("store workspace must be reserved before graph capture "
                                "(HashStore.reserve)")
            self._ws = torch.empty(need, dtype=torch.uint8, device=self.device)
        return self._ws

    def exchange(self, qcodes: torch.Tensor, kcodes: torch.Tensor, values: torch.Tensor,
                 out: torch.Tensor, T: int, g0: int, check: bool = True, rows=None):
        """One pass of P partitions x T positions against the store: item i (partition
        i // T, position i % T, group g0 + i // T) looks `qcodes[i]` up into `out[i]` (zeros
        on a miss) and then inserts `kcodes[i] -> values[i]`, each partition in position
        order. Device tensors: codes [n] int32/int64, values/out [n, d_v]. With `rows` =
        (heads, v_sb, v_sh, v_st, o_sb, o_sh, o_st) (bytes) the value and output rows of
        partition b * heads + h, position t are read and written at those strides instead
        (lema_store_exchange_strided): values and out may then be any views of that layout."""
        qcodes, kcodes = qcodes.reshape(-1), kcodes.reshape(-1)
        if qcodes.dtype != kcodes.dtype:
            kcodes = kcodes.to(qcodes.dtype)
        cb = code_bytes_of(qcodes)
        n = qcodes.numel()
        P = n // T if T else 0
        if g0 < 0 or g0 + P > self.groups:
            raise ValueError(f"groups [{g0}, {g0 + P}) outside the store's {self.groups}")
        if values.numel() != n * self.d_v or out.numel() != n * self.d_v or values.shape[-1] != self.d_v:
            raise ValueError(f"values and out must hold [n, d_v] = [{n}, {self.d_v}] rows, got "
                             f"{tuple(values.shape)} and {tuple(out.shape)}")
        if values.element_size() * values.shape[-1] != self.vbytes:
            raise ValueError(f"value rows of {values.element_size() * values.shape[-1]} bytes, "
                             f"the store holds {self.vbytes}")
        ws = self._workspace(n, T, cb)
        qcodes, kcodes = qcodes.contiguous(), kcodes.contiguous()
        if rows is None:
            if values.dim() != 2 or out.dim() != 2 or not out.is_contiguous():
                raise ValueError("values and out must be [n, d_v] (out contiguous), or pass rows=")
            values = values.contiguous()
            call("lema_store_exchange_seg", ptr(self.table), self.cap, self.vbytes, ptr(qcodes),
                 ptr(kcodes), cb, ptr(values), ptr(out), n, T, g0,
                 ptr(self.counts) + 8 * g0, ptr(self.status), ptr(ws), 0 if ws is None else ws.numel(),
                 self.seg_groups, self.seg_slots, stream_handle(self.device))
        else:
            call("lema_store_exchange_strided", ptr(self.table), self.cap, self.vbytes, ptr(qcodes),
                 ptr(kcodes), cb, ptr(values), ptr(out), n, T, g0,
                 ptr(self.counts) + 8 * g0, ptr(self.status), ptr(ws), 0 if ws is None else ws.numel(),
                 self.seg_groups, self.seg_slots, *rows, stream_handle(self.device))
        if check:
            self.check()

    def exchange_phase(self, qcodes: torch.Tensor, kcodes: torch.Tensor, values: torch.Tensor,
                       out: torch.Tensor, g0: int, phase: int):
        """Half of a decode step's exchange (T = 1, one item per partition): phase 1 looks every
        query up into `out`, phase 2 inserts every key -> value. Phase 1 then phase 2 equals
        `exchange(..., T=1)`; the inserts may run beside later work that needs only `out`."""
        if phase not in (1, 2):
            raise ValueError(f"phase must be 1 (lookups) or 2 (inserts), got {phase}")
        codes = qcodes if phase == 1 else kcodes
        n = codes.numel()
        if g0 < 0 or g0 + n > self.groups:
            raise ValueError(f"groups [{g0}, {g0 + n}) outside the store's {self.groups}")
        call("lema_store_exchange_phase", ptr(self.table), self.cap, self.vbytes,
             ptr(qcodes) if phase == 1 else None, ptr(kcodes) if phase == 2 else None,
             code_bytes_of(codes), ptr(values) if phase == 2 else None,
             ptr(out) if phase == 1 else None, n, g0, ptr(self.counts) + 8 * g0, ptr(self.status),
             self.seg_groups, self.seg_slots, phase, stream_handle(self.device))

    def dump(self):
        """Every entry of the store: (groups int64 [n], codes int64 [n], rows [n, d_v] in the
        store's dtype), in slot order. Codes are the stored 64-bit words (an int32 code's bit
        pattern zero-extended). Reads the table as it is on the device (synchronises)."""
        hdr = self.table.view(-1)[: 16 * self.cap].view(torch.int64).view(self.cap, 2)
        rows = self.table.view(-1)[16 * self.cap:].view(self.cap, self.stride - 16)
        live = (hdr[:, 1] >= 2).nonzero().squeeze(1)
        groups = hdr[live, 1] - 2
        codes = hdr[live, 0]
        vals = rows[live].view(self.dtype)[:, : self.d_v]
        return groups, codes, vals

    def check(self):
        """Raise if a kernel reported a full table (or an internal probe limit). Syncs."""
        s = int(self.status.item())
        if s:
            self.status.zero_()
            if s & LEMA_STATUS_TABLE_FULL:
                raise RuntimeError(FULL_MESSAGE)
            if s & LEMA_STATUS_PROBE_LIMIT:
                raise LemaError("internal: a bounded probe ran out")
            raise LemaError(f"store status {s:#x}")


class Staging:
    """One exchange's device buffers: query and key codes, the new value rows (item-major)
    and the retrieved rows. Unlike the reference's pinned host buffers these need no copy
    to cross a bus; they only fix the item-major layout."""

    __slots__ = ("n", "qc", "kc", "vals", "out", "T", "rows")

    def __init__(self, qc, kc, vals, out, T, rows=None):
        self.n, self.qc, self.kc, self.vals, self.out, self.T = qc.numel(), qc, kc, vals, out, T
        self.rows = rows  # strides of vals and out (a prefill chunk in place), or None


class Buffers:
    """What every layer's view shares besides the store: the codes hook and the per-size
    output buffers of graph-captured decoding."""

    def __init__(self, dtype, codes_hook=None):
        self.dtype, self.codes_hook = dtype, codes_hook
        self._out = {}

    def out(self, n: int, d_v: int, device) -> torch.Tensor:
        o = self._out.get(n)
        if o is None:
            o = self._out[n] = torch.empty(n, d_v, dtype=self.dtype, device=device)
        return o


class LayerStore:
    """One layer's view of the cache: its slice of partitions in the shared store. This is
    all a LEMA block is handed; the attention op only asks it to exchange codes for values.

        s = stage(qc, kc, v)     codes hook, item-major layout
        host(s)                  the exchange kernel
        fetch(s, got)            retrieved rows -> `got`

    `exchange` is the composition of the three.
    """

    __slots__ = ("store", "buffers", "g0", "partitions", "persistent_out")

    def __init__(self, store: HashStore, buffers: Buffers, g0: int, partitions: int):
        self.store, self.buffers, self.g0, self.partitions = store, buffers, g0, partitions
        self.persistent_out = False

    def stage(self, qc: torch.Tensor, kc: torch.Tensor, v: torch.Tensor) -> Staging:
        # [B, H, T] codes and [B, H, T, d_v] values flatten partition-major, position-minor,
        # which is the item order the store takes
        if self.buffers.codes_hook is not None:
            qc, kc = self.buffers.codes_hook(self.g0 // self.partitions, qc, kc)
        n, d_v = qc.numel(), v.shape[-1]
        T = n // self.partitions
        if T > 1 and not self.persistent_out and v.dim() == 4 and v.stride(-1) == 1:
            # a prefill chunk: the values are read where the projection left them ([B, T, H,
            # d_v] memory seen as [B, H, T, d_v]) and the retrieved rows written in the layout
            # the output projection reads, [B, T, H, d_v]: no copy either side
            B, H = v.shape[0], v.shape[1]
            es = v.element_size()
            out = torch.empty((B, T, H, d_v), dtype=v.dtype, device=v.device)
            rows = (H, v.stride(0) * es, v.stride(1) * es, v.stride(2) * es,
                    T * H * d_v * es, d_v * es, H * d_v * es)
            return Staging(qc.reshape(-1).contiguous(), kc.reshape(-1).contiguous(), v, out, T, rows)
        vals = v.reshape(-1, d_v)
        if not vals.is_contiguous():
            vals = vals.contiguous()
        out = (self.buffers.out(n, d_v, vals.device) if self.persistent_out
               else torch.empty(n, d_v, dtype=vals.dtype, device=vals.device))
        return Staging(qc.reshape(-1).contiguous(), kc.reshape(-1).contiguous(), vals, out, T)

    def host(self, s: Staging, check: bool = True):
        self.store.exchange(s.qc, s.kc, s.vals, s.out, s.T, self.g0, check=check, rows=s.rows)

    @staticmethod
    def retrieved(s: Staging, shape) -> torch.Tensor:
        """The retrieved rows as a [B, H, T, d_v] tensor (a view of the staging output)."""
        return s.out.transpose(1, 2) if s.rows is not None else s.out.view(shape)

    @staticmethod
    def fetch(s: Staging, got: torch.Tensor):
        got.copy_(LayerStore.retrieved(s, got.shape), non_blocking=True)

    def lookup(self, qc: torch.Tensor, kc: torch.Tensor, v: torch.Tensor):
        """The first half of a decode step's exchange (one position per partition): stages the
        step and looks every query up. Returns (staging, retrieved rows `[B, H, 1, d_v]`);
        `insert(staging)` is the second half, which must run before this layer's next lookup."""
        s = self.stage(qc, kc, v)
        if s.T != 1:
            raise ValueError(f"lookup/insert split one decode step (T = 1), got T = {s.T}")
        self.store.exchange_phase(s.qc, s.kc, s.vals, s.out, self.g0, 1)
        return s, self.retrieved(s, v.shape)

    def insert(self, s: Staging):
        """The second half of `lookup`'s step: every key of the step into the store."""
        self.store.exchange_phase(s.qc, s.kc, s.vals, s.out, self.g0, 2)

    def exchange(self, qc: torch.Tensor, kc: torch.Tensor, v: torch.Tensor,
                 check: bool = True) -> torch.Tensor:
        """Look up every query, fold in every key: the values each query retrieves,
        `[B, H, T, d_v]` like `v`, zeros where nothing matched."""
        s = self.stage(qc, kc, v)
        self.host(s, check=check and not torch.cuda.is_current_stream_capturing())
        return self.retrieved(s, v.shape)


class LemaCache:
    """The retrieval state of a model: one shared table in device memory, viewed per layer.

    Size it as the reference does: `max_cache_len` (slots = depth * batch * heads * len /
    max_load, the worst case of one distinct code per token) or `capacity` slots exactly.
    `pin` is accepted for signature compatibility and ignored (nothing crosses the bus).
    `codes_hook(layer, qc, kc) -> (qc, kc)` is applied on the device to every layer's
    [B, H, T] codes before the exchange.
    """

    def __init__(self, cfg, dtype=torch.bfloat16, pin: bool = True,
                 max_cache_len: int = 8192, max_load: float = 0.7,
                 batch: int = 1, capacity: int | None = None, codes_hook=None, device=None):
        if dtype not in _CARRIER:
            raise ValueError(f"cache dtype must be one of {list(_CARRIER)}, got {dtype}")
        if not 0 < max_load <= 0.95:
            raise ValueError(f"max_load must be in (0, 0.95], got {max_load}")
        P = batch * cfg.num_heads
        slots = int(capacity) if capacity else math.ceil(cfg.depth * P * max_cache_len / max_load)
        self.cfg, self.batch = cfg, batch
        self.store = HashStore(cfg.d_v, groups=cfg.depth * P, dtype=dtype, capacity=slots,
                               device=device, segments=cfg.depth)
        self.t = 0
        self.buffers = Buffers(dtype, codes_hook)
        self._views = [LayerStore(self.store, self.buffers, i * P, P) for i in range(cfg.depth)]

    def layer(self, i: int) -> LayerStore:
        return self._views[i]

    def counts(self) -> torch.Tensor:
        """Entries per partition as `[depth, batch, heads]` (a host copy)."""
        return self.store.counts.view(self.cfg.depth, self.batch, self.cfg.num_heads).cpu()

    def entries(self) -> int:
        return len(self.store)

    def nbytes(self) -> int:
        """Bytes the table reserves."""
        return self.store.nbytes()

    def load(self) -> float:
        return self.store.load()

    def check(self):
        """Raise if any exchange since the last check found the table full, or if a kernel of
        the model's steps (codes, MLP) reported that a bounded device wait ran out. Reads the
        device status words: call it after stepping (outside graph capture)."""
        self.store.check()
        _lib.check_status(self.store.device, "LEMA step")

    def dump(self, layer: int | None = None):
        """Entries as (layer, batch, head, code, row) tensors, all layers or one."""
        g, c, v = self.store.dump()
        P = self.batch * self.cfg.num_heads
        lay, rest = g // P, g % P
        if layer is not None:
            keep = lay == layer
            lay, rest, c, v = lay[keep], rest[keep], c[keep], v[keep]
        return lay, rest // self.cfg.num_heads, rest % self.cfg.num_heads, c, v


def worst_case_codes(depth: int):
    """A codes hook (LemaCache(codes_hook=...)) for stress runs: every layer's query AND key
    codes are replaced by fresh random 64-bit codes, so every lookup misses after probing its
    run and every insert claims a new slot at a random place -- the worst access pattern a
    model could produce (the stress mode of code/experiments/main_inference/common.py:170-196).
    All layers' codes are drawn at layer 0 in one kernel into a buffer the later layers view;
    inside a CUDA graph the generator advances on every replay, so each step draws anew."""
    bufs = {}

    def hook(layer, qc, kc):
        key = (qc.device, tuple(qc.shape))
        if layer == 0 or key not in bufs:
            if key not in bufs:
                bufs[key] = torch.empty((depth, 2) + tuple(qc.shape), dtype=torch.int64,
                                        device=qc.device)
            bufs[key].random_()
        b = bufs[key]
        return b[layer, 0], b[layer, 1]
    return hook
