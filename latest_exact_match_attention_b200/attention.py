"""The exact LEMA op on the B200: the inference half of code/lema/attention.py.

    pack_codes(z)              code/lema/attention.py:82-97    sign bits -> one code per row
    latest_prev_match(qc, kc)  code/lema/attention.py:100-132  latest earlier matching key
    lema_hard(q, k, v, store)  code/lema/attention.py:135-158  the exact op, dense or stored

Same names, argument meanings and results as the reference; the work runs in the sm_100a
kernels of liblema_b200.so (K2 for the match and gather, the pack kernel for the codes).
Conventions are the reference's: codes are sum_d [z_d >= 0] << d (sign(0) = +1), matching
is STRICTLY causal (a query never sees its own key), and no match gives -1 / zeros.

Differences, all deliberate:
  * CUDA tensors only -- there is no CPU path (a CPU tensor raises);
  * inference only -- the outputs carry no autograd graph (the reference's gather keeps a
    value gradient for training, which is out of scope here);
  * with d_qk <= 32 the op works on 32-bit codes internally (pack_codes(z, narrow=True));
    `pack_codes(z)` itself still returns int64 like the reference.
The training-time surrogates (hard_sign, binarize, lema_soft, lema) are not part of this
package.
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import DTYPE_TAG, LemaError, call, check_status, device_status, ptr, require_cuda, stream_handle

__all__ = ["pack_codes", "proj_codes", "latest_prev_match", "lema_hard", "prefill_match",
           "prefill_match_host", "HostPrefill", "proj_codes_v", "row_rms", "code_bytes_of"]


def code_bytes_of(codes: torch.Tensor) -> int:
    if codes.dtype == torch.int32:
        return 4
    if codes.dtype == torch.int64:
        return 8
    raise LemaError(f"codes must be int32 (uint32 bit patterns) or int64 (uint64 bit "
                    f"patterns), got {codes.dtype}")


def pack_codes(z: torch.Tensor, narrow: bool = False) -> torch.Tensor:
    """[..., D] -> one integer code per row, on z's device: bit d is (z[..., d] >= 0).

    Returns int64 like the reference (at D = 64 the top bit makes the value negative;
    only equality is ever used). `narrow=True` with D <= 32 returns int32 holding the
    uint32 bit pattern instead, the form the kernels prefer.
    """
    require_cuda(z)
    D = z.shape[-1]
    if D > 64:
        raise ValueError(f"d_qk {D} > 64 cannot pack into a uint64")
    if z.dtype not in DTYPE_TAG:
        z = z.float()
    if z.stride(-1) != 1:
        z = z.contiguous()
    lead = tuple(z.shape[:-1])
    if len(lead) > 3:
        z = z.reshape(-1, D)
    dims = list(z.shape[:-1])
    strides = list(z.stride()[:-1])
    while len(dims) < 3:
        dims.insert(0, 1)
        strides.insert(0, 0)
    narrow = narrow and D <= 32
    out = torch.empty(lead, dtype=torch.int32 if narrow else torch.int64, device=z.device)
    if out.numel() == 0:
        return out
    call("lema_pack_codes", ptr(z), DTYPE_TAG[z.dtype], dims[0], dims[1], dims[2],
         strides[0], strides[1], strides[2], D, ptr(out), 4 if narrow else 8,
         stream_handle(z.device))
    return out


def proj_codes(x: torch.Tensor, w_qk: torch.Tensor, hq: int, hk: int,
               status: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Query and key codes of `x` [B, T, dim] under the stacked projection weights
    `w_qk` [(hq + hk) * 32, dim] (q_proj.weight over k_proj.weight), both bf16:
    the codes of `pack_codes(x @ w_qk.T)` per head, without z ever reaching memory.

    Returns (qcodes [B, hq, T], kcodes [B, hk, T]) as int32 holding uint32 bit patterns.
    The tensor-core GEMM accumulates in fp32, so a bit can differ from a bf16 GEMM followed
    by pack_codes only where that pre-activation is within rounding of zero.
    Mirrors code/lema/model.py:224-227 (`Block.gpu_pre`) minus the norm and v_proj.
    Device-side conditions go to `status`, or to the package's status word of the device
    (`_lib.check_status` raises on them).
    """
    dev = require_cuda(x, w_qk)
    if x.dtype != torch.bfloat16 or w_qk.dtype != torch.bfloat16:
        raise LemaError("proj_codes takes bf16 x and w_qk")
    if x.dim() != 3 or w_qk.dim() != 2 or w_qk.shape != ((hq + hk) * 32, x.shape[-1]):
        raise LemaError(f"shapes x {tuple(x.shape)}, w_qk {tuple(w_qk.shape)} do not fit "
                        f"hq={hq}, hk={hk}, d_qk=32")
    x = x.contiguous()
    w_qk = w_qk.contiguous()
    B, T, dim = x.shape
    qc = torch.empty((B, hq, T), dtype=torch.int32, device=dev)
    kc = torch.empty((B, hk, T), dtype=torch.int32, device=dev)
    if status is None:
        status = device_status(dev)
    call("lema_proj_codes", ptr(x), ptr(w_qk), B * T, dim, T, hq, hk, 32, ptr(qc), ptr(kc),
         ptr(status), stream_handle(dev))
    return qc, kc


def row_rms(x: torch.Tensor, eps: float) -> torch.Tensor:
    """1 / sqrt(mean(x^2, -1) + eps) per row of a bf16 [..., K] tensor, fp32 [rows]."""
    dev = require_cuda(x)
    x = x.contiguous()
    K = x.shape[-1]
    out = torch.empty(x.numel() // K, dtype=torch.float32, device=dev)
    call("lema_row_rms", ptr(x), out.numel(), K, float(eps), ptr(out), stream_handle(dev))
    return out


def proj_codes_v(x: torch.Tensor, w_all: torch.Tensor, hq: int, hk: int, n_v: int,
                 row_scale: torch.Tensor | None = None, status: torch.Tensor | None = None):
    """Codes and values in one tcgen05 GEMM: `w_all` [(hq + hk) * 32 + n_v, dim] stacks the
    query, key and value projection weights (bf16). Returns (qcodes [B, hq, T], kcodes
    [B, hk, T], v [B, T, n_v] bf16 = row_scale * (x @ w_v.T))."""
    dev = require_cuda(x, w_all, row_scale)
    if x.dtype != torch.bfloat16 or w_all.dtype != torch.bfloat16:
        raise LemaError("proj_codes_v takes bf16 x and w_all")
    B, T, dim = x.shape
    if w_all.shape != ((hq + hk) * 32 + n_v, dim):
        raise LemaError(f"w_all {tuple(w_all.shape)} does not fit hq={hq}, hk={hk}, n_v={n_v}")
    x, w_all = x.contiguous(), w_all.contiguous()
    qc = torch.empty((B, hq, T), dtype=torch.int32, device=dev)
    kc = torch.empty((B, hk, T), dtype=torch.int32, device=dev)
    v = torch.empty((B, T, n_v), dtype=torch.bfloat16, device=dev)
    if status is None:
        status = device_status(dev)
    call("lema_proj_codes_v", ptr(x), ptr(w_all), B * T, dim, T, hq, hk, 32, ptr(qc), ptr(kc),
         n_v, ptr(v), ptr(row_scale), ptr(status), stream_handle(dev))
    return qc, kc, v


def _workspace(nbytes: int, device) -> torch.Tensor | None:
    # the caching allocator hands out 512-byte aligned blocks, above the 256 required
    return torch.empty(nbytes, dtype=torch.uint8, device=device) if nbytes else None


def prefill_match(qc: torch.Tensor, kc: torch.Tensor, v: torch.Tensor | None = None, *,
                  want_src: bool = True, status: torch.Tensor | None = None):
    """The native K2 call: `qc`, `kc` [N, T] codes (int32 or int64, one dtype), `v` [N, T,
    ...] value rows (optional). Returns (src, out): src [N, T] int32 (latest j < i with an
    equal key code, else -1) when want_src, out like v with the gathered rows (zeros on a
    miss) when v is given. Device status bits are OR-ed into `status` (an int32 [1] device
    tensor) when given, else into the package's status word of the device, which
    `_lib.check_status` reads."""
    dev = require_cuda(qc, kc, v, status)
    if qc.dim() != 2 or qc.shape != kc.shape:
        raise ValueError(f"qc and kc must be [N, T] of one shape, got {tuple(qc.shape)} and "
                         f"{tuple(kc.shape)}")
    if qc.dtype != kc.dtype:
        raise ValueError(f"qc and kc must share a dtype, got {qc.dtype} and {kc.dtype}")
    cb = code_bytes_of(qc)
    N, T = qc.shape
    qc, kc = qc.contiguous(), kc.contiguous()
    src = torch.empty((N, T), dtype=torch.int32, device=dev) if want_src else None
    out = vbytes = None
    if v is not None:
        if v.shape[:2] != (N, T):
            raise ValueError(f"values must be [N, T, ...] = [{N}, {T}, ...], got {tuple(v.shape)}")
        v = v.contiguous()
        out = torch.empty_like(v)
        vbytes = v[0, 0].numel() * v.element_size() if N * T else 0
    ws = _workspace(_lib.lib().lema_prefill_workspace_bytes(N, T, cb), dev)
    if status is None and N * T:
        status = device_status(dev)
    call("lema_prefill_match", ptr(qc), ptr(kc), cb, N, T, ptr(src), ptr(v), vbytes or 0,
         ptr(out), ptr(ws), 0 if ws is None else ws.numel(), ptr(status), stream_handle(dev))
    return src, out


def latest_prev_match(qc: torch.Tensor, kc: torch.Tensor) -> torch.Tensor:
    """For each i, the largest j < i with kc[j] == qc[i], else -1 (int64 [N, T], as
    code/lema/attention.py:100-132 returns). Raises LemaError if a device-side bound ran out
    (the check reads the device status word, so the call returns once the kernels are done;
    inside a CUDA graph capture it is skipped)."""
    src, _ = prefill_match(qc, kc)
    check_status(src.device, "latest_prev_match")
    return src.to(torch.int64)


def lema_hard(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, store=None) -> torch.Tensor:
    """Exact latest match: o_i = v_j for the largest j < i with k_j == q_i, else 0.

    q, k: [B, H, T, d_qk] binarized codes OR raw pre-activations (only their signs are
    read); v: [B, H, T, d_v]. With a `store` (a LayerStore) the rule is one exchange
    against it, so this window's queries also see every key fed before; without one it is
    a self-contained forward over the window. Returns [B, H, T, d_v] in v's dtype.
    Raises LemaError if a device-side bound ran out (see latest_prev_match).
    """
    B, H, T, D = q.shape
    narrow = D <= 32
    qc, kc = pack_codes(q, narrow=narrow), pack_codes(k, narrow=narrow)
    if store is not None:
        return store.exchange(qc, kc, v)
    d_v = v.shape[-1]
    _, out = prefill_match(qc.view(B * H, T), kc.view(B * H, T),
                           v.reshape(B * H, T, d_v), want_src=False)
    check_status(out.device, "lema_hard")
    return out.view(B, H, T, d_v)


class HostPrefill:
    """`prefill_match` for inputs and outputs in HOST memory (pinned for overlap), streamed
    through the device in batches of `batch` streams. The host->device copies of batch b+1,
    the kernels of batch b and the device->host copies of batch b-1 run at once on three CUDA
    streams, so the call costs about the slower copy direction instead of the sum of both.
    Device buffers (`slots` batches in flight, so that neither copy direction waits for the
    other's slot) and the three streams are allocated once; one instance serves calls of its
    shape. The call returns once the work is queued; the host outputs are complete when the
    caller's current stream reaches that point."""

    def __init__(self, device, T: int, code_dtype=torch.int32, row_shape=(), row_dtype=None,
                 batch: int = 64, want_src: bool = True, slots: int = 3):
        self.device = torch.device(device)
        self.T, self.batch, self.want_src = T, batch, want_src
        self.slots = max(2, int(slots))
        self.code_dtype = code_dtype
        self.cb = torch.empty((), dtype=code_dtype).element_size()
        mk = lambda shape, dt: [torch.empty(shape, dtype=dt, device=self.device) for _ in range(self.slots)]
        self.dq = mk((batch, T), code_dtype)
        self.dk = mk((batch, T), code_dtype)
        none = [None] * self.slots
        self.dsrc = mk((batch, T), torch.int32) if want_src else none
        self.has_v = row_dtype is not None
        self.dv = mk((batch, T) + tuple(row_shape), row_dtype) if self.has_v else none
        self.dout = mk((batch, T) + tuple(row_shape), row_dtype) if self.has_v else none
        self.vbytes = (self.dv[0][0, 0].numel() * self.dv[0].element_size()) if self.has_v else 0
        nb = int(_lib.lib().lema_prefill_workspace_bytes(batch, T, self.cb))
        self.ws = _workspace(nb, self.device)
        self.streams = [torch.cuda.Stream(self.device) for _ in range(3)]

    def __call__(self, qc, kc, v=None, src_out=None, out=None, status=None):
        s_in, s_cp, s_out = self.streams
        cur = torch.cuda.current_stream(self.device)
        if status is None:
            status = device_status(self.device)
        N = qc.shape[0]
        for s in self.streams:
            s.wait_stream(cur)
        ev_cp, ev_out = [], []
        S = self.slots
        for b, n0 in enumerate(range(0, N, self.batch)):
            n, j = min(self.batch, N - n0), b % S
            with torch.cuda.stream(s_in):
                if b >= S:
                    s_in.wait_event(ev_cp[b - S])        # slot j's inputs were read
                self.dq[j][:n].copy_(qc[n0:n0 + n], non_blocking=True)
                self.dk[j][:n].copy_(kc[n0:n0 + n], non_blocking=True)
                if self.has_v:
                    self.dv[j][:n].copy_(v[n0:n0 + n], non_blocking=True)
                e_in = torch.cuda.Event()
                e_in.record(s_in)
            with torch.cuda.stream(s_cp):
                s_cp.wait_event(e_in)
                if b >= S:
                    s_cp.wait_event(ev_out[b - S])       # slot j's outputs were copied out
                call("lema_prefill_match", ptr(self.dq[j]), ptr(self.dk[j]), self.cb, n, self.T,
                     ptr(self.dsrc[j]), ptr(self.dv[j]), self.vbytes, ptr(self.dout[j]),
                     ptr(self.ws), 0 if self.ws is None else self.ws.numel(), ptr(status),
                     s_cp.cuda_stream)
                e = torch.cuda.Event()
                e.record(s_cp)
                ev_cp.append(e)
            with torch.cuda.stream(s_out):
                s_out.wait_event(e)
                if self.want_src and src_out is not None:
                    src_out[n0:n0 + n].copy_(self.dsrc[j][:n], non_blocking=True)
                if self.has_v and out is not None:
                    out[n0:n0 + n].copy_(self.dout[j][:n], non_blocking=True)
                e = torch.cuda.Event()
                e.record(s_out)
                ev_out.append(e)
        for s in self.streams:
            cur.wait_stream(s)


def prefill_match_host(qc: torch.Tensor, kc: torch.Tensor, v: torch.Tensor | None = None, *,
                       device=None, batch: int = 64, want_src: bool = True):
    """`prefill_match` on host tensors: returns (src, out) as pinned host tensors, filled once
    the current stream of `device` (default: the current CUDA device) has run the queued work
    (synchronise before reading them)."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    N, T = qc.shape
    run = HostPrefill(dev, T, qc.dtype, tuple(v.shape[2:]) if v is not None else (),
                      v.dtype if v is not None else None, batch=min(batch, max(N, 1)),
                      want_src=want_src)
    src = torch.empty((N, T), dtype=torch.int32).pin_memory() if want_src else None
    out = torch.empty(v.shape, dtype=v.dtype).pin_memory() if v is not None else None
    run(qc, kc, v, src, out)
    return src, out
