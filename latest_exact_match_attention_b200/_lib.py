"""ctypes binding of liblema_b200.so (the C ABI in include/lema_b200.h).

The library is loaded from this package's directory, where build.py writes it. There is no
fallback: if it is missing or fails to load, every entry point raises LemaError.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().with_name("liblema_b200.so")

LEMA_OK = 0
LEMA_STATUS_TABLE_FULL = 0x1
LEMA_STATUS_PROBE_LIMIT = 0x2
F32, BF16, F16 = 0, 1, 2
DTYPE_TAG = {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16}


class LemaError(RuntimeError):
    """A failing call into liblema_b200.so."""


_lib = None
_lock = threading.Lock()

_P, _I64, _I, _SZ = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_size_t
_SIGNATURES = {
    "lema_last_error": ([], ctypes.c_char_p),
    "lema_version": ([], _I),
    "lema_pack_codes": ([_P, _I, _I64, _I64, _I64, _I64, _I64, _I64, _I, _P, _I, _P], _I),
    "lema_proj_codes": ([_P, _P, _I64, _I64, _I64, _I, _I, _I, _P, _P, _P, _P], _I),
    "lema_proj_codes_v": ([_P, _P, _I64, _I64, _I64, _I, _I, _I, _P, _P, _I64, _P, _P, _P, _P], _I),
    "lema_row_rms": ([_P, _I64, _I64, ctypes.c_float, _P, _P], _I),
    "lema_swiglu": ([_P, _I, _I64, _I64, _P, _P], _I),
    "lema_rms_norm": ([_P, _P, _I, _I64, _I64, ctypes.c_float, _P, _P], _I),
    "lema_gemm_swiglu": ([_P, _P, _I64, _I64, _I64, _P, _P, _P], _I),
    "lema_prefill_workspace_bytes": ([_I64, _I64, _I], _SZ),
    "lema_prefill_match": ([_P, _P, _I, _I64, _I64, _P, _P, _I64, _P, _P, _SZ, _P, _P], _I),
    "lema_prefill_match_noalloc": ([_P, _P, _I, _I64, _I64, _P, _P, _I64, _P, _P, _P], _I),
    "lema_prefill_match_strided": ([_P, _P, _I, _I64, _I64, _P, _P, _I64, _P, _I64, _I64, _I64,
                                    _I64, _I64, _I64, _I64, _P, _SZ, _P, _P], _I),
    "lema_store_exchange_seg": ([_P, _I64, _I64, _P, _P, _I, _P, _P, _I64, _I64, _I64, _P, _P,
                                 _P, _SZ, _I64, _I64, _P], _I),
    "lema_store_exchange_phase": ([_P, _I64, _I64, _P, _P, _I, _P, _P, _I64, _I64, _P, _P, _I64,
                                   _I64, _I, _P], _I),
    "lema_store_exchange_strided": ([_P, _I64, _I64, _P, _P, _I, _P, _P, _I64, _I64, _I64, _P, _P,
                                     _P, _SZ, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64,
                                     _P], _I),
    "lema_segment_workspace_bytes": ([_I64, _I64, _I], _SZ),
    "lema_segment_match": ([_P, _P, _I, _I64, _I64, _P, _P, _P, _P, _P, _SZ, _P, _P], _I),
    "lema_lt_table_slots": ([_I64], _I64),
    "lema_lt_insert": ([_P, _I64, _I64, _P, _P, _P, _I64, _P, _P], _I),
    "lema_lt_resolve": ([_P, _I64, _I64, _P, _P, _I64, _P], _I),
    "lema_lt_resolve_tables": ([_P, _P, _I, _I64, _P, _P, _I64, _P], _I),
    "lema_lt_extract": ([_P, _I64, _I64, ctypes.c_int32, _P, _P, _P, _P, _I64, _P, _P], _I),
    "lema_shard_sweep": ([_P, _I64, _I64, _P, _P, _I64, _I64, _P, _P, _P, _I64, _I64, _P, _P], _I),
    "lema_lt_resolve_rows": ([_P, _I64, _I64, _I64, _P, _P, _I64, _P], _I),
    "lema_shard_gather": ([_P, _I64, _P, _P, _P, _I64, _P, _I64, _I64, _P, _P], _I),
    "lema_shard_gather_peer": ([_P, _I64, _P, _I, _I64, _P, _I64, _I64, _P, _P], _I),
    "lema_ipc_export": ([_P, _P, _P], _I),
    "lema_ipc_import": ([_P, _I64, _P], _I),
    "lema_ipc_close": ([_P, _I64], _I),
    "lema_store_slot_bytes": ([_I64], _I64),
    "lema_store_workspace_bytes": ([_I64, _I64, _I], _SZ),
    "lema_store_exchange": ([_P, _I64, _I64, _P, _P, _I, _P, _P, _I64, _I64, _I64, _P, _P, _P,
                             _SZ, _P], _I),
}


def lib() -> ctypes.CDLL:
    """The loaded library (raises LemaError when it is not built)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise LemaError(
                        f"{LIB_PATH.name} is not built: run `python -m "
                        f"latest_exact_match_attention_b200.build` (needs nvcc); there is no "
                        f"CPU fallback")
                try:
                    L = ctypes.CDLL(str(LIB_PATH))
                except OSError as e:
                    raise LemaError(f"could not load {LIB_PATH}: {e}") from e
                for name, (args, res) in _SIGNATURES.items():
                    fn = getattr(L, name)
                    fn.argtypes = args
                    fn.restype = res
                _lib = L
    return _lib


def call(name: str, *args) -> None:
    """Call an entry point that returns a status code; raise LemaError on failure."""
    rc = getattr(lib(), name)(*args)
    if rc != LEMA_OK:
        msg = lib().lema_last_error().decode(errors="replace")
        raise LemaError(f"{name} failed (code {rc}): {msg}")


_status_words: dict[int, torch.Tensor] = {}


def device_status(device) -> torch.Tensor:
    """The package's status word on `device` (int32 [1], zero-initialised): every product call
    that is given no status word of its own ORs its device-side conditions into it (a bounded
    wait that ran out, a full table). Allocated on first use, which must not be inside a CUDA
    graph capture (one eager call first: the decoder's warm-up steps make it)."""
    dev = torch.device(device)
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    st = _status_words.get(idx)
    if st is None:
        if torch.cuda.is_current_stream_capturing():
            raise LemaError("the device status word is allocated on first use: make one call "
                            "outside CUDA graph capture first")
        st = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _status_words[idx] = st
    return st


def check_status(device, what: str = "LEMA kernel") -> None:
    """Raise LemaError if a call that used the package's status word on `device` reported a
    device-side condition since the last check (then clear the word). Reads the word, so it
    waits for the work queued so far; does nothing inside a CUDA graph capture (check after
    the replay instead)."""
    dev = torch.device(device)
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    st = _status_words.get(idx)
    if st is None or torch.cuda.is_current_stream_capturing():
        return
    s = int(st.item())
    if s:
        st.zero_()
        raise LemaError(status_message(s, what))


def status_message(s: int, what: str) -> str:
    parts = []
    if s & LEMA_STATUS_PROBE_LIMIT:
        parts.append("a bounded device-side wait or probe ran out: the outputs are incomplete")
    if s & LEMA_STATUS_TABLE_FULL:
        parts.append("hash table full")
    rest = s & ~(LEMA_STATUS_PROBE_LIMIT | LEMA_STATUS_TABLE_FULL)
    if rest:
        parts.append(f"status bits {rest:#x}")
    return f"{what}: " + "; ".join(parts)


def stream_handle(device: torch.device | None = None) -> int:
    """The raw cudaStream_t of torch's current stream on `device`."""
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    """All tensors on one CUDA device; the product path has no CPU implementation."""
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise LemaError("LEMA B200 kernels take CUDA tensors only (there is no CPU path); "
                            f"got a tensor on {t.device}")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise LemaError(f"tensors on different devices: {dev} and {t.device}")
    return dev
