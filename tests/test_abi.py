"""liblema_b200.so loads, exports every entry point include/lema_b200.h declares, and rejects
bad arguments on the host before touching a device (no GPU needed)."""
import ctypes
import re
from pathlib import Path

import pytest
import torch

from latest_exact_match_attention_b200 import _lib
from latest_exact_match_attention_b200._lib import LemaError

HEADER = Path(__file__).resolve().parents[1] / "include" / "lema_b200.h"


def declared():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[\w\s\*]+?\b(lema_\w+)\s*\(", text, re.M)))


def test_header_declares_the_abi():
    names = declared()
    for must in ("lema_pack_codes", "lema_proj_codes", "lema_prefill_match",
                 "lema_prefill_workspace_bytes", "lema_store_exchange", "lema_store_slot_bytes",
                 "lema_store_workspace_bytes", "lema_last_error", "lema_version"):
        assert must in names


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    for name in declared():
        assert hasattr(L, name), f"{name} declared in lema_b200.h but not exported"
    assert L.lema_version() >= 100


def test_sizes():
    L = _lib.lib()
    assert L.lema_store_slot_bytes(48) == 64          # 16-byte header + 48-byte bf16 row
    assert L.lema_store_slot_bytes(256) == 272
    assert L.lema_store_slot_bytes(8) == 32           # rows padded to 16 bytes
    # index scratch (used when the caller passes no src) and the pipelined mode's control
    # words (4 KiB + 4 bytes per stream, 256-byte rounded) ...
    assert L.lema_prefill_workspace_bytes(8, 4096, 4) == 8 * 4096 * 4 + 4352
    # ... plus global-table room when a stream can outgrow the shared-memory table
    assert L.lema_prefill_workspace_bytes(512, 16384, 4) > 512 * 16384 * 4
    assert L.lema_store_workspace_bytes(1024, 1, 4) == 0        # a decode step needs none
    assert L.lema_store_workspace_bytes(8 * 4096, 4096, 8) > 0


def rc(name, *args):
    return getattr(_lib.lib(), name)(*args)


def test_argument_validation_on_host():
    P = ctypes.c_void_p(16)   # never dereferenced: every call below fails validation first
    # code width
    assert rc("lema_prefill_match", P, P, 3, 1, 8, None, None, 0, None, None, 0, None, None) == 1
    assert b"code_bytes" in _lib.lib().lema_last_error()
    # negative shapes
    assert rc("lema_prefill_match", P, P, 4, -1, 8, None, None, 0, None, None, 0, None, None) == 1
    # empty work is a no-op success
    assert rc("lema_prefill_match", None, None, 4, 0, 8, None, None, 0, None, None, 0, None, None) == 0
    # out without values
    assert rc("lema_prefill_match", P, P, 4, 1, 8, None, None, 48, P, None, 0, None, None) == 1
    # odd value row
    assert rc("lema_prefill_match", P, P, 4, 1, 8, None, P, 3, P, None, 0, None, None) == 1
    # workspace too small (config 2 needs one)
    assert rc("lema_prefill_match", P, P, 4, 512, 16384, None, None, 0, None, None, 0, None, None) == 3
    # the pipelined mode's control words (4 KiB + 4 bytes per stream, 256-byte rounded) are the
    # workspace's last bytes and optional: one byte less than the rest is refused, while the
    # rest alone passes validation (the call would run the two-kernel path) and, with no GPU
    # here, gets as far as looking for a device. Never run that half with a GPU present: the
    # pointers are fake.
    W = ctypes.c_void_p(1 << 20)   # 256-byte aligned, never dereferenced
    full = _lib.lib().lema_prefill_workspace_bytes(512, 16384, 4)
    ctl = (4112 + 4 * 512 + 255) // 256 * 256
    assert rc("lema_prefill_match", P, P, 4, 512, 16384, None, None, 0, None, W, full - ctl - 1, None, None) == 3
    assert b"needed" in _lib.lib().lema_last_error()
    if not torch.cuda.is_available():
        assert rc("lema_prefill_match", P, P, 4, 512, 16384, None, None, 0, None, W, full - ctl, None, None) == 2
    # store: value row not a multiple of 8, n not partitions x T, zero capacity
    assert rc("lema_store_exchange", P, 100, 12, P, P, 4, P, P, 8, 1, 0, P, None, None, 0, None) == 1
    assert rc("lema_store_exchange", P, 100, 16, P, P, 4, P, P, 10, 4, 0, P, None, None, 0, None) == 1
    assert rc("lema_store_exchange", P, 0, 16, P, P, 4, P, P, 8, 1, 0, P, None, None, 0, None) == 1
    # pack: d_qk too wide for the code width
    assert rc("lema_pack_codes", P, 0, 1, 1, 1, 0, 0, 0, 33, P, 4, None) == 1
    assert rc("lema_pack_codes", P, 0, 1, 1, 1, 0, 0, 0, 65, P, 8, None) == 1
    # projection: only d_qk = 32; K a multiple of 64; whole sequences of T rows
    assert rc("lema_proj_codes", P, P, 128, 64, 128, 1, 1, 16, P, P, None, None) == 1
    assert rc("lema_proj_codes", P, P, 128, 96, 128, 1, 1, 32, P, P, None, None) == 1
    assert rc("lema_proj_codes", P, P, 100, 64, 64, 1, 1, 32, P, P, None, None) == 1
    # fused gate/up GEMM + SwiGLU: K a multiple of 64, F of 128, no null pointers
    assert rc("lema_gemm_swiglu", P, P, 4096, 100, 128, P, None, None) == 1
    assert rc("lema_gemm_swiglu", P, P, 4096, 128, 100, P, None, None) == 1
    assert rc("lema_gemm_swiglu", P, None, 4096, 128, 128, P, None, None) == 1
    assert rc("lema_gemm_swiglu", None, None, 0, 128, 128, None, None, None) == 0   # no rows: no-op
    # RMSNorm: 16-bit rows only, D a multiple of 8 (else the caller's own norm), no nulls
    assert rc("lema_rms_norm", P, P, 0, 4, 64, ctypes.c_float(1e-5), P, None) == 4      # fp32
    assert rc("lema_rms_norm", P, P, 1, 4, 100, ctypes.c_float(1e-5), P, None) == 4     # D % 8
    assert rc("lema_rms_norm", P, None, 1, 4, 64, ctypes.c_float(1e-5), P, None) == 1
    assert rc("lema_rms_norm", None, None, 1, 0, 64, ctypes.c_float(1e-5), None, None) == 0


def test_python_layer_refuses_cpu_tensors():
    from latest_exact_match_attention_b200 import latest_prev_match, lema_hard, pack_codes
    q = torch.zeros(4, 8, dtype=torch.int32)
    with pytest.raises(LemaError, match="CUDA tensors only"):
        latest_prev_match(q, q)
    with pytest.raises(LemaError, match="CUDA tensors only"):
        pack_codes(torch.zeros(2, 32))
    with pytest.raises(LemaError, match="CUDA tensors only"):
        lema_hard(torch.zeros(1, 1, 4, 8), torch.zeros(1, 1, 4, 8), torch.zeros(1, 1, 4, 8))
