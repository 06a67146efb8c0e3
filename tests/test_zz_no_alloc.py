"""lema_prefill_match_noalloc, the matcher for callers that cannot allocate device memory
(a plugin handed only its input and output tensors by an engine that owns all device memory,
a C caller with no device allocator, a loop where cudaMalloc / cudaFree are not allowed).
Its scratch is a fixed array inside liblema_b200.so, so it takes no workspace argument.

It must give exactly the results of lema_prefill_match (the workspace entry point) -- indices
and copied value rows are bit-exact -- on two calls in a row, since every call reuses the one
scratch array and keeps whatever the previous call left there. This file is named to be
collected last: a failure here leaves every other test already run.
"""
import numpy as np
import pytest
import torch

from latest_exact_match_attention_b200 import prefill_match, synth
from latest_exact_match_attention_b200._lib import LemaError, call, lib, ptr, stream_handle

pytestmark = pytest.mark.gpu


def noalloc(q, k, v, want_src=True):
    N, T = q.shape
    dev = q.device
    src = torch.empty((N, T), dtype=torch.int32, device=dev) if want_src else None
    out = torch.empty_like(v) if v is not None else None
    vbytes = v[0, 0].numel() * v.element_size() if v is not None else 0
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    call("lema_prefill_match_noalloc", ptr(q), ptr(k), q.element_size(), N, T, ptr(src), ptr(v),
         vbytes, ptr(out), ptr(status), stream_handle(dev))
    return src, out, status


def config2_case(dev, n, seed):
    qc, kc = synth.code_streams(n, 16384, synth.CONFIG2, seed=seed, config_id=2)
    v = torch.from_numpy(np.random.default_rng(seed).integers(0, 1 << 16, size=(n, 16384, 24),
                                                              dtype=np.uint16)).to(dev)
    return (torch.from_numpy(qc.view(np.int32)).to(dev), torch.from_numpy(kc.view(np.int32)).to(dev), v)


def distinct_case(dev):
    """Streams with more distinct key codes than the on-chip table takes: the overflow path
    runs, with its tables in the fixed scratch array."""
    rng = np.random.default_rng(5)
    T = 12000
    kc = rng.permutation(1 << 28)[: 3 * T].astype(np.uint32).reshape(3, T)
    qc = kc.copy()
    for n in range(3):
        back = rng.integers(1, 300, size=T)
        idx = np.arange(T) - back
        qc[n] = np.where(idx >= 0, kc[n, np.maximum(idx, 0)], rng.integers(1 << 29, 1 << 30, size=T))
    v = torch.from_numpy(rng.standard_normal((3, T, 16)).astype(np.float32)).to(dev)
    return (torch.from_numpy(qc.view(np.int32)).to(dev), torch.from_numpy(kc.view(np.int32)).to(dev), v)


def small_case(dev):
    rng = np.random.default_rng(9)
    qc = rng.integers(0, 300, size=(96, 3000)).astype(np.int64)
    kc = rng.integers(0, 300, size=(96, 3000)).astype(np.int64)
    v = torch.from_numpy(rng.standard_normal((96, 3000, 4)).astype(np.float32)).to(dev)
    return torch.from_numpy(qc).to(dev), torch.from_numpy(kc).to(dev), v


@pytest.mark.parametrize("want_src", [True, False])
def test_noalloc_equals_workspace_entry_point_twice(cuda, want_src):
    # two different calls in a row through the shared scratch, each against the workspace path
    for q, k, v in (config2_case(cuda, 48, 3), distinct_case(cuda), small_case(cuda), config2_case(cuda, 40, 4)):
        src_ref, out_ref = prefill_match(q, k, v)
        src, out, status = noalloc(q, k, v, want_src=want_src)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        if want_src:
            assert torch.equal(src, src_ref)
        assert torch.equal(out.view(torch.uint8), out_ref.view(torch.uint8))


def test_noalloc_pipelined_mode_and_sweep_twice(cuda, monkeypatch):
    """At least one wave of matchers (296 streams) of 32-bit codes with 16-byte rows and src
    passed: the call takes the pipelined mode, whose control block and per-stream progress
    words also live in the shared array (cleared by every call); without value rows the same
    streams take the dictionary + sweep matcher. Two calls in a row each, then the two-kernel
    path (LEMA_K2_PIPELINE=0) through the same array."""
    q, k, v = config2_case(cuda, 320, 6)
    src_ref, out_ref = prefill_match(q, k, v)
    for _ in range(2):
        src, out, status = noalloc(q, k, v)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert torch.equal(src, src_ref) and torch.equal(out, out_ref)
        src, _, status = noalloc(q, k, None)
        torch.cuda.synchronize()
        assert int(status.item()) == 0 and torch.equal(src, src_ref)
    monkeypatch.setenv("LEMA_K2_PIPELINE", "0")
    src, out, status = noalloc(q, k, v)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert torch.equal(src, src_ref) and torch.equal(out, out_ref)


def test_noalloc_rejects_oversized_calls(cuda):
    # the indices of 512 x 16384 positions alone fill the 32 MiB; the overflow counter, list
    # and one overflow-path table on top of them do not fit
    q = torch.zeros((512, 16384), dtype=torch.int32, device=cuda)
    v = torch.zeros((512, 16384, 24), dtype=torch.bfloat16, device=cuda)
    with pytest.raises(LemaError, match="scratch"):
        noalloc(q, q, v, want_src=False)
    assert lib().lema_version() >= 100
