"""K2's pipelined mode (one launch: matcher CTAs on most SMs, row-copying CTAs on the rest,
following the matchers' published progress) against the two-kernel path and the oracle.
Calls of fewer streams than one wave of matchers (2 per SM: 296 on a B200) take the
two-kernel path; LEMA_K2_PIPELINE=0 selects it always; LEMA_K2_MATCH_FRAC moves the SM split.
Every case must give the same indices and rows bit for bit, and leave the status word 0
(no bounded wait ran out)."""
import numpy as np
import pytest
import torch

import oracle
from latest_exact_match_attention_b200 import _lib, prefill_match, synth
from latest_exact_match_attention_b200._lib import call, ptr

pytestmark = pytest.mark.gpu


def codes(N, T, seed, spec=synth.CONFIG2):
    qc, kc = synth.code_streams(N, T, spec, seed=seed, config_id=2)
    return qc, kc


def run(qc, kc, v, dev):
    st = torch.zeros(1, dtype=torch.int32, device=dev)
    src, out = prefill_match(torch.from_numpy(qc.view(np.int32)).to(dev),
                             torch.from_numpy(kc.view(np.int32)).to(dev),
                             torch.from_numpy(v).to(dev), status=st)
    torch.cuda.synchronize()
    assert int(st.item()) == 0, "device status raised"
    return src.cpu().numpy(), out.cpu().numpy()


@pytest.mark.parametrize("N,T,d", [
    (1, 20000, 24),      # one stream: the two-kernel path
    (296, 20000, 8),     # one full wave of matchers; 5 units per stream, the last ragged
    (600, 5000, 24),     # three waves of matchers, a ragged last unit and chunk
    (2048, 1024, 8),     # many one-chunk streams (one unit each)
    (300, 4096, 64),     # 128-byte rows, a unit = the whole stream
])
def test_pipe_equals_two_kernel_and_oracle(cuda, monkeypatch, N, T, d):
    qc, kc = codes(N, T, seed=N + T)
    v = np.random.default_rng(N).integers(0, 1 << 16, size=(N, T, d), dtype=np.uint16)
    src_p, out_p = run(qc, kc, v, cuda)
    monkeypatch.setenv("LEMA_K2_PIPELINE", "0")
    src_2, out_2 = run(qc, kc, v, cuda)
    assert np.array_equal(src_p, src_2)
    assert np.array_equal(out_p, out_2)
    want = oracle.latest_prev_match(qc, kc)
    assert np.array_equal(src_p, want)
    assert np.array_equal(out_p, oracle.gather(want, v))


@pytest.mark.parametrize("frac", ["0.05", "0.5", "1.0"])
def test_pipe_sm_split(cuda, monkeypatch, frac):
    # few matcher SMs (many waves, gather CTAs far ahead of the matchers) to none spare
    monkeypatch.setenv("LEMA_K2_MATCH_FRAC", frac)
    qc, kc = codes(700, 3000, seed=5)
    v = np.random.default_rng(5).integers(0, 1 << 16, size=(700, 3000, 24), dtype=np.uint16)
    src, out = run(qc, kc, v, cuda)
    want = oracle.latest_prev_match(qc, kc)
    assert np.array_equal(src, want)
    assert np.array_equal(out, oracle.gather(want, v))


def test_pipe_with_overflow_streams(cuda):
    # streams with more distinct keys than the shared-memory table leave the pipelined launch
    # part-way (their rows are copied by the overflow kernel); the others are piped
    rng = np.random.default_rng(12)
    N, T = 320, 12000
    qc, kc = codes(N, T, seed=12)
    for n in range(0, N, 37):
        # T distinct codes: an odd multiplier is a bijection modulo 2^30
        kc[n] = ((np.arange(T, dtype=np.uint64) * 2654435761 + 977 * n) & ((1 << 30) - 1)).astype(np.uint32)
        back = rng.integers(1, 300, size=T)
        idx = np.arange(T) - back
        ok = idx >= 0
        qc[n, ok] = kc[n, idx[ok]]
    v = rng.integers(0, 1 << 16, size=(N, T, 24), dtype=np.uint16)
    src, out = run(qc, kc, v, cuda)
    want = oracle.latest_prev_match(qc, kc)
    assert np.array_equal(src, want)
    assert np.array_equal(out, oracle.gather(want, v))


def test_pipe_strided_rows(cuda):
    # the model's layout: values [B, T, H, dv] read in place, output [B, T, H, dv]
    B, H, T, dv = 3, 100, 3000, 32
    qc, kc = codes(B * H, T, seed=3)
    vals = torch.from_numpy(np.random.default_rng(3).integers(0, 1 << 16, size=(B, T, H, dv),
                                                             dtype=np.uint16).view(np.int16)).to(cuda)
    out = torch.empty_like(vals)
    q = torch.from_numpy(qc.view(np.int32)).to(cuda)
    k = torch.from_numpy(kc.view(np.int32)).to(cuda)
    src = torch.empty((B * H, T), dtype=torch.int32, device=cuda)
    nb = int(_lib.lib().lema_prefill_workspace_bytes(B * H, T, 4))
    ws = torch.empty(nb, dtype=torch.uint8, device=cuda)
    st = torch.zeros(1, dtype=torch.int32, device=cuda)
    es = 2
    call("lema_prefill_match_strided", ptr(q), ptr(k), 4, B * H, T, ptr(src), ptr(vals), dv * es,
         ptr(out), H, T * H * dv * es, dv * es, H * dv * es, T * H * dv * es, dv * es, H * dv * es,
         ptr(ws), nb, ptr(st), torch.cuda.current_stream(cuda).cuda_stream)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    want = oracle.latest_prev_match(qc, kc)
    assert np.array_equal(src.cpu().numpy(), want)
    v_nt = vals.permute(0, 2, 1, 3).reshape(B * H, T, dv).cpu().numpy()
    got = out.permute(0, 2, 1, 3).reshape(B * H, T, dv).cpu().numpy()
    assert np.array_equal(got, oracle.gather(want, v_nt))


def test_pipe_repeated_calls_reuse_workspace(cuda):
    # the control words are cleared by every call: back-to-back calls on one workspace
    qc, kc = codes(400, 4096, seed=8)
    v = np.random.default_rng(8).integers(0, 1 << 16, size=(400, 4096, 24), dtype=np.uint16)
    q = torch.from_numpy(qc.view(np.int32)).to(cuda)
    k = torch.from_numpy(kc.view(np.int32)).to(cuda)
    vd = torch.from_numpy(v).to(cuda)
    want = oracle.latest_prev_match(qc, kc)
    wv = oracle.gather(want, v)
    st = torch.zeros(1, dtype=torch.int32, device=cuda)
    for _ in range(3):
        src, out = prefill_match(q, k, vd, status=st)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    assert np.array_equal(src.cpu().numpy(), want)
    assert np.array_equal(out.cpu().numpy(), wv)


def test_workspace_without_control_words_runs_two_kernels(cuda):
    # a workspace that holds everything but the pipelined mode's control words (its last
    # 4 KiB + 4 bytes per stream, 256-byte rounded) is accepted and gives the same results
    N, T = 300, 7000
    qc, kc = codes(N, T, seed=30)
    v = np.random.default_rng(30).integers(0, 1 << 16, size=(N, T, 24), dtype=np.uint16)
    q = torch.from_numpy(qc.view(np.int32)).to(cuda)
    k = torch.from_numpy(kc.view(np.int32)).to(cuda)
    vd = torch.from_numpy(v).to(cuda)
    full = int(_lib.lib().lema_prefill_workspace_bytes(N, T, 4))
    ctl = (4112 + 4 * N + 255) // 256 * 256
    want = oracle.latest_prev_match(qc, kc)
    wv = oracle.gather(want, v)
    for nb in (full, full - ctl):
        ws = torch.empty(nb, dtype=torch.uint8, device=cuda)
        src = torch.empty((N, T), dtype=torch.int32, device=cuda)
        out = torch.empty_like(vd)
        st = torch.zeros(1, dtype=torch.int32, device=cuda)
        call("lema_prefill_match", ptr(q), ptr(k), 4, N, T, ptr(src), ptr(vd), 48, ptr(out),
             ptr(ws), nb, ptr(st), torch.cuda.current_stream(cuda).cuda_stream)
        torch.cuda.synchronize()
        assert int(st.item()) == 0
        assert np.array_equal(src.cpu().numpy(), want)
        assert np.array_equal(out.cpu().numpy(), wv)
