"""K2's dictionary + sweep matcher (the default for calls without value rows of at least one
wave of sweep CTAs) against the oracle and the chunked matcher. LEMA_K2_SWEEP=1 makes every
call it can serve take it (value rows are then copied by the gather kernel), =0 turns it off;
the results must not depend on the path, bit for bit."""
import numpy as np
import pytest
import torch

import oracle
from latest_exact_match_attention_b200 import _lib, prefill_match, synth
from latest_exact_match_attention_b200._lib import call, ptr
from tests import golden_data as G

pytestmark = pytest.mark.gpu


def dev_codes(a, dev):
    if a.dtype.itemsize <= 4:
        return torch.from_numpy(a.astype(np.uint32).view(np.int32)).to(dev)
    return torch.from_numpy(a.astype(np.uint64).view(np.int64)).to(dev)


def run(qc, kc, v, dev):
    st = torch.zeros(1, dtype=torch.int32, device=dev)
    src, out = prefill_match(dev_codes(qc, dev), dev_codes(kc, dev),
                             None if v is None else torch.from_numpy(v).to(dev), status=st)
    torch.cuda.synchronize()
    assert int(st.item()) == 0, "device status raised"
    return src.cpu().numpy(), None if out is None else out.cpu().numpy()


@pytest.fixture
def sweep(monkeypatch):
    monkeypatch.setenv("LEMA_K2_SWEEP", "1")


@pytest.mark.parametrize("T", [1, 31, 32, 33, 511, 512, 513, 4608, 6145, 16384, 65535])
@pytest.mark.parametrize("width", [4, 8])
def test_sweep_random_vs_oracle(cuda, sweep, T, width):
    rng = np.random.default_rng(T * 7 + width)
    dt = np.uint32 if width == 4 else np.uint64
    n = 3 if T < 60000 else 1
    for space in (5, 3000, 1 << 31):
        qc = rng.integers(0, space, size=(n, T)).astype(dt)
        kc = rng.integers(0, space, size=(n, T)).astype(dt)
        v = rng.integers(0, 1 << 16, size=(n, T, 8), dtype=np.uint16)
        src, out = run(qc, kc, v, cuda)
        want = oracle.latest_prev_match(qc, kc)
        np.testing.assert_array_equal(src, want)
        np.testing.assert_array_equal(out, oracle.gather(want, v))


@pytest.mark.parametrize("name", sorted(G.edge_cases()))
def test_sweep_edge_golden(cuda, sweep, name):
    qc, kc, want = G.edge_cases()[name]
    src, _ = run(qc, kc, None, cuda)
    np.testing.assert_array_equal(src, want)


def test_sweep_golden_config1_and_slice(cuda, sweep):
    g = G.load("config1")
    src, out = run(g["qc"], g["kc"], G.config1_values(), cuda)
    np.testing.assert_array_equal(src, g["src"])
    assert G.sha(out) == str(g["out_sha"])
    g = G.load("config2_slice")
    src, out = run(g["qc"], g["kc"], G.config2_values_u16(), cuda)
    np.testing.assert_array_equal(src, g["src"])
    assert G.sha(out) == str(g["out_sha"])


def test_sweep_all_ones_and_overflow_streams(cuda, sweep):
    """The all-ones code (the table's free marker) as an ordinary key, and streams with more
    distinct keys than the table takes (the overflow path), in one call."""
    rng = np.random.default_rng(5)
    N, T = 6, 12000
    kc = rng.integers(0, 40, size=(N, T)).astype(np.uint32)
    qc = rng.integers(0, 40, size=(N, T)).astype(np.uint32)
    kc[0, ::7] = 0xFFFFFFFF
    qc[0, 3::5] = 0xFFFFFFFF
    for n in (2, 4):   # T distinct codes: an odd multiplier is a bijection modulo 2^30
        kc[n] = ((np.arange(T, dtype=np.uint64) * 2654435761 + 31 * n) & ((1 << 30) - 1)).astype(np.uint32)
        back = rng.integers(1, 300, size=T)
        idx = np.arange(T) - back
        ok = idx >= 0
        qc[n, ok] = kc[n, idx[ok]]
    v = rng.integers(0, 1 << 16, size=(N, T, 24), dtype=np.uint16)
    src, out = run(qc, kc, v, cuda)
    want = oracle.latest_prev_match(qc, kc)
    np.testing.assert_array_equal(src, want)
    np.testing.assert_array_equal(out, oracle.gather(want, v))


def test_sweep_default_for_match_only_calls(cuda, monkeypatch):
    """Config 2's shape without value rows: the default (sweep) equals the chunked matcher."""
    qc, kc = synth.code_streams(320, 16384, synth.CONFIG2, seed=4, config_id=2)
    q, k = dev_codes(qc, cuda), dev_codes(kc, cuda)
    a, _ = prefill_match(q, k)
    monkeypatch.setenv("LEMA_K2_SWEEP", "0")
    b, _ = prefill_match(q, k)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    np.testing.assert_array_equal(a.cpu().numpy(), oracle.latest_prev_match(qc, kc))


def test_sweep_last_occurrence_tables(cuda, sweep):
    """lema_segment_match's per-stream last-occurrence tables from the sweep path."""
    rng = np.random.default_rng(8)
    N, T = 5, 3000
    qc = rng.integers(0, 400, size=(N, T)).astype(np.uint32)
    kc = rng.integers(0, 400, size=(N, T)).astype(np.uint32)
    kc[1, 10] = 0xFFFFFFFF
    q, k = dev_codes(qc, cuda), dev_codes(kc, cuda)
    src = torch.empty((N, T), dtype=torch.int32, device=cuda)
    ltc = torch.empty((N, T), dtype=torch.int32, device=cuda)
    ltp = torch.empty((N, T), dtype=torch.int32, device=cuda)
    cnt = torch.empty(N, dtype=torch.int32, device=cuda)
    nb = int(_lib.lib().lema_segment_workspace_bytes(N, T, 4))
    ws = torch.empty(max(nb, 1), dtype=torch.uint8, device=cuda)
    st = torch.zeros(1, dtype=torch.int32, device=cuda)
    call("lema_segment_match", ptr(q), ptr(k), 4, N, T, ptr(src), ptr(ltc), ptr(ltp), ptr(cnt),
         ptr(ws), nb, ptr(st), torch.cuda.current_stream(cuda).cuda_stream)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    np.testing.assert_array_equal(src.cpu().numpy(), oracle.latest_prev_match(qc, kc))
    for n in range(N):
        c = int(cnt[n])
        got = dict(zip(ltc[n, :c].cpu().numpy().view(np.uint32).tolist(), ltp[n, :c].cpu().tolist()))
        want = {}
        for j, code in enumerate(kc[n].tolist()):
            want[code] = j
        assert got == want
