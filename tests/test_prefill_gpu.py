"""K2 (latest exact match + gather) and the pack kernel on the GPU, through the C ABI,
against the reference's golden vectors and the CPU oracle. Bit-exact: indices are integers
and value rows are copied bytes."""
import numpy as np
import pytest
import torch

import oracle
from latest_exact_match_attention_b200 import latest_prev_match, lema_hard, pack_codes, prefill_match, synth
from tests import golden_data as G

pytestmark = pytest.mark.gpu


def as_dev_codes(a: np.ndarray, dev) -> torch.Tensor:
    """uint16/uint32 -> int32 bit patterns, uint64 -> int64 bit patterns, on the device."""
    if a.dtype.itemsize <= 4:
        return torch.from_numpy(a.astype(np.uint32).view(np.int32)).to(dev)
    return torch.from_numpy(a.astype(np.uint64).view(np.int64)).to(dev)


def run(qc, kc, v=None, dev=None):
    st = torch.zeros(1, dtype=torch.int32, device=dev)
    src, out = prefill_match(as_dev_codes(qc, dev), as_dev_codes(kc, dev),
                             None if v is None else torch.from_numpy(v).to(dev), status=st)
    torch.cuda.synchronize()
    assert int(st.item()) == 0, "device status raised"
    return src.cpu().numpy(), (None if out is None else out.cpu().numpy())


def test_config1_golden(cuda):
    g = G.load("config1")
    v = G.config1_values()
    src, out = run(g["qc"], g["kc"], v, cuda)
    np.testing.assert_array_equal(src, g["src"])
    assert G.sha(out) == str(g["out_sha"])


def test_config2_slice_golden(cuda):
    g = G.load("config2_slice")
    v = G.config2_values_u16()
    src, out = run(g["qc"], g["kc"], v, cuda)
    np.testing.assert_array_equal(src, g["src"])
    assert G.sha(out) == str(g["out_sha"])


@pytest.mark.parametrize("name", sorted(G.edge_cases()))
def test_edge_golden(cuda, name):
    qc, kc, want = G.edge_cases()[name]
    src, _ = run(qc, kc, None, cuda)
    np.testing.assert_array_equal(src, want)


@pytest.mark.parametrize("T", [1, 2, 31, 32, 33, 2047, 2048, 2049, 4097, 6144, 6145, 9000])
@pytest.mark.parametrize("width", [4, 8])
def test_random_vs_oracle(cuda, T, width):
    rng = np.random.default_rng(T * 10 + width)
    dt = np.uint32 if width == 4 else np.uint64
    for space in (7, 4000, 1 << 31):
        qc = rng.integers(0, space, size=(5, T)).astype(dt)
        kc = rng.integers(0, space, size=(5, T)).astype(dt)
        v = rng.integers(0, 1 << 16, size=(5, T, 24), dtype=np.uint16)
        src, out = run(qc, kc, v, cuda)
        want = oracle.latest_prev_match(qc, kc)
        np.testing.assert_array_equal(src, want)
        np.testing.assert_array_equal(out, oracle.gather(want, v))


@pytest.mark.parametrize("row", [(np.uint16, 1), (np.uint16, 2), (np.uint16, 3), (np.uint32, 2),
                                 (np.uint32, 3), (np.uint16, 24), (np.float32, 64), (np.uint8, 6)])
def test_value_row_widths(cuda, row):
    dt, d = row
    rng = np.random.default_rng(d)
    T = 3000
    qc = rng.integers(0, 50, size=(3, T)).astype(np.uint32)
    kc = rng.integers(0, 50, size=(3, T)).astype(np.uint32)
    v = (rng.integers(0, 200, size=(3, T, d)).astype(dt))
    src, out = run(qc, kc, v, cuda)
    np.testing.assert_array_equal(out, oracle.gather(oracle.latest_prev_match(qc, kc), v))


def test_unaligned_value_rows(cuda):
    """Rows that start off a 16-byte boundary take the narrower copy path."""
    rng = np.random.default_rng(9)
    T = 2500
    qc = rng.integers(0, 30, size=(2, T)).astype(np.uint32)
    kc = rng.integers(0, 30, size=(2, T)).astype(np.uint32)
    big = torch.from_numpy(rng.integers(0, 1 << 16, size=(2 * T * 24 + 1,), dtype=np.uint16)).to(cuda)
    v = big[1:].view(2, T, 24)                        # 2-byte aligned only
    src, out = prefill_match(as_dev_codes(qc, cuda), as_dev_codes(kc, cuda), v)
    want = oracle.latest_prev_match(qc, kc)
    np.testing.assert_array_equal(src.cpu().numpy(), want)
    np.testing.assert_array_equal(out.cpu().numpy(), oracle.gather(want, v.cpu().numpy()))


@pytest.mark.parametrize("segs", ["1", "2", ""])
def test_overflow_path_many_distinct(cuda, monkeypatch, segs):
    """More distinct key codes than the shared-memory table takes: the global-table path
    (one CTA per stream, or two segments of 8192 distinct keys each, both past the table's
    limit; by default eight segments of 2048, which fit and are resolved across segments)."""
    if segs:
        monkeypatch.setenv("LEMA_K2_SEGMENTS", segs)
    rng = np.random.default_rng(21)
    T = 16384
    # 3T distinct codes: an odd multiplier is a bijection modulo 2^30
    kc = ((np.arange(3 * T, dtype=np.uint64) * 2654435761 + 12345) & ((1 << 30) - 1)).astype(np.uint32).reshape(3, T)
    qc = kc.copy()
    for n in range(3):  # queries repeat keys from a little earlier, or miss
        back = rng.integers(-5, 200, size=T)
        idx = np.arange(T) - back
        ok = (idx >= 0) & (idx < T)
        qc[n, ok] = kc[n, idx[ok]]
        qc[n, ~ok] = rng.integers(1 << 30, 1 << 31, size=(~ok).sum())
    # stream 1 stays small (fast path) to mix both paths in one call
    kc[1] = rng.integers(0, 100, size=T)
    qc[1] = rng.integers(0, 100, size=T)
    v = rng.integers(0, 1 << 16, size=(3, T, 24), dtype=np.uint16)
    src, out = run(qc, kc, v, cuda)
    want = oracle.latest_prev_match(qc, kc)
    np.testing.assert_array_equal(src, want)
    np.testing.assert_array_equal(out, oracle.gather(want, v))


@pytest.mark.parametrize("segs", ["1", "2", "4", "8"])
@pytest.mark.parametrize("width", [4, 8])
def test_segmented_matcher(cuda, monkeypatch, segs, width):
    """Streams split over a cluster of 1 / 2 / 4 / 8 CTAs (runs of whole chunks; with 9 chunks
    and 8 CTAs the last runs are empty), misses resolved against the earlier runs' tables:
    small, medium and huge code spaces, the all-ones code (kept beside the table), a stream
    whose codes never repeat, and value rows -- against the oracle."""
    monkeypatch.setenv("LEMA_K2_SEGMENTS", segs)
    rng = np.random.default_rng(int(segs) * 10 + width)
    dt = np.uint32 if width == 4 else np.uint64
    ones = np.iinfo(dt).max
    T = 9000
    for space in (7, 4000, 1 << 31):
        qc = rng.integers(0, space, size=(6, T)).astype(dt)
        kc = rng.integers(0, space, size=(6, T)).astype(dt)
        qc[:, ::97] = ones
        kc[:, ::89] = ones
        kc[5] = np.arange(T, dtype=dt) * 3 + 1        # stream 5: every key new
        qc[5] = rng.integers(0, 3 * T, size=T).astype(dt)
        v = rng.integers(0, 1 << 16, size=(6, T, 24), dtype=np.uint16)
        src, out = run(qc, kc, v, cuda)
        want = oracle.latest_prev_match(qc, kc)
        np.testing.assert_array_equal(src, want)
        np.testing.assert_array_equal(out, oracle.gather(want, v))


def test_long_stream_direct_global_path(cuda):
    """T above the shared-memory path's range (2^20) goes straight to global tables."""
    rng = np.random.default_rng(33)
    T = (1 << 20) + 4096
    qc = rng.integers(0, 3000, size=(2, T)).astype(np.uint32)
    kc = rng.integers(0, 3000, size=(2, T)).astype(np.uint32)
    src, _ = run(qc, kc, None, cuda)
    np.testing.assert_array_equal(src, oracle.latest_prev_match(qc, kc))


def test_config2_full_size_vs_oracle(cuda):
    """The benchmark's shape (B=8, H=64, T=16384, 32-bit codes), every index and row."""
    from latest_exact_match_attention_b200 import synth
    qc, kc = synth.code_streams(512, 16384, synth.CONFIG2, seed=0, config_id=2)
    v = np.random.default_rng(1).integers(0, 1 << 16, size=(512, 16384, 24), dtype=np.uint16)
    src, out = run(qc, kc, v, cuda)
    want = oracle.latest_prev_match(qc, kc)
    np.testing.assert_array_equal(src, want)
    np.testing.assert_array_equal(out, oracle.gather(want, v))
    # size-independent properties, for the record
    i = np.arange(16384)[None]
    hit = src >= 0
    assert (src < i).all()
    assert (np.take_along_axis(kc, np.maximum(src, 0), 1)[hit] == qc[hit]).all()


def test_pack_codes_golden(cuda):
    g = G.load("pack")
    z = torch.from_numpy(g["z"]).to(cuda)
    assert torch.equal(pack_codes(z).cpu(), torch.from_numpy(g["codes64"]))
    assert torch.equal(pack_codes(z[..., :32]).cpu(), torch.from_numpy(g["codes32"]))
    assert torch.equal(pack_codes(z[..., :16]).cpu(), torch.from_numpy(g["codes16"]))
    n32 = pack_codes(z[..., :32], narrow=True).cpu()
    assert n32.dtype == torch.int32
    assert torch.equal(n32.numpy().view(np.uint32).astype(np.int64), g["codes32"]) if False else \
        np.array_equal(n32.numpy().view(np.uint32).astype(np.int64), g["codes32"])
    # bf16 / fp16 inputs pack their own signs
    for dt in (torch.bfloat16, torch.float16):
        zz = z.to(dt)
        want = oracle.pack_codes(zz.float().cpu().numpy()).view(np.int64)
        assert np.array_equal(pack_codes(zz).cpu().numpy(), want)


def test_pack_codes_strided_view(cuda):
    """The [B, H, T, d] transpose view that Attention.project returns."""
    rng = np.random.default_rng(4)
    B, T, H, D = 2, 300, 5, 32
    y = torch.from_numpy(rng.standard_normal((B, T, H * D)).astype(np.float32)).to(cuda).bfloat16()
    z = y.view(B, T, H, D).transpose(1, 2)
    got = pack_codes(z).cpu().numpy()
    want = oracle.pack_codes(z.float().cpu().contiguous().numpy()).view(np.int64)
    np.testing.assert_array_equal(got, want)


def test_latest_prev_match_api(cuda):
    g = G.load("config2_slice")
    qc = torch.from_numpy(g["qc"].astype(np.int64)).to(cuda)
    kc = torch.from_numpy(g["kc"].astype(np.int64)).to(cuda)
    src = latest_prev_match(qc, kc)
    assert src.dtype == torch.int64
    np.testing.assert_array_equal(src.cpu().numpy(), g["src"])


@pytest.mark.parametrize("d_qk,dtype", [(16, torch.float32), (32, torch.bfloat16), (64, torch.float32)])
def test_lema_hard_dense(cuda, d_qk, dtype):
    rng = np.random.default_rng(d_qk)
    B, H, T, dv = 2, 3, 1500, 8
    # few distinct sign patterns so that matches happen
    protos = rng.standard_normal((12, d_qk)).astype(np.float32)
    q = torch.from_numpy(protos[rng.integers(0, 12, size=(B, H, T))]).to(cuda, dtype)
    k = torch.from_numpy(protos[rng.integers(0, 12, size=(B, H, T))]).to(cuda, dtype)
    v = torch.from_numpy(rng.standard_normal((B, H, T, dv)).astype(np.float32)).to(cuda, dtype)
    y = lema_hard(q, k, v)
    qc = oracle.pack_codes(q.float().cpu().numpy()).reshape(B * H, T)
    kc = oracle.pack_codes(k.float().cpu().numpy()).reshape(B * H, T)
    want = oracle.lema_hard(qc, kc, v.cpu().view(B * H, T, dv).numpy() if dtype != torch.bfloat16
                            else v.cpu().view(torch.int16).view(B * H, T, dv).numpy())
    got = y.cpu() if dtype != torch.bfloat16 else y.cpu().view(torch.int16)
    np.testing.assert_array_equal(got.reshape(B * H, T, dv).numpy(), want)


@pytest.mark.parametrize("N,T", [(400, 2048), (340, 8192)])
def test_more_streams_than_one_matcher_wave(cuda, N, T):
    # more streams than one wave of matcher CTAs (2 per SM); T > 6144 also launches the
    # overflow kernel
    qc, kc = synth.code_streams(N, T, synth.CONFIG2, seed=N, config_id=2)
    v = np.random.default_rng(N).integers(0, 1 << 16, size=(N, T, 8), dtype=np.uint16)
    q = torch.from_numpy(qc.view(np.int32)).to(cuda)
    k = torch.from_numpy(kc.view(np.int32)).to(cuda)
    src, out = prefill_match(q, k, torch.from_numpy(v).to(cuda))
    want = oracle.latest_prev_match(qc, kc)
    assert np.array_equal(src.cpu().numpy(), want)
    assert np.array_equal(out.cpu().numpy(), oracle.gather(want, v))
