"""The CPU oracle pinned against the reference: golden vectors made by the reference's own
code (tests/golden/make_golden.py), and the reference's C++ store compiled from its source
(oracle/_ref) where it was built."""
import numpy as np
import pytest

import oracle
from tests import golden_data as G


def test_config1_indices_and_store_outputs():
    g = G.load("config1")
    v = G.config1_values()
    assert G.sha(v) == str(g["values_sha"]), "value regeneration drifted"
    src = oracle.latest_prev_match(g["qc"], g["kc"])
    np.testing.assert_array_equal(src, g["src"])
    assert G.sha(oracle.gather(src, v)) == str(g["out_sha"])
    # the oracle store, prefill chunk then 512 single-step exchanges (the reference's path)
    T0 = int(g["prefill_T"])
    qc, kc = g["qc"].astype(np.int64), g["kc"].astype(np.int64)
    tab = oracle.new_table(8 * 4608 * 2, 256)
    outs = np.empty_like(v)
    o, added, full = oracle.store_exchange(tab, qc[:, :T0], kc[:, :T0], v[:, :T0].reshape(-1, 64), T0, 0)
    outs[:, :T0] = o.reshape(8, T0, 64)
    np.testing.assert_array_equal(added, g["counts_prefill"])
    counts = added.copy()
    for t in range(T0, 4608):
        o, added, full = oracle.store_exchange(tab, qc[:, t], kc[:, t], v[:, t], 1, 0)
        outs[:, t] = o
        counts += added
        assert not full
    np.testing.assert_array_equal(counts, g["counts_final"])
    assert G.sha(outs) == str(g["out_sha"])


def test_config2_slice():
    g = G.load("config2_slice")
    v = G.config2_values_u16()
    assert G.sha(v) == str(g["values_sha"])
    src = oracle.latest_prev_match(g["qc"], g["kc"])
    np.testing.assert_array_equal(src, g["src"])
    assert G.sha(oracle.gather(src, v)) == str(g["out_sha"])


@pytest.mark.parametrize("name", sorted(G.edge_cases()))
def test_edge_cases(name):
    qc, kc, src = G.edge_cases()[name]
    np.testing.assert_array_equal(oracle.latest_prev_match(qc, kc), src)


def test_pack_codes():
    g = G.load("pack")
    np.testing.assert_array_equal(oracle.pack_codes(g["z"]).view(np.int64), g["codes64"])
    np.testing.assert_array_equal(oracle.pack_codes(g["z"][..., :32]).view(np.int64), g["codes32"])
    np.testing.assert_array_equal(oracle.pack_codes(g["z"][..., :16]).view(np.int64), g["codes16"])


@pytest.mark.parametrize("name", sorted(G.store_cases()))
def test_store_cases(name):
    c = G.store_cases()[name]
    P, T, chunk = c["P"], c["T"], c["chunk"]
    vals = G.store_case_values(P, T, 8, c["seed"])
    assert G.sha(vals) == c["values_sha"]
    tab = oracle.new_table(c["cap"], 16)
    outs = np.empty_like(vals)
    counts = np.zeros(P, np.int64)
    for lo in range(0, T, chunk):
        hi = min(T, lo + chunk)
        o, added, full = oracle.store_exchange(tab, c["codes"][0, :, lo:hi], c["codes"][1, :, lo:hi],
                                               vals[:, lo:hi].reshape(-1, 8), hi - lo, 0)
        assert not full
        outs[:, lo:hi] = o.reshape(P, hi - lo, 8)
        counts += added
    np.testing.assert_array_equal(counts, c["counts"])
    assert G.sha(outs) == c["out_sha"]


def test_store_overfull():
    rng = np.random.default_rng(3)
    codes = rng.integers(0, 100, size=(2, 50, 100), dtype=np.int64) * 7919 % 102
    vals = rng.integers(0, 1 << 16, size=(50 * 100, 8), dtype=np.uint16)
    _, _, full = oracle.store_exchange(oracle.new_table(1000, 16), codes[0], codes[1], vals, 100, 0)
    assert full


def test_oracle_store_equals_dense_in_any_chunking():
    rng = np.random.default_rng(5)
    P, T = 6, 700
    qc = rng.integers(0, 40, size=(P, T)).astype(np.uint32)
    kc = rng.integers(0, 40, size=(P, T)).astype(np.uint32)
    v = rng.standard_normal((P, T, 4)).astype(np.float32)
    dense = oracle.lema_hard(qc, kc, v)
    for chunk in (T, 64, 7, 1):
        tab = oracle.new_table(P * T * 2, 16)
        got = np.empty_like(v)
        for lo in range(0, T, chunk):
            hi = min(T, lo + chunk)
            o, _, _ = oracle.store_exchange(tab, qc[:, lo:hi], kc[:, lo:hi], v[:, lo:hi].reshape(-1, 4), hi - lo, 0)
            got[:, lo:hi] = o.reshape(P, hi - lo, 4)
        np.testing.assert_array_equal(got, dense)


@pytest.mark.skipif(oracle.ref_path() is None, reason="oracle/_ref not built (reference absent)")
def test_reference_store_agrees_with_oracle():
    import torch
    ref = oracle.ref_store()
    rng = np.random.default_rng(11)
    for P, T, n_codes, cap in [(30, 500, 60, 20000), (100, 1, 5, 400), (7, 1000, 1 << 30, 16000)]:
        qc = rng.integers(0, n_codes, size=(P, T)).astype(np.int64)
        kc = rng.integers(0, n_codes, size=(P, T)).astype(np.int64)
        v = rng.integers(0, 1 << 16, size=(P * T, 8)).astype(np.uint16)
        out, added, full = oracle.store_exchange(oracle.new_table(cap, 16), qc, kc, v, T, 3)
        tab = torch.zeros((cap, 32), dtype=torch.uint8)
        ro = torch.empty((P * T, 8), dtype=torch.uint16)
        ra = ref.exchange(tab, torch.from_numpy(qc.reshape(-1)), torch.from_numpy(kc.reshape(-1)),
                          torch.from_numpy(v), ro, T, 3, cap, 16)
        np.testing.assert_array_equal(ro.numpy(), out)
        np.testing.assert_array_equal(ra.numpy(), added)
