"""K3, the HBM store, on the GPU through the C ABI: the reference's store tests
(code/tests/test_store.py shapes, golden outputs of its C++ store), config 1's prefill +
512 decode steps, the overfull error, and chunking invariance against the dense op
(code/tests/test_gpu.py:68-90's claim, at the op level)."""
import numpy as np
import pytest
import torch

import oracle
from latest_exact_match_attention_b200.cache import HashStore
from tests import golden_data as G

pytestmark = pytest.mark.gpu


def dev_codes(a, dev):
    a = np.ascontiguousarray(a)
    if a.dtype.itemsize <= 4:
        return torch.from_numpy(a.astype(np.uint32).view(np.int32)).to(dev)
    return torch.from_numpy(a.astype(np.int64)).to(dev)


@pytest.mark.parametrize("segments", [1, 7])
@pytest.mark.parametrize("name", sorted(G.store_cases()))
def test_reference_store_cases(cuda, name, segments):
    # segments: home slots of each run of groups in its own slice of the table (probing still
    # spans the table), which must change nothing in the results
    c = G.store_cases()[name]
    P, T, chunk = c["P"], c["T"], c["chunk"]
    vals = G.store_case_values(P, T, 8, c["seed"])
    st = HashStore(8, groups=P, dtype=torch.float16, capacity=c["cap"], device=cuda,
                   segments=segments)
    v16 = torch.from_numpy(vals.view(np.float16))
    outs = np.empty_like(vals)
    for lo in range(0, T, chunk):
        hi = min(T, lo + chunk)
        q = dev_codes(c["codes"][0, :, lo:hi].reshape(-1), cuda)
        k = dev_codes(c["codes"][1, :, lo:hi].reshape(-1), cuda)
        vv = v16[:, lo:hi].reshape(-1, 8).contiguous().to(cuda)
        o = torch.empty_like(vv)
        st.exchange(q, k, vv, o, hi - lo, 0)
        outs[:, lo:hi] = o.cpu().numpy().view(np.uint16).reshape(P, hi - lo, 8)
    np.testing.assert_array_equal(st.counts.cpu().numpy(), c["counts"])
    assert G.sha(outs) == c["out_sha"]


def test_overfull_raises(cuda):
    rng = np.random.default_rng(3)
    codes = rng.integers(0, 100, size=(2, 50, 100), dtype=np.int64) * 7919 % 102
    st = HashStore(8, groups=50, dtype=torch.float16, capacity=1000, device=cuda)
    v = torch.randn(5000, 8, device=cuda, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="full"):
        st.exchange(dev_codes(codes[0].reshape(-1), cuda), dev_codes(codes[1].reshape(-1), cuda),
                    v, torch.empty_like(v), 100, 0)
    # decode-sized steps raise too
    st = HashStore(8, groups=64, dtype=torch.float16, capacity=16, device=cuda)
    with pytest.raises(RuntimeError, match="full"):
        for t in range(3):
            c = torch.arange(64, device=cuda, dtype=torch.int32) + 64 * t
            st.exchange(c, c, v[:64], torch.empty_like(v[:64]), 1, 0)


@pytest.mark.parametrize("width", [4, 8])
def test_config1_prefill_then_decode(cuda, width):
    g = G.load("config1")
    v = G.config1_values()
    T0 = int(g["prefill_T"])
    qc, kc = g["qc"], g["kc"]
    if width == 8:
        qc, kc = qc.astype(np.int64), kc.astype(np.int64)
    st = HashStore(64, groups=8, dtype=torch.float32, capacity=8 * 4608 * 2, device=cuda)
    vd = torch.from_numpy(v).to(cuda)
    outs = torch.empty_like(vd)
    o = torch.empty(8 * T0, 64, device=cuda)
    st.exchange(dev_codes(qc[:, :T0].reshape(-1), cuda), dev_codes(kc[:, :T0].reshape(-1), cuda),
                vd[:, :T0].reshape(-1, 64), o, T0, 0)
    outs[:, :T0] = o.view(8, T0, 64)
    np.testing.assert_array_equal(st.counts.cpu().numpy(), g["counts_prefill"])
    qd, kd = dev_codes(qc, cuda), dev_codes(kc, cuda)
    step_out = torch.empty(8, 64, device=cuda)
    for t in range(T0, 4608):
        st.exchange(qd[:, t].contiguous(), kd[:, t].contiguous(), vd[:, t].contiguous(), step_out, 1, 0,
                    check=False)
        outs[:, t] = step_out
    st.check()
    np.testing.assert_array_equal(st.counts.cpu().numpy(), g["counts_final"])
    assert G.sha(outs.cpu().numpy()) == str(g["out_sha"])


@pytest.mark.parametrize("chunk", [1300, 64, 7, 1])
def test_chunking_invariance(cuda, chunk):
    """Fed in any chunking, the store reproduces the dense one-shot op exactly."""
    rng = np.random.default_rng(chunk)
    P, T = 12, 1300
    qc = rng.integers(0, 60, size=(P, T)).astype(np.uint32)
    kc = rng.integers(0, 60, size=(P, T)).astype(np.uint32)
    v = rng.standard_normal((P, T, 24)).astype(np.float32)
    dense = oracle.lema_hard(qc, kc, v)
    st = HashStore(24, groups=P + 5, dtype=torch.float32, capacity=P * T, device=cuda)
    vd = torch.from_numpy(v).to(cuda)
    got = torch.empty_like(vd)
    for lo in range(0, T, chunk):
        hi = min(T, lo + chunk)
        o = torch.empty(P * (hi - lo), 24, device=cuda)
        st.exchange(dev_codes(qc[:, lo:hi].reshape(-1), cuda), dev_codes(kc[:, lo:hi].reshape(-1), cuda),
                    vd[:, lo:hi].reshape(-1, 24), o, hi - lo, 5, check=False)
        got[:, lo:hi] = o.view(P, hi - lo, 24)
    st.check()
    np.testing.assert_array_equal(got.cpu().numpy(), dense)
    want_counts = [len(set(kc[p].tolist())) for p in range(P)]
    np.testing.assert_array_equal(st.counts.cpu().numpy()[5:], want_counts)
    assert st.counts[:5].sum().item() == 0


@pytest.mark.parametrize("segments", [1, 12])
def test_store_vs_oracle_store_random(cuda, segments):
    """Many partitions sharing a small code space, capacity tight: the GPU store and the
    oracle store agree call by call, including the counts (also with a segmented table,
    where full segments spill into their neighbours)."""
    rng = np.random.default_rng(17)
    P, T, cap = 300, 40, 20000
    tab = oracle.new_table(cap, 16)
    st = HashStore(8, groups=P, dtype=torch.float16, capacity=cap, device=cuda, segments=segments)
    for step in range(6):
        qc = rng.integers(0, 50, size=(P, T)).astype(np.int64)
        kc = rng.integers(0, 50, size=(P, T)).astype(np.int64)
        v = rng.integers(0, 1 << 16, size=(P * T, 8), dtype=np.uint16)
        want, added, full = oracle.store_exchange(tab, qc, kc, v, T, 0)
        assert not full
        vd = torch.from_numpy(v.view(np.float16)).to(cuda)
        o = torch.empty_like(vd)
        st.exchange(dev_codes(qc.reshape(-1), cuda), dev_codes(kc.reshape(-1), cuda), vd, o, T, 0)
        np.testing.assert_array_equal(o.cpu().numpy().view(np.uint16), want)
    counts = st.counts.cpu().numpy()
    assert counts.sum() == int((tab.view(np.uint64).reshape(cap, -1)[:, 1] != 0).sum())


@pytest.mark.parametrize("dv", [8, 64])
@pytest.mark.parametrize("group", ["8", "16", "32"])
@pytest.mark.parametrize("interleave", ["0", "1"])
def test_decode_steps_every_probe_mode(cuda, monkeypatch, interleave, group, dv):
    """Decode-sized exchanges (T = 1) in every probe mode -- lookup and insert probes one after
    the other or interleaved, 8 / 16 / 32 lanes per item -- against the oracle store, call by
    call: a small code space on a tight table (hits at home and down the chain, long chains,
    lost claims), a third of the items with query code == key code (both probes on the same
    slots: the lookup must return the row from before the step's own write), and rows of one
    (dv 8, fp16) or several (dv 64, fp32) 16-byte words per lane."""
    monkeypatch.setenv("LEMA_K3_INTERLEAVE", interleave)
    monkeypatch.setenv("LEMA_K3_GROUP", group)
    rng = np.random.default_rng(int(group) + 100 * int(interleave) + dv)
    P, cap = 400, 4000
    dtype, u = (torch.float16, np.uint16) if dv == 8 else (torch.float32, np.uint32)
    tab = oracle.new_table(cap, dv * np.dtype(u).itemsize)
    st = HashStore(dv, groups=P, dtype=dtype, capacity=cap, device=cuda)
    for step in range(12):
        qc = rng.integers(0, 12, size=(P, 1)).astype(np.int64)
        kc = rng.integers(0, 12, size=(P, 1)).astype(np.int64)
        same = rng.random(P) < 0.33
        kc[same, 0] = qc[same, 0]
        v = rng.integers(0, 1 << 16, size=(P, dv)).astype(u)
        want, added, full = oracle.store_exchange(tab, qc, kc, v, 1, 0)
        assert not full
        vd = torch.from_numpy(v.view(np.float16 if dv == 8 else np.float32)).to(cuda)
        o = torch.empty_like(vd)
        st.exchange(dev_codes(qc.reshape(-1), cuda), dev_codes(kc.reshape(-1), cuda), vd, o, 1, 0)
        np.testing.assert_array_equal(o.cpu().numpy().view(u), want)
    counts = st.counts.cpu().numpy()
    assert counts.sum() == int((tab.view(np.uint64).reshape(cap, -1)[:, 1] != 0).sum())


@pytest.mark.parametrize("dtype,dv", [(torch.bfloat16, 24), (torch.float32, 2), (torch.float16, 16)])
def test_strided_rows_equal_item_major(cuda, dtype, dv):
    """lema_store_exchange_strided on [B, T, H, d_v] value memory (seen as [B, H, T, d_v]) writing
    [B, T, H, d_v] output rows: the same store state, counts and retrieved rows as the
    item-major exchange, over prefill chunks and then single steps."""
    rng = np.random.default_rng(dv)
    B, H, T0, chunk, steps = 3, 5, 96, 32, 6
    Ttot = T0 + steps
    qc = rng.integers(0, 60, size=(B, H, Ttot)).astype(np.uint32)
    kc = rng.integers(0, 60, size=(B, H, Ttot)).astype(np.uint32)
    v_bthd = torch.from_numpy(rng.standard_normal((B, Ttot, H, dv)).astype(np.float32)).to(cuda, dtype)
    outs = []
    for strided in (False, True):
        st = HashStore(dv, groups=B * H, dtype=dtype, capacity=4 * B * H * Ttot, device=cuda)
        got = torch.empty((B, H, Ttot, dv), dtype=dtype, device=cuda)
        es = v_bthd.element_size()
        for t0 in list(range(0, T0, chunk)) + list(range(T0, Ttot)):
            t1 = t0 + (chunk if t0 < T0 else 1)
            q = dev_codes(qc[:, :, t0:t1].reshape(-1), cuda)
            k = dev_codes(kc[:, :, t0:t1].reshape(-1), cuda)
            vv = v_bthd[:, t0:t1].transpose(1, 2)              # [B, H, t, dv] view
            n, T = B * H * (t1 - t0), t1 - t0
            if strided:
                o = torch.empty((B, T, H, dv), dtype=dtype, device=cuda)
                rows = (H, vv.stride(0) * es, vv.stride(1) * es, vv.stride(2) * es,
                        T * H * dv * es, dv * es, H * dv * es)
                st.exchange(q, k, vv, o, T, 0, rows=rows)
                got[:, :, t0:t1] = o.transpose(1, 2)
            else:
                o = torch.empty((n, dv), dtype=dtype, device=cuda)
                st.exchange(q, k, vv.reshape(n, dv), o, T, 0)
                got[:, :, t0:t1] = o.view(B, H, T, dv)
        torch.cuda.synchronize()
        outs.append((got.cpu(), st.counts.cpu(), len(st)))
    assert torch.equal(outs[0][0].view(torch.uint8), outs[1][0].view(torch.uint8))
    assert torch.equal(outs[0][1], outs[1][1]) and outs[0][2] == outs[1][2]
    dense = oracle.lema_hard(qc.reshape(B * H, Ttot), kc.reshape(B * H, Ttot),
                             v_bthd.transpose(1, 2).reshape(B * H, Ttot, dv).contiguous().view(torch.uint8).cpu().numpy())
    assert np.array_equal(outs[1][0].view(torch.uint8).reshape(B * H, Ttot, -1).numpy(), dense)
