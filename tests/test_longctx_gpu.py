"""Sequence-sharded prefill (config 5's path) on one GPU: W shards emulated as threads through
the protocol a multi-GPU run takes (latest_exact_match_attention_b200.longctx), checked
bit-exact against ONE pass of the matcher over the whole sequence -- which the oracle and
golden tests pin to the reference's latest_prev_match -- and, on a small case, against the
oracle directly."""
import numpy as np
import pytest
import torch

import oracle
from latest_exact_match_attention_b200 import prefill_match, synth
from latest_exact_match_attention_b200.longctx import emulated_sharded_prefill, sharded_prefill

pytestmark = pytest.mark.gpu


def case(H, T, spec, seed, dv=64, dev="cuda"):
    qc, kc = synth.code_streams(H, T, spec, seed=seed, config_id=5)
    q = torch.from_numpy(qc.view(np.int32)).to(dev)
    k = torch.from_numpy(kc.view(np.int32)).to(dev)
    v = torch.randn((H, T, dv), generator=torch.Generator().manual_seed(seed)).to(torch.bfloat16).to(dev)
    return q, k, v


SMALL_POOL = synth.CodeSpec(bits=32, pool=3000, alpha=1.05, fresh=0.05)
BIG_POOL = synth.CodeSpec(bits=32, pool=1 << 18, alpha=1.05, fresh=0.05)


@pytest.mark.parametrize("n_shards,seg_len,spec", [
    (1, 1024, SMALL_POOL), (2, 1024, SMALL_POOL), (4, 512, SMALL_POOL),
    (3, 2048, BIG_POOL), (2, 8192, BIG_POOL),   # 8192-position segments: some overflow K2's table
])
@pytest.mark.parametrize("peer", ["1", "0"])
def test_sharded_equals_one_pass(cuda, monkeypatch, n_shards, seg_len, spec, peer):
    # peer=1: earlier shards' rows read in place by the gather; 0: requested and exchanged
    monkeypatch.setenv("LEMA_SHARD_PEER", peer)
    H = 4
    T = n_shards * seg_len * 12
    q, k, v = case(H, T, spec, seed=n_shards * 10 + seg_len)
    src1, out1 = prefill_match(q, k, v)
    src, out = emulated_sharded_prefill(q, k, v, n_shards, seg_len)
    torch.cuda.synchronize()
    assert torch.equal(src, src1)
    assert torch.equal(out.view(torch.int16), out1.view(torch.int16))
    hits = (src >= 0)
    # the shards did talk: some matches reach back across a shard boundary
    if n_shards > 1:
        L = T // n_shards
        shard_of_query = torch.arange(T, device=cuda)[None, :] // L
        assert bool(((src // L < shard_of_query) & hits).any())


def test_sharded_vs_oracle_small(cuda):
    H, T = 2, 3 * 2048
    q, k, v = case(H, T, SMALL_POOL, seed=7, dv=8)
    src, out = emulated_sharded_prefill(q, k, v, 3, 512)
    qs = q.cpu().numpy().view(np.uint32)
    ks = k.cpu().numpy().view(np.uint32)
    ref = oracle.latest_prev_match(qs, ks)
    assert np.array_equal(src.cpu().numpy(), ref)
    vf = v.float().cpu().numpy()
    assert np.array_equal(out.float().cpu().numpy(), oracle.gather(ref, vf))


@pytest.mark.parametrize("peer", ["1", "0"])
@pytest.mark.parametrize("kind", ["all_equal", "all_distinct", "q_is_k"])
def test_sharded_edge_cases(cuda, monkeypatch, kind, peer):
    monkeypatch.setenv("LEMA_SHARD_PEER", peer)
    H, T, n_sh, seg = 2, 4 * 1024, 4, 256
    rng = np.random.default_rng(3)
    if kind == "all_equal":
        kc = np.full((H, T), 0xFFFFFFFF, dtype=np.uint32)
        qc = kc.copy()
    elif kind == "all_distinct":
        kc = rng.permutation(1 << 24)[: H * T].astype(np.uint32).reshape(H, T)
        qc = (kc + (1 << 25)).astype(np.uint32)
    else:
        kc = rng.integers(0, 50, size=(H, T)).astype(np.uint32)
        qc = kc.copy()
    q = torch.from_numpy(qc.view(np.int32)).to(cuda)
    k = torch.from_numpy(kc.view(np.int32)).to(cuda)
    v = torch.randn((H, T, 16), device=cuda)
    src1, out1 = prefill_match(q, k, v)
    src, out = emulated_sharded_prefill(q, k, v, n_sh, seg)
    assert torch.equal(src, src1) and torch.equal(out, out1)


@pytest.mark.parametrize("rows", [2, 4])
def test_sweep_rows_per_head(cuda, rows):
    # each head swept as independent rows, then merged: the same result
    from latest_exact_match_attention_b200.longctx import CudaOps, ThreadComm, _Board
    q, k, v = case(4, 2 * 8 * 1024, SMALL_POOL, seed=11)
    src1, out1 = prefill_match(q, k, v)
    L = q.shape[1] // 2
    board = _Board(2)
    res = [None, None]
    import threading

    def run(r):
        sl = slice(r * L, (r + 1) * L)
        res[r] = sharded_prefill(q[:, sl], k[:, sl], v[:, sl], ThreadComm(board, r),
                                 CudaOps(q.device, rows_per_head=rows), seg_len=1024)
    th = [threading.Thread(target=run, args=(r,)) for r in range(2)]
    for t in th:
        t.start()
    for t in th:
        t.join()
    assert torch.equal(torch.cat([res[0][0], res[1][0]], 1), src1)
    assert torch.equal(torch.cat([res[0][1], res[1][1]], 1), out1)


def test_single_rank_entry_point(cuda):
    q, k, v = case(3, 4096, SMALL_POOL, seed=1)
    src1, out1 = prefill_match(q, k, v)
    src, out = sharded_prefill(q, k, v, seg_len=1024)
    assert torch.equal(src, src1) and torch.equal(out, out1)
