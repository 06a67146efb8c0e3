"""Generate the golden vectors of tests/golden/ by running the REFERENCE's own code.

Run in the build container, where the reference checkout exists (it does not on the GPU box,
which only reads the committed .npz files):

    CXX=/usr/bin/g++ CC=/usr/bin/gcc python tests/golden/make_golden.py [REFERENCE_ROOT]

Inputs come from this repository's seeded generator (latest_exact_match_attention_b200.synth)
and are stored in the fixtures, so the fixtures do not depend on the generator staying the
same. Outputs come from the reference:
    code/lema/attention.py:82-97    pack_codes
    code/lema/attention.py:100-132  latest_prev_match (CPU torch)
    code/lema/cache.py:129-201      HashStore.exchange (its C++ store, code/lema/csrc/store.cpp)
    code/lema/model.py:257-363      Transformer: a tiny random-init LEMA model's weights, and
                                    its hard-mode logits and store counts (fp32, CPU)
Value rows are regenerated from their seed at test time; each fixture stores a SHA-256 of the
values and of the reference outputs, so a regeneration that drifted is detected.
"""
from __future__ import annotations

import hashlib
import os
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

from latest_exact_match_attention_b200 import synth  # noqa: E402


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def config1_values():
    """Config 1 value rows: [8, 4608, 64] fp32, N(0, 1)."""
    return synth.values_np(8, 4608, 64, seed=0, config_id=1)


def config2_values():
    """Values of the config-2 slice: [4, 16384, 24] bf16 (as uint16 bit patterns)."""
    import torch
    f = synth.values_np(4, 16384, 24, seed=0, config_id=2)
    return torch.from_numpy(f).to(torch.bfloat16).view(torch.uint16).numpy()


def store_case_values(P, T, dv, seed):
    rng = np.random.default_rng([seed, 77])
    return rng.integers(0, 1 << 16, size=(P, T, dv), dtype=np.uint16)


def main(ref_root: str):
    os.environ["CXX"] = "/usr/bin/g++"   # the default CXX wrapper cannot link -fopenmp
    os.environ["CC"] = "/usr/bin/gcc"
    os.environ.setdefault("TORCH_EXTENSIONS_DIR", tempfile.mkdtemp(prefix="lema_ref_ext_"))
    sys.dont_write_bytecode = True
    sys.path.insert(0, str(Path(ref_root) / "code"))
    import torch
    from lema.attention import latest_prev_match, pack_codes
    from lema.cache import HashStore

    def ref_lpm(qc, kc):
        return latest_prev_match(torch.from_numpy(qc.astype(np.int64)),
                                 torch.from_numpy(kc.astype(np.int64))).numpy()

    # ---------------------------------------------------------------- config 1
    # B=1, H=8, 16-bit codes, pool 1024, Zipf 1.2, 10% fresh; prefill 4096 then 512 decode
    # steps through the reference's store; fp32 d_v 64.
    qc, kc = synth.code_streams(8, 4608, synth.CONFIG1, seed=0, config_id=1)
    v = config1_values()
    src = ref_lpm(qc, kc)
    store = HashStore(64, groups=8, dtype=np.float32, capacity=8 * 4608 * 2)
    outs = np.empty_like(v)
    T0 = 4096
    q64, k64 = qc.astype(np.int64), kc.astype(np.int64)
    o = torch.empty(8 * T0, 64)
    store.exchange(torch.from_numpy(np.ascontiguousarray(q64[:, :T0]).reshape(-1)),
                   torch.from_numpy(np.ascontiguousarray(k64[:, :T0]).reshape(-1)),
                   torch.from_numpy(np.ascontiguousarray(v[:, :T0]).reshape(-1, 64)), o, T0, 0)
    outs[:, :T0] = o.numpy().reshape(8, T0, 64)
    counts_prefill = store.counts.numpy().copy()
    for t in range(T0, 4608):
        o = torch.empty(8, 64)
        store.exchange(torch.from_numpy(np.ascontiguousarray(q64[:, t])),
                       torch.from_numpy(np.ascontiguousarray(k64[:, t])),
                       torch.from_numpy(np.ascontiguousarray(v[:, t])), o, 1, 0)
        outs[:, t] = o.numpy()
    # the store and the dense op must agree (the reference's own invariant)
    dense = np.where((src >= 0)[..., None], np.take_along_axis(v, np.maximum(src, 0)[..., None], 1), 0)
    assert np.array_equal(dense, outs), "reference store and dense op disagree"
    np.savez_compressed(HERE / "config1.npz", qc=qc, kc=kc, src=src.astype(np.int32),
                        counts_prefill=counts_prefill, counts_final=store.counts.numpy(),
                        values_sha=sha(v), out_sha=sha(outs), prefill_T=T0)
    print("config1: hits", float((src >= 0).mean()), "entries", int(store.counts.sum()))

    # ------------------------------------------------------ config 2 (4-stream slice)
    qc, kc = synth.code_streams(4, 16384, synth.CONFIG2, seed=0, config_id=2)
    v = config2_values()
    src = ref_lpm(qc, kc)
    dense = np.where((src >= 0)[..., None], np.take_along_axis(v, np.maximum(src, 0)[..., None], 1), 0)
    np.savez_compressed(HERE / "config2_slice.npz", qc=qc, kc=kc, src=src.astype(np.int32),
                        values_sha=sha(v), out_sha=sha(dense))
    print("config2 slice: hits", float((src >= 0).mean()))

    # ---------------------------------------------------------------- edge cases
    rng = np.random.default_rng(123)
    edge = {}

    def add(name, q, k):
        q, k = np.atleast_2d(q), np.atleast_2d(k)
        edge[f"{name}__qc"], edge[f"{name}__kc"] = q, k
        edge[f"{name}__src"] = ref_lpm(q, k).astype(np.int32)

    add("t1", np.array([[5]], np.uint32), np.array([[5]], np.uint32))
    add("t2_self", np.array([[7, 7]], np.uint32), np.array([[7, 9]], np.uint32))
    add("all_equal", np.full((3, 100), 42, np.uint32), np.full((3, 100), 42, np.uint32))
    ext = np.array([0, 0xFFFFFFFF, 1, 0x80000000], np.uint32)
    add("extremes", ext[rng.integers(0, 4, size=(2, 300))], ext[rng.integers(0, 4, size=(2, 300))])
    add("q_is_k", *(lambda a: (a, a.copy()))(rng.integers(0, 8, size=(4, 64)).astype(np.uint32)))
    add("two_codes", rng.integers(0, 2, size=(5, 5000)).astype(np.uint32),
        rng.integers(0, 2, size=(5, 5000)).astype(np.uint32))
    add("all_distinct", rng.permutation(1 << 20)[:20000].astype(np.uint32).reshape(1, 20000),
        rng.permutation(1 << 20)[:20000].astype(np.uint32).reshape(1, 20000))
    # keys all distinct + queries repeating keys: forces > 6144 distinct keys per stream
    kd = rng.permutation(1 << 24)[:12000].astype(np.uint32)
    add("many_distinct_hits", kd[np.maximum(np.arange(12000) - rng.integers(1, 50, 12000), 0)][None],
        kd[None])
    add("odd_T", rng.integers(0, 30, size=(7, 2049)).astype(np.uint32),
        rng.integers(0, 30, size=(7, 2049)).astype(np.uint32))
    c64 = rng.integers(0, 1 << 63, size=16, dtype=np.uint64) | (np.uint64(1) << np.uint64(63))
    add("u64_top_bit", c64[rng.integers(0, 16, size=(3, 3000))], c64[rng.integers(0, 16, size=(3, 3000))])
    np.savez_compressed(HERE / "edge.npz", **edge)
    print("edge cases:", len(edge) // 3)

    # ---------------------------------------------------------------- pack_codes
    z = rng.standard_normal((2, 3, 40, 64)).astype(np.float32)
    z[0, 0, 0, :8] = 0.0
    z[0, 0, 1, :8] = -0.0
    z[0, 0, 2, 3] = np.nan
    z[1, 2, 5, 63] = -1e-30
    codes64 = pack_codes(torch.from_numpy(z)).numpy()
    codes32 = pack_codes(torch.from_numpy(z[..., :32].copy())).numpy()
    codes16 = pack_codes(torch.from_numpy(z[..., :16].copy())).numpy()
    np.savez_compressed(HERE / "pack.npz", z=z, codes64=codes64, codes32=codes32, codes16=codes16)

    # ----------------------------------------------- store cases (code/tests/test_store.py
    # shapes: heavy code sharing across partitions, codes 0 and 1 as ordinary keys)
    cases = {}
    for name, seed, P, T, chunk, n_codes, cap in [("chunked", 0, 200, 2000, 500, 400, 90_000),
                                                  ("decode", 1, 64, 300, 1, 150, 11_000),
                                                  ("oneshot", 2, 400, 1000, 1000, 300, 130_000)]:
        r = np.random.default_rng(seed)
        codes = r.integers(0, n_codes, size=(2, P, T), dtype=np.int64) * 7919 % (n_codes + 2)
        vals = store_case_values(P, T, 8, seed)
        st = HashStore(8, groups=P, dtype=np.uint16, capacity=cap)
        outs = np.empty_like(vals)
        for lo in range(0, T, chunk):
            hi = min(T, lo + chunk)
            q = torch.from_numpy(np.ascontiguousarray(codes[0, :, lo:hi]).reshape(-1))
            k = torch.from_numpy(np.ascontiguousarray(codes[1, :, lo:hi]).reshape(-1))
            vv = torch.from_numpy(np.ascontiguousarray(vals[:, lo:hi]).reshape(-1, 8))
            o = torch.empty_like(vv)
            st.exchange(q, k, vv, o, hi - lo, 0)
            outs[:, lo:hi] = o.numpy().reshape(P, hi - lo, 8)
        cases[f"{name}__codes"] = codes.astype(np.uint16)
        cases[f"{name}__meta"] = np.array([seed, P, T, chunk, cap])
        cases[f"{name}__counts"] = st.counts.numpy()
        cases[f"{name}__out_sha"] = np.array(sha(outs))
        cases[f"{name}__values_sha"] = np.array(sha(vals))
        print(f"store {name}: load {st.load():.2f}")
    np.savez_compressed(HERE / "store.npz", **cases)

    # ---- a tiny LEMA model end to end: code/lema/model.py (Transformer, hard mode, fp32 CPU)
    from lema.model import ModelConfig, Transformer
    cfg = ModelConfig(vocab_size=128, depth=2, dim=64, num_heads=2, d_qk=32, d_v=32,
                      dim_ff=128, attn="lema")
    torch.manual_seed(0)
    model = Transformer(cfg).eval()
    model.set_hard(True)
    r = np.random.default_rng(11)
    idx = torch.from_numpy(r.integers(0, 24, size=(2, 96), dtype=np.int64))  # many repeats
    with torch.no_grad():
        dense = model(idx)
        cache = model.new_cache("ram", max_cache_len=96, batch=2)
        chunked = torch.cat([model(idx[:, s:s + 16], cache=cache) for s in range(0, 96, 16)], 1)
    assert torch.equal(dense, chunked)
    sd = {f"w__{k}": v.numpy() for k, v in model.state_dict().items()}
    np.savez_compressed(HERE / "model_tiny.npz", idx=idx.numpy(), logits=dense.numpy(),
                        counts=cache.counts().numpy(),
                        cfg=np.array([128, 2, 64, 2, 32, 32, 128]), **sd)
    print(f"model_tiny: {len(sd)} tensors, entries {int(cache.counts().sum())}")


if __name__ == "__main__":
    from oracle.build_ref import reference_root
    main(sys.argv[1] if len(sys.argv) > 1 else str(reference_root()))
