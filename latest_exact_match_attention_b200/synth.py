"""Seeded synthetic inputs with the shapes and distributions of the benchmark configurations.

The reference ships no generator for these distributions (its benchmarks use worst-case
uniform codes, code/experiments/main_inference/common.py:170-196); this one is built to the
benchmark description:

  * each stream (one (batch, head) pair) has a POOL of `pool` distinct random codes of `bits`
    bits; its order is the stream's rank -> code map, shared by queries and keys, so a code
    popular among keys is popular among queries too;
  * queries and keys independently draw ranks from a finite Zipf law, p(r) ~ r^-alpha over
    ranks 1..pool;
  * a fraction `fresh` of positions (independently for queries and keys) instead gets a FRESH
    code: drawn without replacement from outside the pool, all fresh codes of a stream
    distinct, so a query-fresh code matches no key at all (a guaranteed miss) and a
    key-fresh code is a key no query asks for.

Everything is drawn from numpy.random.default_rng([seed, config_id]).

The presets name the benchmark configurations (Cfg 1..5).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class CodeSpec:
    bits: int = 32
    pool: int = 8192
    alpha: float = 1.1
    fresh: float = 0.1


CONFIG1 = CodeSpec(bits=16, pool=1024, alpha=1.2, fresh=0.1)   # B=1, H=8, d_v 64 fp32, 4096+512
CONFIG2 = CodeSpec(bits=32, pool=8192, alpha=1.1, fresh=0.1)   # B=8, H=64, T=16384, d_v 24 bf16
CONFIG5 = CodeSpec(bits=32, pool=1 << 20, alpha=1.05, fresh=0.05)  # T=2^26, H=16, d_v 64 bf16


def zipf_cdf(pool: int, alpha: float) -> np.ndarray:
    w = np.arange(1, pool + 1, dtype=np.float64) ** -alpha
    c = np.cumsum(w)
    return c / c[-1]


def _code_dtype(bits: int):
    return np.uint16 if bits <= 16 else (np.uint32 if bits <= 32 else np.uint64)


def distinct_codes(rng: np.random.Generator, bits: int, k: int,
                   exclude: np.ndarray | None = None) -> np.ndarray:
    """k distinct uniformly random `bits`-bit codes, none in `exclude`, in random order."""
    space = 1 << bits
    if exclude is not None and exclude.size:
        excl = np.unique(exclude.astype(np.uint64))
    else:
        excl = np.empty(0, dtype=np.uint64)
    if k + excl.size > space:
        raise ValueError(f"cannot draw {k} distinct {bits}-bit codes outside {excl.size}")
    out = np.empty(0, dtype=np.uint64)
    while out.size < k:
        need = k - out.size
        cand = rng.integers(0, space, size=int(need * 1.25) + 64, dtype=np.uint64)
        cand = cand[~np.isin(cand, excl, assume_unique=False)]
        cand = cand[~np.isin(cand, out)]
        _, first = np.unique(cand, return_index=True)
        cand = cand[np.sort(first)]               # distinct, in draw order
        out = np.concatenate([out, cand[:need]])
    return out.astype(_code_dtype(bits))


def code_streams(n_streams: int, T: int, spec: CodeSpec = CONFIG2, seed: int = 0,
                 config_id: int = 2) -> tuple[np.ndarray, np.ndarray]:
    """Query and key codes, each [n_streams, T] of the spec's width (uint16/32/64)."""
    rng = np.random.default_rng([seed, config_id])
    cdf = zipf_cdf(spec.pool, spec.alpha)
    dt = _code_dtype(spec.bits)
    qc = np.empty((n_streams, T), dtype=dt)
    kc = np.empty((n_streams, T), dtype=dt)
    for n in range(n_streams):
        pool = distinct_codes(rng, spec.bits, spec.pool)
        rq = np.minimum(np.searchsorted(cdf, rng.random(T), side="right"), spec.pool - 1)
        rk = np.minimum(np.searchsorted(cdf, rng.random(T), side="right"), spec.pool - 1)
        q, k = pool[rq], pool[rk]
        fq = rng.random(T) < spec.fresh
        fk = rng.random(T) < spec.fresh
        nq, nk = int(fq.sum()), int(fk.sum())
        if nq + nk:
            fresh = distinct_codes(rng, spec.bits, nq + nk, exclude=pool)
            k[fk] = fresh[:nk]
            q[fq] = fresh[nk:]
        qc[n], kc[n] = q, k
    return qc, kc


def values_np(n_streams: int, T: int, d_v: int, seed: int = 0, config_id: int = 2) -> np.ndarray:
    """N(0, 1) float32 values [n_streams, T, d_v] from a numpy stream (portable; for fixtures
    and CPU-side checks). Cast to bf16/fp16 with torch, which rounds to nearest even."""
    rng = np.random.default_rng([seed, config_id, 1])
    return rng.standard_normal((n_streams, T, d_v), dtype=np.float32)


def values_torch(n_streams: int, T: int, d_v: int, dtype, device, seed: int = 0,
                 config_id: int = 2):
    """N(0, 1) values drawn directly on `device` (large benchmark inputs)."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(int(seed) * 1000003 + int(config_id))
    return torch.randn((n_streams, T, d_v), generator=g, device=device, dtype=torch.float32).to(dtype)


def token_stream(batch: int, T: int, vocab: int, seed: int = 0, config_id: int = 3,
                 alpha: float = 1.1, copy: float = 0.2) -> np.ndarray:
    """Token ids [batch, T] (int64) for the model configurations: Zipf(alpha) unigrams over
    the vocabulary (rank -> token through a random permutation), where a fraction `copy` of
    the positions start a copy of a bigram from earlier in the same sequence (the two tokens
    at a uniformly drawn earlier position j, j + 1 are written at t, t + 1). Seeded with
    numpy's default_rng([seed, config_id])."""
    rng = np.random.default_rng([seed, config_id])
    perm = rng.permutation(vocab)
    cdf = zipf_cdf(vocab, alpha)
    out = perm[np.minimum(np.searchsorted(cdf, rng.random((batch, T))), vocab - 1)]
    start = rng.random((batch, T)) < copy
    pick = rng.random((batch, T))
    rows = np.arange(batch)
    busy = np.zeros(batch, dtype=bool)     # position t is the second token of a copy
    for t in range(2, T - 1):
        go = start[:, t] & ~busy
        if go.any():
            j = np.minimum((pick[:, t] * (t - 1)).astype(np.int64), t - 2)  # j + 1 < t
            r = rows[go]
            out[r, t] = out[r, j[go]]
            out[r, t + 1] = out[r, j[go] + 1]
        busy = go
    return out.astype(np.int64)


def _mix32_torch(x):
    """MurmurHash3's 32-bit finalizer on an int64 tensor of values < 2^32 (a bijection of the
    32-bit integers), computed in int64 with explicit wrap-around."""
    m = (1 << 32) - 1
    x = x & m
    x = x ^ (x >> 16)
    x = (x * 0x85EBCA6B) & m
    x = x ^ (x >> 13)
    x = (x * 0xC2B2AE35) & m
    return x ^ (x >> 16)


def long_code_shard(H: int, start: int, length: int, spec: CodeSpec = CONFIG5, seed: int = 0,
                    device="cuda", chunk: int = 1 << 20, d_v: int = 64, heads=None,
                    values: bool = True):
    """Positions [start, start + length) of config 5's single long sequence, generated on the
    device: (qcodes [H, length] int32, kcodes [H, length] int32, values [H, length, d_v] bf16).

    Built in fixed chunks of `chunk` positions, each from its own seeded torch generator, so a
    shard is the same slice of the same sequence whatever the number of shards. Codes are the
    image of a 32-bit bijection (MurmurHash3's finalizer) of disjoint input ranges: per head a
    pool of `spec.pool` codes (inputs h * 2^20 + rank, below 2^30), key-fresh codes (inputs in
    [2^31, 3 * 2^30)) and query-fresh codes (inputs in [3 * 2^30, 2^32)) -- so query-fresh codes
    match no key. Ranks
    are drawn Zipf(spec.alpha) over the pool; a fraction spec.fresh of queries and of keys is
    fresh. start and length must be multiples of `chunk`. `heads` (a list of head indices
    below H) generates only those heads, the same codes as in the full draw; values=False
    skips the value rows (returns None for them)."""
    import torch
    if start % chunk or length % chunk:
        raise ValueError("start and length must be whole chunks")
    if spec.pool > 1 << 20 or H > 1 << 10:
        raise ValueError("pool <= 2^20 codes per head and H <= 1024")
    dev = torch.device(device)
    cdf = torch.from_numpy(zipf_cdf(spec.pool, spec.alpha)).to(dev)
    heads = list(range(H)) if heads is None else list(heads)
    qc = torch.empty((len(heads), length), dtype=torch.int32, device=dev)
    kc = torch.empty((len(heads), length), dtype=torch.int32, device=dev)
    v = torch.empty((len(heads), length, d_v), dtype=torch.bfloat16, device=dev) if values else None
    g = torch.Generator(device=dev)
    for row, h in enumerate(heads):
        for c0 in range(0, length, chunk):
            c = (start + c0) // chunk
            g.manual_seed(((seed * 1009 + h) * 1_000_003 + c) & ((1 << 62) - 1))
            for which, out in ((0, kc), (1, qc)):
                u = torch.rand(chunk, generator=g, device=dev, dtype=torch.float64)
                rank = torch.searchsorted(cdf, u, right=True).clamp_(max=spec.pool - 1)
                x = h * (1 << 20) + rank
                fresh = torch.rand(chunk, generator=g, device=dev) < spec.fresh
                fx = torch.randint(0, 1 << 30, (chunk,), generator=g, device=dev) + ((2 + which) << 30)
                x = torch.where(fresh, fx, x)
                code = _mix32_torch(x)
                out[row, c0:c0 + chunk] = (code - ((code >> 31) << 32)).to(torch.int32)
            if values:
                v[row, c0:c0 + chunk] = torch.randn((chunk, d_v), generator=g, device=dev).to(torch.bfloat16)
    return qc, kc, v
