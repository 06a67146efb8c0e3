"""Loading the golden vectors of tests/golden/ (made by tests/golden/make_golden.py from the
reference's own code) and regenerating their value rows from the seeds."""
from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def load(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


def edge_cases() -> dict:
    d = load("edge")
    names = sorted({k.split("__")[0] for k in d})
    return {n: (d[f"{n}__qc"], d[f"{n}__kc"], d[f"{n}__src"]) for n in names}


def store_cases() -> dict:
    d = load("store")
    names = sorted({k.split("__")[0] for k in d})
    out = {}
    for n in names:
        seed, P, T, chunk, cap = (int(x) for x in d[f"{n}__meta"])
        out[n] = dict(codes=d[f"{n}__codes"].astype(np.int64), seed=seed, P=P, T=T, chunk=chunk,
                      cap=cap, counts=d[f"{n}__counts"], out_sha=str(d[f"{n}__out_sha"]),
                      values_sha=str(d[f"{n}__values_sha"]))
    return out


def config1_values() -> np.ndarray:
    from latest_exact_match_attention_b200 import synth
    return synth.values_np(8, 4608, 64, seed=0, config_id=1)


def config2_values_u16() -> np.ndarray:
    import torch
    from latest_exact_match_attention_b200 import synth
    f = synth.values_np(4, 16384, 24, seed=0, config_id=2)
    return torch.from_numpy(f).to(torch.bfloat16).view(torch.uint16).numpy()


def store_case_values(P, T, dv, seed) -> np.ndarray:
    rng = np.random.default_rng([seed, 77])
    return rng.integers(0, 1 << 16, size=(P, T, dv), dtype=np.uint16)


def dense_gather(src: np.ndarray, v: np.ndarray) -> np.ndarray:
    return np.where((src >= 0)[..., None], np.take_along_axis(v, np.maximum(src, 0)[..., None], 1),
                    np.zeros((), v.dtype))
