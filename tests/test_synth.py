"""The seeded generator: determinism and the distribution's structural promises."""
import numpy as np

from latest_exact_match_attention_b200 import synth


def test_deterministic():
    a = synth.code_streams(3, 500, synth.CONFIG2, seed=4, config_id=2)
    b = synth.code_streams(3, 500, synth.CONFIG2, seed=4, config_id=2)
    c = synth.code_streams(3, 500, synth.CONFIG2, seed=5, config_id=2)
    assert all(np.array_equal(x, y) for x, y in zip(a, b))
    assert not np.array_equal(a[0], c[0])


def test_fresh_codes_structure():
    spec = synth.CodeSpec(bits=16, pool=64, alpha=1.2, fresh=0.2)
    qc, kc = synth.code_streams(4, 3000, spec, seed=1, config_id=9)
    assert qc.dtype == np.uint16
    for n in range(4):
        keys = set(kc[n].tolist())
        # queries outside every key code exist (fresh) and are guaranteed misses
        q_only = [q for q in qc[n].tolist() if q not in keys]
        assert len(q_only) > 0.1 * 3000
        # pool codes (repeated) + distinct fresh codes: popular codes dominate
        vals, cnt = np.unique(kc[n], return_counts=True)
        assert cnt.max() > 100
        fresh_k = vals[cnt == 1]
        assert len(fresh_k) > 0.1 * 3000


def test_query_fresh_never_matches():
    import oracle
    spec = synth.CodeSpec(bits=32, pool=128, alpha=1.1, fresh=0.3)
    qc, kc = synth.code_streams(2, 4000, spec, seed=2, config_id=3)
    src = oracle.latest_prev_match(qc, kc)
    for n in range(2):
        keys = set(kc[n].tolist())
        fresh_q = np.array([q not in keys for q in qc[n].tolist()])
        assert (src[n][fresh_q] == -1).all()


def test_zipf_cdf():
    c = synth.zipf_cdf(1000, 1.1)
    assert c[-1] == 1.0 and np.all(np.diff(c) > 0)
