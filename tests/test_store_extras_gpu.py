"""Store introspection (HashStore.dump / LemaCache.dump) and the worst-case codes hook."""
import numpy as np
import pytest
import torch

from latest_exact_match_attention_b200.cache import HashStore, worst_case_codes
from latest_exact_match_attention_b200.decode import decoder
from latest_exact_match_attention_b200.model import ModelConfig, Transformer

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("segments", [1, 3])
def test_dump_is_the_latest_write_per_key(cuda, segments):
    rng = np.random.default_rng(2)
    P, T, steps = 12, 30, 3
    st = HashStore(8, groups=P, dtype=torch.float16, capacity=4000, device=cuda, segments=segments)
    latest = {}
    for s in range(steps):
        kc = rng.integers(0, 25, size=(P, T)).astype(np.int64)
        v = rng.standard_normal((P, T, 8)).astype(np.float16)
        for p in range(P):
            for t in range(T):
                latest[(p, int(kc[p, t]))] = v[p, t]
        vd = torch.from_numpy(v.reshape(-1, 8)).to(cuda)
        k = torch.from_numpy(kc.reshape(-1)).to(cuda)
        st.exchange(k, k, vd, torch.empty_like(vd), T, 0)
    g, c, rows = st.dump()
    assert g.numel() == len(latest) == int(st.counts.sum())
    got = {(int(a), int(b)): r for a, b, r in zip(g.tolist(), c.tolist(), rows.cpu().numpy())}
    assert got.keys() == latest.keys()
    for key, val in latest.items():
        assert np.array_equal(got[key], val)


def test_worst_case_codes_claim_a_slot_per_token(cuda):
    torch.manual_seed(0)
    cfg = ModelConfig(vocab_size=128, depth=2, dim=256, num_heads=4, d_qk=32, d_v=32)
    m = Transformer(cfg).to(cuda).to(torch.bfloat16).eval()
    B, T0, steps = 2, 20, 5
    c = m.new_cache("hbm", max_cache_len=64, batch=B, codes_hook=worst_case_codes(cfg.depth))
    m(torch.randint(0, 128, (B, T0), device=cuda), cache=c, return_logits=False)
    assert c.entries() == cfg.depth * B * cfg.num_heads * T0
    d = decoder(m, c, tok=torch.zeros(B, 1, dtype=torch.long, device=cuda))
    for _ in range(steps):
        d.step()
    c.check()
    assert c.entries() == cfg.depth * B * cfg.num_heads * (T0 + steps)
    lay, b, h, codes, rows = c.dump(layer=1)
    assert lay.numel() == B * cfg.num_heads * (T0 + steps) and bool((lay == 1).all())
