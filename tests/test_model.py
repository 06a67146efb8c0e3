"""Host-side checks of the model mirror (no GPU): configuration rules and the parameter
names and shapes of code/lema/model.py, against the state dict the reference's own
Transformer wrote into tests/golden/model_tiny.npz."""
from pathlib import Path

import numpy as np
import pytest
import torch

from latest_exact_match_attention_b200.model import ModelConfig, Transformer

GOLDEN = Path(__file__).resolve().parent / "golden" / "model_tiny.npz"


def tiny_cfg():
    g = np.load(GOLDEN)
    vocab, depth, dim, H, dqk, dv, ff = (int(x) for x in g["cfg"])
    return ModelConfig(vocab_size=vocab, depth=depth, dim=dim, num_heads=H, d_qk=dqk, d_v=dv,
                       dim_ff=ff)


def test_state_dict_names_and_shapes_match_reference():
    g = np.load(GOLDEN)
    ref = {k[3:]: g[k].shape for k in g.files if k.startswith("w__")}
    ours = {k: tuple(v.shape) for k, v in Transformer(tiny_cfg()).state_dict().items()}
    assert ours == ref


def test_config_defaults_and_padding():
    c = ModelConfig(vocab_size=50257, depth=24, dim=1536, num_heads=64, d_qk=32, d_v=24)
    assert c.vocab_size == 50304 and c.dim_ff == 4096
    c2 = ModelConfig(vocab_size=100, depth=1, dim=256, num_heads=8)
    assert (c2.d_qk, c2.d_v, c2.num_kv_heads) == (32, 32, 8)


@pytest.mark.parametrize("kw", [dict(attn="softmax"), dict(pos="rope"), dict(d_qk=65),
                                dict(num_kv_heads=4)])
def test_config_rejects_what_is_not_served(kw):
    base = dict(vocab_size=128, depth=1, dim=256, num_heads=8)
    with pytest.raises(ValueError):
        ModelConfig(**{**base, **kw})


def test_init_scales_like_reference():
    torch.manual_seed(0)
    m = Transformer(ModelConfig(vocab_size=1024, depth=4, dim=512, num_heads=8))
    b = m.blocks[0]
    assert abs(float(b.attn.q_proj.weight.std()) - 512 ** -0.5) < 2e-3
    assert abs(float(b.attn.o_proj.weight.std()) - 512 ** -0.5 / 8 ** 0.5) < 2e-3
    assert abs(float(m.tok_emb.weight.std()) - 512 ** -0.5) < 2e-3
