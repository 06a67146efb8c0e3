"""Device-side bounded waits give up, report, and leave the next call exact.

Every wait of one warp, CTA or pipeline role on another's progress is bounded (4 s by
default; LEMA_WAIT_NS in the environment shortens it, read at each launch). A wait that runs
out sets LEMA_STATUS_PROBE_LIMIT in the status word and returns -- nothing traps or hangs --
and the product paths raise LemaError when they read the word (latest_prev_match, lema_hard,
Transformer.forward, LemaCache.check, _lib.check_status). These tests shorten the bound so
that waits run out on purpose, then check that the next call with the default bound is bit
for bit the result of a clean call."""
import numpy as np
import pytest
import torch

from latest_exact_match_attention_b200 import _lib, prefill_match, proj_codes, synth
from latest_exact_match_attention_b200._lib import LEMA_STATUS_PROBE_LIMIT, LemaError

pytestmark = pytest.mark.gpu


def _clean(dev):
    torch.cuda.synchronize(dev)
    try:
        _lib.check_status(dev)
    except LemaError:
        pass


def test_k2_row_copy_wait_runs_out(cuda, monkeypatch):
    # one wave of matchers or more: the pipelined launch, whose row-copying CTAs wait for the
    # matchers' progress; a 1 us bound runs out while the matchers work
    qc, kc = synth.code_streams(320, 8192, synth.CONFIG2, seed=11, config_id=2)
    q = torch.from_numpy(qc.view(np.int32)).to(cuda)
    k = torch.from_numpy(kc.view(np.int32)).to(cuda)
    v = torch.randint(-30000, 30000, (320, 8192, 24), dtype=torch.int16, device=cuda)
    _clean(cuda)
    src0, out0 = prefill_match(q, k, v)
    _lib.check_status(cuda)
    monkeypatch.setenv("LEMA_WAIT_NS", "1000")
    st = torch.zeros(1, dtype=torch.int32, device=cuda)
    prefill_match(q, k, v, status=st)
    torch.cuda.synchronize()
    assert int(st.item()) & LEMA_STATUS_PROBE_LIMIT
    # the package's own word: the Python call raises
    prefill_match(q, k, v)
    with pytest.raises(LemaError, match="ran out"):
        _lib.check_status(cuda, "prefill")
    monkeypatch.delenv("LEMA_WAIT_NS")
    src1, out1 = prefill_match(q, k, v)
    _lib.check_status(cuda)
    assert torch.equal(src0, src1) and torch.equal(out0, out1)


def test_k1_pipeline_wait_runs_out(cuda, monkeypatch):
    # a long K loop per tile: the epilogue's wait for the first accumulator (and the other
    # roles' stage waits) outlast a 1 ns bound; the roles abort together, drain what they
    # issued and free the tensor memory
    g = torch.Generator(device=cuda).manual_seed(5)
    x = torch.randn((2, 4096, 8192), generator=g, device=cuda).to(torch.bfloat16)
    w = (0.01 * torch.randn((2 * 16 * 32, 8192), generator=g, device=cuda)).to(torch.bfloat16)
    _clean(cuda)
    q0, k0 = proj_codes(x, w, 16, 16)
    _lib.check_status(cuda)
    monkeypatch.setenv("LEMA_WAIT_NS", "1")
    st = torch.zeros(1, dtype=torch.int32, device=cuda)
    proj_codes(x, w, 16, 16, status=st)
    torch.cuda.synchronize()
    assert int(st.item()) & LEMA_STATUS_PROBE_LIMIT
    monkeypatch.delenv("LEMA_WAIT_NS")
    q1, k1 = proj_codes(x, w, 16, 16)
    _lib.check_status(cuda)
    assert torch.equal(q0, q1) and torch.equal(k0, k1)


def test_model_forward_raises_on_a_wait_that_ran_out(cuda, monkeypatch):
    from latest_exact_match_attention_b200.model import ModelConfig, Transformer
    torch.manual_seed(3)
    m = Transformer(ModelConfig(vocab_size=256, depth=1, dim=256, num_heads=64, d_qk=32,
                                d_v=8)).to(cuda).to(torch.bfloat16).eval()
    idx = torch.randint(0, 200, (8, 2048), device=cuda)   # 512 streams: pipelined K2
    _clean(cuda)
    ref = m(idx)
    monkeypatch.setenv("LEMA_WAIT_NS", "1000")
    with pytest.raises(LemaError, match="Transformer.forward"):
        m(idx)
    monkeypatch.delenv("LEMA_WAIT_NS")
    assert torch.equal(m(idx), ref)
