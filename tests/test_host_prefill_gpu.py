"""prefill_match on host buffers (attention.HostPrefill / prefill_match_host): batches of
streams pipelined through the device must give exactly the device call's results, including a
last batch that is not full."""
import numpy as np
import pytest
import torch

from latest_exact_match_attention_b200 import synth
from latest_exact_match_attention_b200.attention import HostPrefill, prefill_match, prefill_match_host

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("batch,slots", [(16, 2), (16, 3), (8, 4), (64, 3)])
def test_host_pipeline_equals_device_call(cuda, batch, slots):
    N, T = 70, 4096
    qc, kc = synth.code_streams(N, T, synth.CONFIG2, seed=4, config_id=2)
    q = torch.from_numpy(qc.view(np.int32)).pin_memory()
    k = torch.from_numpy(kc.view(np.int32)).pin_memory()
    v = synth.values_torch(N, T, 24, torch.bfloat16, "cpu", seed=4, config_id=2).pin_memory()
    src_d, out_d = prefill_match(q.to(cuda), k.to(cuda), v.to(cuda))
    hp = HostPrefill(cuda, T, torch.int32, (24,), torch.bfloat16, batch=batch, slots=slots)
    src = torch.empty((N, T), dtype=torch.int32).pin_memory()
    out = torch.empty_like(v).pin_memory()
    for _ in range(2):                      # the buffers are reused across calls
        src.fill_(-7)
        hp(q, k, v, src, out)
        torch.cuda.synchronize()
        assert torch.equal(src, src_d.cpu())
        assert torch.equal(out.view(torch.int16), out_d.cpu().view(torch.int16))
    s2, o2 = prefill_match_host(q, k, v, batch=batch)
    torch.cuda.synchronize()
    assert torch.equal(s2, src_d.cpu()) and torch.equal(o2.view(torch.int16), out_d.cpu().view(torch.int16))
