"""Host-buffer entry point: streamed chunks give the same results as the device
API on the whole batch, and argument errors are raised before any device use."""
import math

import pytest
import torch

from tests._common import make_inputs


def test_streaming_rejects_bad_arguments_on_cpu():
    from co_alibi_attn.streaming import co_alibi_attention_from_host
    q, k, v, do = make_inputs(2, 4, 2, 64, 64, 64, torch.float16)
    with pytest.raises(ValueError):
        co_alibi_attention_from_host(q, k[:1], v[:1])          # batch mismatch
    with pytest.raises(ValueError):
        co_alibi_attention_from_host(q, k, v, do[:, :2])       # do shape
    with pytest.raises(ValueError):
        co_alibi_attention_from_host(q, k.float(), v)          # dtype mismatch
    with pytest.raises(ValueError):
        co_alibi_attention_from_host(q, k, v, chunks=0)
    with pytest.raises(ValueError):
        co_alibi_attention_from_host(q, k, v, out=(torch.empty(1),))
    with pytest.raises(ValueError):
        co_alibi_attention_from_host(q, k, v, slopes=torch.ones(3))             # slope table length


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [
    (3, 4, 2, 300, 300, 128, True, torch.float16, 16),   # GQA, one kv head per chunk
    (5, 6, 6, 257, 190, 64, False, torch.bfloat16, 3),   # a whole batch element per chunk
    (2, 8, 8, 200, 200, 128, True, torch.float16, 5),    # uneven head ranges
])
def test_streaming_matches_device_api(shape):
    import co_alibi_attn
    from co_alibi_attn.streaming import co_alibi_attention_from_host
    B, Hq, Hkv, Sq, Skv, D, causal, dt, chunks = shape
    q, k, v, do = make_inputs(B, Hq, Hkv, Sq, Skv, D, dt, seed=21)
    q, k, v, do = (t.pin_memory() for t in (q, k, v, do))
    o_h, dq_h, dk_h, dv_h = co_alibi_attention_from_host(q, k, v, do, causal=causal, chunks=chunks)
    qc, kc, vc = (t.cuda().requires_grad_(True) for t in (q, k, v))
    o = co_alibi_attn.co_alibi_attention(qc, kc, vc, causal=causal)
    o.backward(do.cuda())
    torch.cuda.synchronize()
    for name, a, b in (("o", o_h, o), ("dq", dq_h, qc.grad), ("dk", dk_h, kc.grad), ("dv", dv_h, vc.grad)):
        assert torch.equal(a, b.cpu()), name
    (o_only,) = co_alibi_attention_from_host(q, k, v, causal=causal, chunks=chunks)
    assert torch.equal(o_only, o_h)
    assert co_alibi_attn.device_status(reset=True) == 0
