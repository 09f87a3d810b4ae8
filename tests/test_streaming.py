"""Host-buffer entry point: streamed chunks give the same results as the device
API on the whole batch, and argument errors are raised before any device use."""
import math

import pytest
import torch

from tests._common import make_inputs


@pytest.mark.parametrize("B,Hkv,chunks", [(8, 16, 16), (1, 1, 16), (2, 8, 16), (4, 8, 1), (3, 5, 7),
                                          (8, 16, 32), (1, 12, 4), (1, 32, 16), (2, 2, 16)])
def test_chunk_plan_covers_every_unit_in_order(B, Hkv, chunks):
    from co_alibi_attn.streaming import chunk_plan
    units = chunk_plan(B, Hkv, chunks)
    assert all(0 <= g0 < g1 <= Hkv for _, g0, g1 in units)
    assert [(b, g) for b, g0, g1 in units for g in range(g0, g1)] == [(b, g) for b in range(B) for g in range(Hkv)]
    m = max(1, min(Hkv, -(-(B * Hkv) // chunks)))
    assert max(g1 - g0 for _, g0, g1 in units) <= 2 * m
    if chunks >= 4 and m > 1:
        # small pieces first and last: the pipeline's fill and drain
        assert units[0][2] - units[0][1] == 1 and units[-1][2] - units[-1][1] == 1


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
