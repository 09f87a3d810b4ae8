"""The small Co-ALiBi GPT (the caller side of the kernels): the model and its
data-parallel wiring on CPU with the oracle's attention injected, and on the GPU
the model with the sm_100a kernels against the same weights with the oracle's
attention in float32."""
import math
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def oracle_attention(q, k, v, causal=True, bias_max=8.0):
    """Co-ALiBi attention from the oracle, float32, differentiable (test only)."""
    from oracle import coalibi_oracle as orc
    sl = orc.api_slopes(q.shape[1], bias_max, q.dtype).to(q.device)
    o = orc.forward(q.float(), k.float(), v.float(), sl, causal, None, torch.float32)[0]
    return o.to(q.dtype)


def _tiny(**kw):
    from co_alibi_gpt import GPTConfig
    c = dict(n_layer=2, d_model=32, n_head=2, vocab=97, seq_len=24)
    c.update(kw)
    return GPTConfig(**c)


def test_gpt_cpu_forward_backward_with_oracle_attention():
    from co_alibi_gpt import build, make_tokens
    cfg = _tiny()
    model, opt = build(cfg, "cpu", seed=1, dtype=torch.float32, attn_fn=oracle_attention)
    tok = make_tokens(cfg, 3, seed=2)
    logits = model(tok[:, :-1])
    assert logits.shape == (3, cfg.seq_len, cfg.vocab)
    loss = model(tok[:, :-1], targets=tok[:, 1:])
    # N(0, 0.02) weights: near-uniform predictions at initialisation
    assert abs(loss.item() - math.log(cfg.vocab)) < 0.05
    loss.backward()
    assert all(p.grad is not None and torch.isfinite(p.grad).all() for p in model.parameters())
    # causality: changing a later token leaves earlier logits unchanged
    tok2 = tok.clone()
    tok2[:, 20] = (tok2[:, 20] + 1) % cfg.vocab
    with torch.no_grad():
        a, b = model(tok[:, :-1]), model(tok2[:, :-1])
    assert torch.allclose(a[:, :20], b[:, :20], atol=1e-6)
    assert not torch.allclose(a[:, 20:], b[:, 20:])


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _ddp_worker(rank, world, port, out):
    import sys
    for p in (ROOT, os.path.join(ROOT, "co-alibi_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    from co_alibi_gpt import build, make_tokens
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = _tiny()
        model, _ = build(cfg, "cpu", seed=1, dtype=torch.float32, ddp=True, attn_fn=oracle_attention)
        tok = make_tokens(cfg, 4, seed=3)[2 * rank:2 * rank + 2]  # each rank: half of the batch
        model(tok[:, :-1], targets=tok[:, 1:]).backward()
        if rank == 0:
            # numpy copies travel by value (tensors would be shared-memory handles that die with the worker)
            out.put({n: p.grad.detach().numpy().copy() for n, p in model.module.named_parameters()})
    finally:
        dist.destroy_process_group()


def test_gpt_ddp_gloo_averages_gradients():
    """Two gloo ranks with half a batch each: the all-reduced gradients equal the
    single-process gradients of the whole batch."""
    from co_alibi_gpt import build, make_tokens
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ddp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    cfg = _tiny()
    model, _ = build(cfg, "cpu", seed=1, dtype=torch.float32, attn_fn=oracle_attention)
    tok = make_tokens(cfg, 4, seed=3)
    model(tok[:, :-1], targets=tok[:, 1:]).backward()
    for n, p in model.named_parameters():
        assert torch.allclose(torch.from_numpy(got[n]), p.grad, rtol=1e-4, atol=1e-6), n


@pytest.mark.gpu
def test_gpt_kernels_match_fp32_oracle_attention():
    """bf16 model, same weights: the sm_100a attention against the oracle's float32
    attention (rounded to bf16) -- loss and every parameter gradient."""
    from co_alibi_gpt import build, make_tokens
    from tests._common import rel_err
    cfg = _tiny(d_model=128, n_head=2, vocab=512, seq_len=256)
    dev = torch.device("cuda", 0)
    tok = make_tokens(cfg, 2, seed=5, device=dev)
    grads, losses = [], []
    for fn in (None, oracle_attention):
        model, _ = build(cfg, dev, seed=4, attn_fn=fn)
        loss = model(tok[:, :-1], targets=tok[:, 1:])
        loss.backward()
        losses.append(loss.item())
        grads.append(torch.cat([p.grad.float().flatten() for p in model.parameters()]))
    assert abs(losses[0] - losses[1]) < 1e-2
    assert rel_err(grads[0], grads[1]) < 3e-2


@pytest.mark.gpu
def test_gpt_train_steps_reduce_the_loss():
    from co_alibi_gpt import build, make_tokens, train_step
    cfg = _tiny(d_model=128, n_head=2, vocab=512, seq_len=256)
    dev = torch.device("cuda", 0)
    model, opt = build(cfg, dev, seed=4, lr=3e-3)
    tok = make_tokens(cfg, 4, seed=6, device=dev)
    losses = [train_step(model, opt, tok).item() for _ in range(8)]
    assert all(math.isfinite(x) for x in losses)
    assert losses[-1] < losses[0] - 0.5
