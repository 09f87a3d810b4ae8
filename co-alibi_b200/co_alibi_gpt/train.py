"""Training step of the Co-ALiBi GPT: data-parallel over one process per GPU.

Each rank holds a full bf16 replica and its own batch of token sequences; the
gradients are averaged with NCCL all-reduce by torch DDP (bucketed, overlapped
with the backward pass), then every rank applies the same AdamW update.
"""
import torch

from .model import CoALiBiGPT, GPTConfig


def make_tokens(cfg: GPTConfig, batch: int, seed: int, device=None):
    """``batch`` sequences of ``seq_len + 1`` token ids uniform over the vocabulary
    (inputs are the first ``seq_len``, targets the last ``seq_len``)."""
    g = torch.Generator().manual_seed(seed)
    t = torch.randint(0, cfg.vocab, (batch, cfg.seq_len + 1), generator=g)
    return t if device is None else t.to(device)


def build(cfg: GPTConfig, device, seed=0, dtype=torch.bfloat16, ddp=False, lr=3e-4, attn_fn=None):
    """Model (weights N(0, 0.02) from ``seed``, cast to ``dtype``), optionally
    wrapped in DistributedDataParallel, and its AdamW optimizer.  ``attn_fn``
    defaults to ``co_alibi_attention``."""
    device = torch.device(device)
    model = CoALiBiGPT(cfg, attn_fn)
    model.reset_parameters(torch.Generator().manual_seed(seed))
    model = model.to(device=device, dtype=dtype)
    if ddp:
        model = torch.nn.parallel.DistributedDataParallel(
            model, device_ids=[device.index] if device.type == "cuda" else None, gradient_as_bucket_view=True)
    opt = torch.optim.AdamW(model.parameters(), lr=lr, betas=(0.9, 0.95), weight_decay=0.1,
                            fused=device.type == "cuda")
    return model, opt


def train_step(model, opt, tokens):
    """One step on ``tokens`` [batch, seq_len + 1]: forward, backward (gradients
    all-reduced across ranks under DDP), AdamW update.  Returns the loss tensor."""
    opt.zero_grad(set_to_none=True)
    loss = model(tokens[:, :-1], targets=tokens[:, 1:])
    loss.backward()
    opt.step()
    return loss.detach()
