"""A small GPT whose self-attention is Co-ALiBi: the caller side of the kernels.

The reference repository ships the attention operator only (no model code), so
this module is new.  Every block runs ``co_alibi_attention`` (the sm_100a
kernels behind the reference's Python API) with causal masking; positions come
from the Co-ALiBi bias alone, so there is no position embedding.  Layer layout:
token embedding -> n_layer x [LayerNorm -> QKV -> Co-ALiBi attention -> output
projection -> residual, LayerNorm -> MLP (4x, GELU) -> residual] -> LayerNorm ->
LM head tied to the embedding -> cross-entropy.
"""
import math
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass
class GPTConfig:
    n_layer: int = 12
    d_model: int = 768
    n_head: int = 12
    vocab: int = 50304
    seq_len: int = 1024
    mlp_ratio: int = 4
    bias_max: float = 8.0
    init_std: float = 0.02


class CoALiBiSelfAttention(nn.Module):
    """QKV projection, Co-ALiBi causal attention over [B, H, S, D] heads, output projection."""

    def __init__(self, cfg: GPTConfig, attn_fn):
        super().__init__()
        assert cfg.d_model % cfg.n_head == 0
        self.n_head = cfg.n_head
        self.head_dim = cfg.d_model // cfg.n_head
        self.qkv = nn.Linear(cfg.d_model, 3 * cfg.d_model)
        self.proj = nn.Linear(cfg.d_model, cfg.d_model)
        self.attn_fn = attn_fn
        self.bias_max = cfg.bias_max

    def forward(self, x):
        B, S, C = x.shape
        qkv = self.qkv(x).view(B, S, 3, self.n_head, self.head_dim)
        # [B, S, 3, H, D] -> three [B, H, S, D] tensors (contiguous: the kernels take row-major heads)
        q, k, v = (t.transpose(1, 2).contiguous() for t in qkv.unbind(dim=2))
        y = self.attn_fn(q, k, v, causal=True, bias_max=self.bias_max)
        return self.proj(y.transpose(1, 2).reshape(B, S, C))


class Block(nn.Module):
    def __init__(self, cfg: GPTConfig, attn_fn):
        super().__init__()
        self.ln1 = nn.LayerNorm(cfg.d_model)
        self.attn = CoALiBiSelfAttention(cfg, attn_fn)
        self.ln2 = nn.LayerNorm(cfg.d_model)
        self.fc = nn.Linear(cfg.d_model, cfg.mlp_ratio * cfg.d_model)
        self.out = nn.Linear(cfg.mlp_ratio * cfg.d_model, cfg.d_model)

    def forward(self, x):
        x = x + self.attn(self.ln1(x))
        return x + self.out(F.gelu(self.fc(self.ln2(x)), approximate="tanh"))


class CoALiBiGPT(nn.Module):
    """``forward(tokens, targets=None)`` -> logits, or the mean cross-entropy when
    targets are given.  ``attn_fn(q, k, v, causal, bias_max)`` defaults to the
    package's ``co_alibi_attention`` (CUDA only; no other attention is used)."""

    def __init__(self, cfg: GPTConfig, attn_fn=None):
        super().__init__()
        if attn_fn is None:
            from co_alibi_attn import co_alibi_attention
            attn_fn = co_alibi_attention
        self.cfg = cfg
        self.emb = nn.Embedding(cfg.vocab, cfg.d_model)
        self.blocks = nn.ModuleList(Block(cfg, attn_fn) for _ in range(cfg.n_layer))
        self.ln_f = nn.LayerNorm(cfg.d_model)
        self.reset_parameters()

    def reset_parameters(self, generator=None):
        """Weights ~ N(0, init_std) (residual output projections scaled by
        1/sqrt(2 n_layer)), biases 0, LayerNorm affine 1 / 0."""
        std = self.cfg.init_std
        with torch.no_grad():
            for name, p in self.named_parameters():
                if name.endswith("bias"):
                    p.zero_()
                elif ".ln" in name or name.startswith("ln_f"):
                    p.fill_(1.0)
                else:
                    s = std / math.sqrt(2 * self.cfg.n_layer) if name.endswith(("proj.weight", "out.weight")) else std
                    p.copy_(torch.randn(p.shape, generator=generator) * s)

    def forward(self, tokens, targets=None):
        x = self.emb(tokens)
        for blk in self.blocks:
            x = blk(x)
        logits = F.linear(self.ln_f(x), self.emb.weight)
        if targets is None:
            return logits
        return F.cross_entropy(logits.float().view(-1, logits.shape[-1]), targets.reshape(-1))

    def flops_per_token(self):
        """Training FLOPs per token: 6 x (matmul parameters) for the dense layers and
        the tied LM head, plus the causal attention GEMMs (QK^T and PV forward, five
        GEMMs backward, on the visible half of the score matrix)."""
        c = self.cfg
        dense = c.n_layer * (4 * c.d_model * c.d_model + 2 * c.mlp_ratio * c.d_model * c.d_model)
        head = c.vocab * c.d_model
        attn = c.n_layer * 14 * c.d_model * (c.seq_len + 1) / 2
        return 6 * (dense + head) + attn
