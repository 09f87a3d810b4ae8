"""(batch x head) sharding of Co-ALiBi attention across the GPUs of one node.

Every (b, kv head) unit -- with its Hq/Hkv query heads -- is independent in the
forward and the backward, so ranks share no data: each rank runs the operator on
its own contiguous block of units and nothing is exchanged on the data path.
"""
from dataclasses import dataclass

import torch

from .co_alibi_attn import CoALIBIAttention, _api_slopes


@dataclass(frozen=True)
class Shard:
    b0: int
    b1: int
    g0: int  # kv heads [g0, g1); query heads [g0*G, g1*G)
    g1: int
    group: int

    @property
    def h0(self):
        return self.g0 * self.group

    @property
    def h1(self):
        return self.g1 * self.group

    def units(self):
        return [(b, g) for b in range(self.b0, self.b1) for g in range(self.g0, self.g1)]


def shard_plan(B: int, Hq: int, Hkv: int, world: int, rank: int) -> Shard:
    """Contiguous, equal block of (b, kv head) units for `rank`: whole batch rows
    when world divides B, otherwise whole kv-head ranges of every batch row."""
    if Hq % Hkv:
        raise ValueError("Hq must be a multiple of Hkv")
    G = Hq // Hkv
    if not 0 <= rank < world:
        raise ValueError("rank out of range")
    if B % world == 0:
        n = B // world
        return Shard(rank * n, (rank + 1) * n, 0, Hkv, G)
    if Hkv % world == 0:
        n = Hkv // world
        return Shard(0, B, rank * n, (rank + 1) * n, G)
    raise ValueError(f"cannot split B={B} x Hkv={Hkv} units evenly over {world} ranks")


def shard_slopes(Hq: int, shard: Shard, bias_max: float, dtype, device) -> torch.Tensor:
    """The API's slope tensor (2 * table, cast to dtype) restricted to the shard's query
    heads: a view into the device table the API caches per (Hq, bias_max, dtype, device),
    so a call copies nothing from the host (a pageable host-to-device copy would wait
    for the stream to drain and stall every step's launches behind the previous step)."""
    return _api_slopes(Hq, bias_max, dtype, device)[shard.h0:shard.h1]


def sharded_attention(q, k, v, shard: Shard, Hq: int, causal=True, sm_scale=None, bias_max=8.0):
    """co_alibi_attention on the local block q[b0:b1, h0:h1], k/v[b0:b1, g0:g1] (which
    the caller already holds) with the slopes of the global head indices."""
    if sm_scale is None:
        sm_scale = 1.0 / (q.shape[-1] ** 0.5)
    slopes = shard_slopes(Hq, shard, bias_max, q.dtype, q.device)
    return CoALIBIAttention.apply(q.contiguous(), k.contiguous(), v.contiguous(), slopes, causal, sm_scale)
