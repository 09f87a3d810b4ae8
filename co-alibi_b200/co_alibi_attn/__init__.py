"""Co-ALiBi attention on B200 (sm_100a): drop-in for the reference package
``co_alibi_attn`` (``co_alibi_attn/__init__.py:1-3``)."""
from .co_alibi_attn import co_alibi_attention, CoALIBIAttention, device_status  # noqa: F401

__all__ = ['co_alibi_attention']
