"""Small GPT with Co-ALiBi self-attention (the sm_100a kernels of ``co_alibi_attn``)
and its data-parallel training step."""
from .model import GPTConfig, CoALiBiGPT  # noqa: F401
from .train import build, make_tokens, train_step  # noqa: F401

__all__ = ["GPTConfig", "CoALiBiGPT", "build", "make_tokens", "train_step"]
