"""llattn_b200 — B200 (sm_100a) kernels of the fused local + latent attention
block of Fenix46/local-latent-attention, behind the reference's module API.

    from llattn_b200 import LocalLatentAttentionB200, build_attention
    from llattn_b200.ops import llattn_attention, pool_chunks, pool_query_blocks

The CUDA work happens in libllattn.so (C ABI: include/llattn.h), loaded on
first use; it is built by ``csrc/build.py``.
"""

from . import ops
from .module import DecodeCache, LocalLatentAttentionB200, build_attention
from .ops import LLAttnFunction, llattn_attention

__all__ = ["LocalLatentAttentionB200", "DecodeCache", "build_attention", "llattn_attention", "LLAttnFunction", "ops"]
