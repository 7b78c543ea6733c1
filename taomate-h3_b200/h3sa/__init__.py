"""h3sa: B200-native streaming audio-video attention for TaoMate-H3.

The compute path is libh3sa.so (hand-written sm_100a kernels behind a C ABI); this
package mirrors the reference's Python interfaces on top of it.
"""

from . import _lib
from .kernels import (
    AttentionProblem,
    attention_fwd,
    kv_copy_rows,
    quantize_fp8_e4m3_per_head,
    quantize_fp8_pool,
)

__all__ = [
    "AttentionProblem",
    "attention_fwd",
    "kv_copy_rows",
    "quantize_fp8_e4m3_per_head",
    "quantize_fp8_pool",
]
