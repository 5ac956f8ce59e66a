"""sm_100a per-token layer operators of the HRM-Text forward pass.

Python front end of libhrm_ops.so (C ABI: include/hrm_ops.h).  Importing this
package loads the library and fails loudly when it has not been built.
"""

from ._lib import HrmError, LIB, LIB_PATH  # noqa: F401
from .ops import (  # noqa: F401
    add_rms_norm,
    additive_inject,
    apply_attn_gate,
    broadcast_vec,
    convert_to_bf16,
    gated_attn_output,
    embed_rms_norm,
    embedding_lookup,
    rms_norm,
    rope_embed,
    rope_embed_token_major,
    rope_table,
    split_gqkv_rope,
    swiglu_ffn,
    wait_timeouts,
)

__all__ = [
    "HrmError",
    "additive_inject",
    "swiglu_ffn",
    "rms_norm",
    "add_rms_norm",
    "rope_table",
    "rope_embed",
    "rope_embed_token_major",
    "embedding_lookup",
    "embed_rms_norm",
    "split_gqkv_rope",
    "apply_attn_gate",
    "gated_attn_output",
    "broadcast_vec",
    "convert_to_bf16",
    "wait_timeouts",
]
