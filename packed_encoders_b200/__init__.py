"""B200-native (sm_100a) packed variable-length attention for packed_encoders.

Public entry points mirror the reference's attention hooks; see ``ops`` for the mapping.
"""

from packed_encoders_b200.errors import PackedEncodersError, UnsupportedTargetError, ValidationError
from packed_encoders_b200.ops import (
    apply_rope_bshd,
    attention_bshd,
    device_error_word,
    flash_attention,
    flash_attention_varlen,
    packed_attention,
    packed_attention_backward,
    packed_short_attention,
    packed_short_attention_supported,
)

__all__ = [
    "PackedEncodersError", "UnsupportedTargetError", "ValidationError",
    "apply_rope_bshd", "attention_bshd", "device_error_word", "flash_attention", "flash_attention_varlen", "packed_attention",
    "packed_attention_backward",
    "packed_short_attention", "packed_short_attention_supported",
]
