"""FlashAttention for NVIDIA B200 (sm_100a) behind the tilelang_fa_v100 API.

Drop-in for the reference package's four exports (tilelang_fa_v100/__init__.py:3-16
of haohervchb/Tilelang-FA-V100); the kernels are hand-written sm_100a CUDA in
libfa_b200.so, reached through a C ABI (include/fa_b200.h).
"""

from .interface import (
    tilelang_flash_attn_func,
    tilelang_flash_attn_gpu,
    tilelang_paged_forward,
    tilelang_decode_forward,
)
# FA2's packed variable-length entry; an addition beyond the reference's four exports,
# so it is importable by name but left out of __all__ (which mirrors the reference's).
from .interface import tilelang_flash_attn_varlen_func

__version__ = "1.0.0"
__all__ = [
    "tilelang_flash_attn_func",
    "tilelang_flash_attn_gpu",
    "tilelang_paged_forward",
    "tilelang_decode_forward",
]
