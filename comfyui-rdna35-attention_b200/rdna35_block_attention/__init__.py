"""B200 (sm_100a) attention hot path behind the ComfyUI-RDNA35-Attention
override API: fixed 64-token block-diagonal attention, exact full attention,
PISA HYD / generic block-sparse attention and the MiniMax-H3 path.  The
compute runs in the in-tree C-ABI library loaded by ``b200_pisa``."""
from .device import b200_device_index, detect_runtime, explain_dispatch, has_native
from .dispatch import fixed_block_attention
from .full_attention import full_attention_b200, full_attention_triton
from .pisa_attention import pisa_attention
from .reference import fixed_block_attention_bthd, fixed_block_attention_ref

__all__ = [
    "b200_device_index",
    "detect_runtime",
    "explain_dispatch",
    "fixed_block_attention",
    "fixed_block_attention_bthd",
    "fixed_block_attention_ref",
    "full_attention_b200",
    "full_attention_triton",
    "has_native",
    "pisa_attention",
]
