"""Pure-PyTorch reference implementations of every hot op.

These are the oracle for the CUDA kernels (tests compare each kernel against the
fp32 evaluation of the function here) and the execution path in CPU mode.  They
restate the semantics of the Trainium plugin's PyTorch fallbacks; each function
cites the fallback it restates.
"""

from .attention import (  # noqa: F401
    paged_attention,
    prefill_attention,
    write_kv_cache,
    gather_kv_from_cache,
    lse_merge,
    cp_count_local,
    cp_global_pos,
    cp_slot_mapping,
)
from .moe import (  # noqa: F401
    clamped_swiglu,
    moe_experts,
    router_topk,
    build_blockwise_mapping,
    permute_routed_tokens,
    topk_reduce,
)
from .mxfp4 import FP4_VALUES, dequant_mxfp4, quantize_mxfp4, quantize_mxfp8, dequant_mxfp8  # noqa: F401
from .norm import rms_norm, fused_add_rms_norm, rmsnorm_quant_fp8  # noqa: F401
from .rope import apply_rope, llama3_inv_freq, mrope_cos_sin, rope_cos_sin, yarn_inv_freq  # noqa: F401
from .sampling import (  # noqa: F401
    sample,
    greedy,
    topk_topp_filter,
    rejection_greedy,
    correct_spec_decode_positions_and_slot_mapping,
    argsort_unstable,
    cumsum,
)
