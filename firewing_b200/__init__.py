"""firewing_b200 -- B200 (sm_100a) sparse-MoE block of x3haloed/firewing.

The product is the C-ABI CUDA library ``libfwmoe`` (include/fwmoe.h).  This
package is its Python host side: a ctypes binding that mirrors the reference
crate's block/expert API (linear_bf16, swiglu_bf16, route, the resident top-k
runner).  There is no CPU fallback: every call runs the CUDA kernels, and
importing the binding fails loudly when the library has not been built.
"""
from .moe import (  # noqa: F401
    EP_TRANSPORT_NCCL,
    EP_TRANSPORT_P2P,
    FW_ECUDA,
    FW_EINVAL,
    FW_ENAN,
    FW_ENCCL,
    FW_ENOMEM,
    FW_ETIMEOUT,
    FW_OK,
    PATH_DECODE,
    PATH_PREFILL,
    FwError,
    MoeBlock,
    MoeConfig,
    add_bf16,
    codec_container_check,
    ep_combine_row,
    ep_held_experts,
    ep_owner,
    ep_unique_id,
    forward_noalloc,
    library,
    library_path,
    linear_bf16,
    route_bf16,
    safetensors_tensor_info,
    swiglu_bf16,
    topk_bf16,
)
