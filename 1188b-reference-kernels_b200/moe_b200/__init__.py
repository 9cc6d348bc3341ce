"""B200-native MoE expert-layer forward path (sm_100a CUDA behind a C ABI).

Public API (torch tensors on a CUDA device; no CPU fallback):
  topk, router_topk, row_id_map, permute, permute_trans, unpermute,
  unpermute_weighted, grouped_gemm, grouped_wgrad, router_logits, router_gemm_topk,
  permute_backward, combine_backward, swiglu_backward, swiglu,
  MoELayer (forward and backward), moe_layer_fwd, MoEWeights
The reference-style ``kernel_function`` entry points live in ``bundles/``.
"""
from ._lib import MoeError, load as load_library
from .ops import (GroupedGemmPlan, RouterOutput, RowIdMap, combine_backward, grouped_gemm,
                  grouped_wgrad, grouped_wgrad_device_error, permute, permute_device_error,
                  permute_backward, permute_trans, router_device_error, router_gemm_topk,
                  router_logits, router_topk, row_id_map, swiglu, swiglu_backward,
                  topk, unpermute, unpermute_weighted)
from .layer import HostPipeline, MoELayer, MoEWeights, moe_layer_fwd

__all__ = [
    "MoeError", "load_library", "GroupedGemmPlan", "RouterOutput", "RowIdMap", "combine_backward",
    "grouped_gemm",
    "grouped_wgrad", "grouped_wgrad_device_error",
    "permute", "permute_device_error", "permute_backward", "permute_trans", "router_device_error", "router_gemm_topk",
    "router_logits", "router_topk", "row_id_map",
    "swiglu", "swiglu_backward", "topk", "unpermute", "unpermute_weighted",
    "MoELayer", "MoEWeights", "HostPipeline", "moe_layer_fwd",
]
