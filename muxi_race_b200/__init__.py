"""muxi_race_b200 — a B200-native (sm_100a) fused Mixture-of-Experts operator.

Entry points:
  run_kernel(...)      drop-in for the contest operator's ``run_kernel`` (10 tensors, padded layout)
  fused_moe(...)       token-major fused MoE (routing alignment + both GEMM stages + top-k combine)
  fused_moe_int8(...)  W8A8 variant; weights from quantize_rows_int8()
  fused_moe_fp8(...)   fp8 (e4m3) variant; weights from quantize_rows_fp8()
  moe_align(...)       device-side routing metadata
  fused_topk(...)      softmax top-k routing of router logits; fused_moe_router(...) routes + runs
  grouped_topk(...)    group-limited sigmoid routing (DeepSeek-V3 router)
  pack_weights(...)    one-buffer weight format (16-bit, int8 or fp8); fused_moe_packed(...) runs on it
  host_pipeline.HostPipeline  host-buffer calls with transfers overlapped across calls
  graphs.GraphedMoE    one call captured into a CUDA graph and replayed
  torch_ops            torch.ops.muxi_race_b200.{fused_moe, fused_moe_int8, fused_moe_fp8, fused_topk,
                       run_kernel} (import to register)
  ep.ExpertParallelMoE expert-parallel fused MoE over torch.distributed (NCCL all-to-all)

All compute runs in hand-written CUDA kernels of ``libmoe_b200.so`` (C ABI in
``include/moe_b200.h``); there is no CPU or library fallback.
"""
from .fused import (Alignment, clear_workspace_cache, device_status, fused_moe, fused_moe_fp8, fused_moe_int8,
                    fused_moe_router, fused_topk, grouped_topk, max_padded_rows, moe_align, quantize_rows_fp8,
                    quantize_rows_int8)
from .packed import PackedWeights, fused_moe_packed, pack_weights
from .submission import run_kernel

__all__ = [
    "Alignment", "clear_workspace_cache", "device_status", "fused_moe", "fused_moe_fp8", "fused_moe_int8",
    "fused_moe_router", "fused_topk", "grouped_topk", "max_padded_rows", "moe_align", "quantize_rows_fp8", "quantize_rows_int8",
    "run_kernel", "PackedWeights", "fused_moe_packed", "pack_weights",
]
