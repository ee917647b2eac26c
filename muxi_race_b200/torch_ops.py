"""PyTorch operator registrations of the library's entry points (``torch.ops.muxi_race_b200.*``).

Registered as custom ops with shape functions, so models can call them like built-in operators:
they pass through ``torch.compile`` graphs as opaque nodes (the kernels stay this library's),
through CUDA-graph capture, and through meta / fake-tensor shape propagation.

    import muxi_race_b200.torch_ops  # registers the ops
    out = torch.ops.muxi_race_b200.fused_moe(x, w_gate_up, w_down, topk_ids, topk_weights)
    torch.ops.muxi_race_b200.run_kernel(x, gate_w, up_w, down_w, routed, gs, go, gpo, gidx, out)

The eager implementations are the Python entry points of this package (C ABI underneath).
"""
from typing import Optional

import torch
from torch import Tensor

from . import fused as _fused
from . import submission as _submission


@torch.library.custom_op("muxi_race_b200::fused_moe", mutates_args=())
def fused_moe(hidden_states: Tensor, w_gate_up: Tensor, w_down: Tensor, topk_ids: Tensor,
              topk_weights: Tensor) -> Tensor:
    return _fused.fused_moe(hidden_states, w_gate_up, w_down, topk_ids, topk_weights)


@fused_moe.register_fake
def _fused_moe_fake(hidden_states, w_gate_up, w_down, topk_ids, topk_weights):
    return hidden_states.new_empty(hidden_states.shape)


@torch.library.custom_op("muxi_race_b200::fused_moe_int8", mutates_args=())
def fused_moe_int8(hidden_states: Tensor, w13_q: Tensor, w13_scale: Tensor, w2_q: Tensor, w2_scale: Tensor,
                   topk_ids: Tensor, topk_weights: Tensor) -> Tensor:
    return _fused.fused_moe_int8(hidden_states, w13_q, w13_scale, w2_q, w2_scale, topk_ids, topk_weights)


@fused_moe_int8.register_fake
def _fused_moe_int8_fake(hidden_states, w13_q, w13_scale, w2_q, w2_scale, topk_ids, topk_weights):
    return hidden_states.new_empty(hidden_states.shape)


@torch.library.custom_op("muxi_race_b200::fused_moe_fp8", mutates_args=())
def fused_moe_fp8(hidden_states: Tensor, w13_q: Tensor, w13_scale: Tensor, w2_q: Tensor, w2_scale: Tensor,
                  topk_ids: Tensor, topk_weights: Tensor) -> Tensor:
    return _fused.fused_moe_fp8(hidden_states, w13_q, w13_scale, w2_q, w2_scale, topk_ids, topk_weights)


@fused_moe_fp8.register_fake
def _fused_moe_fp8_fake(hidden_states, w13_q, w13_scale, w2_q, w2_scale, topk_ids, topk_weights):
    return hidden_states.new_empty(hidden_states.shape)


@torch.library.custom_op("muxi_race_b200::fused_topk", mutates_args=())
def fused_topk(gating_output: Tensor, topk: int, renormalize: bool) -> tuple[Tensor, Tensor]:
    return _fused.fused_topk(gating_output, gating_output, topk, renormalize)


@fused_topk.register_fake
def _fused_topk_fake(gating_output, topk, renormalize):
    T = gating_output.shape[0]
    return (gating_output.new_empty((T, topk), dtype=torch.float32),
            gating_output.new_empty((T, topk), dtype=torch.int32))


@torch.library.custom_op("muxi_race_b200::grouped_topk", mutates_args=())
def grouped_topk(gating_output: Tensor, topk: int, renormalize: bool, num_expert_group: int, topk_group: int,
                 e_score_correction_bias: Optional[Tensor], routed_scaling_factor: float) -> tuple[Tensor, Tensor]:
    return _fused.grouped_topk(gating_output, gating_output, topk, renormalize, num_expert_group, topk_group,
                               e_score_correction_bias, routed_scaling_factor)


@grouped_topk.register_fake
def _grouped_topk_fake(gating_output, topk, renormalize, num_expert_group, topk_group, e_score_correction_bias,
                       routed_scaling_factor):
    T = gating_output.shape[0]
    return (gating_output.new_empty((T, topk), dtype=torch.float32),
            gating_output.new_empty((T, topk), dtype=torch.int32))


@torch.library.custom_op("muxi_race_b200::run_kernel", mutates_args=("out",))
def run_kernel(stacked_expert_tokens: Tensor, gate_w: Tensor, up_w: Tensor, down_w: Tensor,
               routed_expert_weights: Tensor, group_sizes: Tensor, group_offsets: Tensor,
               group_padded_offsets: Tensor, group_idx_for_bx: Tensor, out: Tensor) -> None:
    _submission.run_kernel(stacked_expert_tokens, gate_w, up_w, down_w, routed_expert_weights, group_sizes,
                           group_offsets, group_padded_offsets, group_idx_for_bx, out)


@run_kernel.register_fake
def _run_kernel_fake(stacked_expert_tokens, gate_w, up_w, down_w, routed_expert_weights, group_sizes,
                     group_offsets, group_padded_offsets, group_idx_for_bx, out):
    return None
