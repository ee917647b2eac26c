"""Drop-in replacement for the contest operator's Python entry point.

``run_kernel`` keeps the reference signature and semantics (初审材料/源代码/submission.py:2098-2184):
ten positional tensors, ``out`` is the only tensor written, padding rows of ``out`` end up 0,
empty inputs take the same shortcuts (:2117-2153), the ``up_logits`` scratch is cached (:2081-2095;
here per device and stream, grown as needed) and both fp32 and fp16 routed weights are accepted
(:2125-2128). The work runs in
two sm_100a kernels of ``libmoe_b200.so`` on the current CUDA stream, with no host
synchronisation.
"""
from __future__ import annotations

import threading

import torch

from . import _lib

_WORKSPACE_CACHE: dict = {}
_WS_LOCK = threading.Lock()

_DTYPES = {torch.float16: _lib.MOE_F16, torch.bfloat16: _lib.MOE_BF16}
_ROUTED_DTYPES = {torch.float32: _lib.MOE_F32, torch.float16: _lib.MOE_F16}


def _stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _get_workspace(x: torch.Tensor, intermediate: int) -> torch.Tensor:
    """Scratch for the Stage1 output ``up_logits`` [P, I] (reference ``_get_workspace``, which caches
    one buffer per shape). Here one buffer per device and stream, grown when a call needs more:
    calls on one stream run in order, so they can share it whatever their shapes, calls on
    different streams never share it, and the cache is bounded by the largest call."""
    nbytes = _lib.lib().moe_run_kernel_workspace_bytes(x.shape[0], intermediate, _DTYPES[x.dtype])
    key = (x.device, _stream_handle(x.device))
    with _WS_LOCK:
        ws = _WORKSPACE_CACHE.get(key)
        if ws is None or ws.numel() < nbytes:
            ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=x.device)
            _WORKSPACE_CACHE[key] = ws
    return ws


def _require(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(msg)


def run_kernel(
    stacked_expert_tokens: torch.Tensor,
    gate_w: torch.Tensor,
    up_w: torch.Tensor,
    down_w: torch.Tensor,
    routed_expert_weights: torch.Tensor,
    group_sizes: torch.Tensor,
    group_offsets: torch.Tensor,
    group_padded_offsets: torch.Tensor,
    group_idx_for_bx: torch.Tensor,
    out: torch.Tensor,
) -> None:
    """out[p] = (silu(x_p Wg_e^T) * (x_p Wu_e^T)) Wd_e^T * routed[raw(p)] for valid rows, 0 for padding.

    Same arguments as the reference ``run_kernel``. Tensors must be contiguous CUDA tensors on one
    device; token/weight/output dtype fp16 or bf16 (the reference is fp16 only); metadata int32.
    """
    x = stacked_expert_tokens
    hidden = int(x.shape[1])
    intermediate = int(gate_w.shape[1])
    num_experts = int(gate_w.shape[0])
    total_padded_tokens = int(x.shape[0])
    total_valid_tokens = int(routed_expert_weights.shape[0])
    num_blocks_m = int(group_idx_for_bx.shape[0])

    tensors = (x, gate_w, up_w, down_w, routed_expert_weights, group_sizes, group_offsets,
               group_padded_offsets, group_idx_for_bx, out)
    _require(all(t.is_cuda for t in tensors), "run_kernel: all tensors must be CUDA tensors")
    _require(all(t.device == x.device for t in tensors), "run_kernel: tensors on different devices")
    _require(all(t.is_contiguous() for t in tensors), "run_kernel: tensors must be contiguous")
    _require(x.dtype in _DTYPES, f"run_kernel: unsupported token dtype {x.dtype}")
    _require(gate_w.dtype == x.dtype and up_w.dtype == x.dtype and down_w.dtype == x.dtype and out.dtype == x.dtype,
             "run_kernel: tokens, weights and out must share one dtype")
    _require(routed_expert_weights.dtype in _ROUTED_DTYPES, "run_kernel: routed weights must be fp32 or fp16")
    _require(all(t.dtype == torch.int32 for t in (group_sizes, group_offsets, group_padded_offsets, group_idx_for_bx)),
             "run_kernel: group metadata must be int32")
    _require(tuple(up_w.shape) == (num_experts, intermediate, hidden), "run_kernel: up_w shape mismatch")
    _require(tuple(gate_w.shape) == (num_experts, intermediate, hidden), "run_kernel: gate_w shape mismatch")
    _require(tuple(down_w.shape) == (num_experts, hidden, intermediate), "run_kernel: down_w shape mismatch")
    _require(tuple(out.shape) == (total_padded_tokens, hidden), "run_kernel: out shape mismatch")
    _require(group_sizes.numel() == num_experts and group_offsets.numel() == num_experts + 1
             and group_padded_offsets.numel() == num_experts + 1, "run_kernel: group metadata length mismatch")

    if total_padded_tokens == 0:  # reference :2117-2120
        return
    ws = _get_workspace(x, intermediate) if total_valid_tokens > 0 else None
    _lib.call(
        "moe_run_kernel",
        x.data_ptr(), gate_w.data_ptr(), up_w.data_ptr(), down_w.data_ptr(),
        routed_expert_weights.data_ptr() if total_valid_tokens > 0 else None,
        _ROUTED_DTYPES[routed_expert_weights.dtype],
        group_sizes.data_ptr(), group_offsets.data_ptr(), group_padded_offsets.data_ptr(),
        group_idx_for_bx.data_ptr() if num_blocks_m > 0 else None,
        out.data_ptr(),
        total_padded_tokens, hidden, intermediate, num_experts, total_valid_tokens, num_blocks_m,
        _DTYPES[x.dtype],
        ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0,
        _stream_handle(x.device),
    )
