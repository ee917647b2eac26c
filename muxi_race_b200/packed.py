"""Packed expert weights: one device buffer in the layout the fused kernels read.

``pack_weights(gate_w, up_w, down_w, kind)`` turns the reference's weight tensors (gate_w, up_w
[E, I, H], down_w [E, H, I]; 初审材料/源代码/submission.py:2098-2109) into one buffer: w13
[E, 2I, H] with each expert's gate rows followed by its up rows (one TMA stream, one [gate | up]
accumulator per tile), w2 [E, H, I], and for the 8-bit kinds their per-row fp32 scales — each
section 256-byte aligned (``moe_packed_weights_layout``). The layout depends only on (E, H, I,
kind), so ``save`` / ``load`` move a packed set through a file as raw bytes plus a small header.
"""
from __future__ import annotations

import ctypes
import json
from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib
from .fused import _DTYPES, _ID_DTYPES, _W_DTYPES, _check, _stream, _workspace

KINDS = {"fp16": _lib.MOE_F16, "bf16": _lib.MOE_BF16, "int8": _lib.MOE_I8, "fp8": _lib.MOE_F8E4M3}
_MAGIC = "muxi_race_b200.packed_weights.v1"


def packed_layout(E: int, H: int, I: int, kind: str) -> tuple[list[int], int]:
    """(section offsets [w13, w13_scale, w2, w2_scale], total bytes) of a packed set."""
    off = (ctypes.c_size_t * 4)()
    total = ctypes.c_size_t(0)
    _lib.call("moe_packed_weights_layout", E, H, I, KINDS[kind], off, ctypes.byref(total))
    return list(off), int(total.value)


@dataclass
class PackedWeights:
    blob: torch.Tensor  # uint8 [total bytes]
    E: int
    H: int
    I: int
    kind: str           # "fp16" | "bf16" | "int8" | "fp8"

    def save(self, path: str) -> None:
        header = json.dumps({"magic": _MAGIC, "E": self.E, "H": self.H, "I": self.I, "kind": self.kind}).encode()
        with open(path, "wb") as f:
            f.write(len(header).to_bytes(8, "little"))
            f.write(header)
            f.write(self.blob.cpu().numpy().tobytes())

    @staticmethod
    def load(path: str, device="cuda") -> "PackedWeights":
        with open(path, "rb") as f:
            n = int.from_bytes(f.read(8), "little")
            meta = json.loads(f.read(n).decode())
            _check(meta.get("magic") == _MAGIC, f"{path} is not a packed weight file")
            data = f.read()
        _, total = packed_layout(meta["E"], meta["H"], meta["I"], meta["kind"])
        _check(len(data) == total, f"{path}: {len(data)} bytes of weights, the layout needs {total}")
        blob = torch.frombuffer(bytearray(data), dtype=torch.uint8).to(device)
        return PackedWeights(blob, meta["E"], meta["H"], meta["I"], meta["kind"])


def pack_weights(gate_w: torch.Tensor, up_w: torch.Tensor, down_w: torch.Tensor, kind: Optional[str] = None
                 ) -> PackedWeights:
    """Pack reference-layout weights (fp16/bf16 CUDA tensors); kind defaults to their dtype."""
    for t in (gate_w, up_w, down_w):
        _check(t.is_cuda and t.is_contiguous() and t.dtype in _DTYPES, "weights must be contiguous fp16/bf16 CUDA")
    _check(gate_w.dim() == 3 and gate_w.shape == up_w.shape, "gate_w and up_w must both be [E, I, H]")
    E, I, H = gate_w.shape
    _check(tuple(down_w.shape) == (E, H, I), f"down_w must be {(E, H, I)}")
    kind = kind or ("fp16" if gate_w.dtype == torch.float16 else "bf16")
    _check(kind in KINDS, f"kind must be one of {sorted(KINDS)}")
    _, total = packed_layout(E, H, I, kind)
    blob = torch.empty(total, dtype=torch.uint8, device=gate_w.device)
    _lib.call("moe_pack_weights", gate_w.data_ptr(), up_w.data_ptr(), down_w.data_ptr(), _DTYPES[gate_w.dtype],
              E, H, I, KINDS[kind], blob.data_ptr(), total, _stream(gate_w.device))
    return PackedWeights(blob, int(E), int(H), int(I), kind)


def fused_moe_packed(hidden_states: torch.Tensor, packed: PackedWeights, topk_ids: torch.Tensor,
                     topk_weights: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``fused_moe`` (or its int8 / fp8 route, by the packed kind) on packed weights."""
    _check(hidden_states.dim() == 2 and hidden_states.dtype in _DTYPES, "hidden_states must be fp16/bf16 [T, H]")
    T, H = hidden_states.shape
    _check(H == packed.H, f"hidden size {H} != packed {packed.H}")
    _check(topk_ids.shape == topk_weights.shape and topk_ids.dim() == 2 and topk_ids.shape[0] == T,
           "topk_ids and topk_weights must both be [T, topk]")
    for t in (hidden_states, packed.blob, topk_ids, topk_weights):
        _check(t.is_cuda and t.is_contiguous() and t.device == hidden_states.device,
               "all tensors must be contiguous CUDA tensors on one device")
    _check(topk_ids.dtype in _ID_DTYPES and topk_weights.dtype in _W_DTYPES, "bad routing dtypes")
    k = int(topk_ids.shape[1])
    if out is None:
        out = torch.empty((T, H), dtype=hidden_states.dtype, device=hidden_states.device)
    if T == 0:
        return out
    dev = hidden_states.device
    dt = _DTYPES[hidden_states.dtype]
    kind = KINDS[packed.kind]
    nbytes = _lib.lib().moe_fused_packed_workspace_bytes(T, k, packed.E, H, packed.I, kind, dt)
    ws = _workspace(("fused_packed", dev, _stream(dev)), nbytes, dev)
    _lib.call("moe_fused_packed", hidden_states.data_ptr(), packed.blob.data_ptr(), kind, topk_ids.data_ptr(),
              _ID_DTYPES[topk_ids.dtype], topk_weights.data_ptr(), _W_DTYPES[topk_weights.dtype], out.data_ptr(),
              T, H, packed.I, packed.E, k, dt, ws.data_ptr(), ws.numel(), _stream(dev))
    return out
