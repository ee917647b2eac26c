"""Oracle for the router step ahead of the fused MoE — TEST INFRASTRUCTURE ONLY.

Only ``tests/`` may use this module, as the checker of ``moe_router_topk`` / ``fused_topk``. The
product (``muxi_race_b200``) never imports it.

The reference receives its routing pre-built (the problem statement excludes the router); the
routing its benchmark inputs stand for, and the one the synthetic workloads here use, is
softmax -> top-k -> renormalise of router logits (``tests/golden/cases.py:118-129`` with torch).
``router_topk_ref`` restates it with the selection order made total, so that the ids are
comparable bit for bit:

* ids: the k largest logits per token, in descending order; logits compare by their fp32 value
  through an order-preserving integer image (every bit pattern has a place, +0 ranks above -0),
  and equal logits rank the lower expert id first (a stable sort);
* weights: ``torch.softmax`` in fp32 over all experts, gathered at the ids, divided by their sum
  when renormalising — the torch formula the workloads use.

Parity of the ids is pinned against ``torch.topk(torch.softmax(logits))`` on tie-free inputs
(``tests/test_router_ref.py``); with ties torch leaves the order unspecified and this oracle fixes it.
"""
from __future__ import annotations

import numpy as np
import torch


def order_keys(logits: torch.Tensor) -> np.ndarray:
    """Order-preserving uint32 image of the fp32 logits (negative: all bits flipped; else sign set)."""
    u = logits.detach().to(torch.float32).cpu().contiguous().numpy().view(np.uint32)
    return np.where(u & np.uint32(0x80000000), ~u, u | np.uint32(0x80000000)).astype(np.uint32)


def router_ids_ref(logits: torch.Tensor, topk: int) -> torch.Tensor:
    """[T, k] int32 expert ids: descending logit order, equal logits by ascending id."""
    keys = order_keys(logits).astype(np.int64)
    order = np.argsort(-keys, axis=1, kind="stable")[:, :topk]
    return torch.from_numpy(np.ascontiguousarray(order.astype(np.int32)))


def router_topk_ref(logits: torch.Tensor, topk: int, renormalize: bool = True):
    """(topk_weights [T, k] fp32, topk_ids [T, k] int32) on CPU."""
    ids = router_ids_ref(logits, topk)
    probs = torch.softmax(logits.detach().to(torch.float32).cpu(), dim=-1)
    w = torch.gather(probs, 1, ids.long())
    if renormalize:
        w = w / w.sum(-1, keepdim=True)
    return w.contiguous(), ids
