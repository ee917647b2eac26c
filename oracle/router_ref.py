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

``router_grouped_ref`` restates group-limited sigmoid routing (the published DeepSeek-V3 router:
sigmoid scores, a per-expert selection bias, groups scored by the sum of their two best biased
scores, the best ``topk_group`` groups eligible, weights = unbiased scores renormalised and scaled)
with the same total selection order.
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


def router_grouped_ref(logits: torch.Tensor, topk: int, n_group: int, topk_group: int, bias=None,
                       renormalize: bool = True, scale: float = 1.0):
    """(topk_weights [T, k] fp32, topk_ids [T, k] int32, margins) on CPU. ``margins`` [T] is, per
    token, the smallest relative gap at the selection boundaries (groups and experts), to tell
    near-ties (where a one-ulp difference in the sigmoid may change the choice) from real order."""
    lf = logits.detach().to(torch.float32).cpu()
    T, E = lf.shape
    s = torch.sigmoid(lf)
    c = s + (bias.detach().float().cpu() if bias is not None else 0.0)
    gs = E // n_group
    cg = c.view(T, n_group, gs)
    top2 = torch.sort(cg, dim=-1, descending=True).values
    gscore = top2[..., 0] + top2[..., 1] if gs > 1 else top2[..., 0]
    gkeys = order_keys(gscore).astype(np.int64)
    gorder = np.argsort(-gkeys, axis=1, kind="stable")
    sel = np.zeros((T, n_group), dtype=bool)
    np.put_along_axis(sel, gorder[:, :topk_group], True, axis=1)
    keys = order_keys(c).astype(np.int64)
    eligible = np.repeat(sel, gs, axis=1)
    keys = np.where(eligible, keys, -1)
    ids = np.argsort(-keys, axis=1, kind="stable")[:, :topk].astype(np.int32)
    w = torch.gather(s, 1, torch.from_numpy(ids).long())
    if renormalize:
        w = w / (w.sum(-1, keepdim=True) + 1e-20)
    w = w * scale
    # boundary gaps (relative): group topk_group vs topk_group + 1, expert topk vs topk + 1
    gsorted = torch.sort(gscore, dim=-1, descending=True).values
    cm = torch.where(torch.from_numpy(eligible), c, torch.full_like(c, -float("inf")))
    csorted = torch.sort(cm, dim=-1, descending=True).values
    inf = torch.full((T,), float("inf"))
    ggap = (gsorted[:, topk_group - 1] - gsorted[:, topk_group]).abs() if topk_group < n_group else inf
    cgap = (csorted[:, topk - 1] - csorted[:, topk]).abs() if topk < topk_group * gs else inf
    # An exact tie between candidates computed from identical inputs is not a near-tie: any
    # implementation computes the same score for both and breaks the tie by the lower id. With bf16
    # logits such ties are frequent. (Expert boundary: same logit and bias; group boundary: the
    # same two best c values.)
    b = bias.detach().float().cpu() if bias is not None else torch.zeros(E)
    if topk < topk_group * gs:
        cidx = torch.sort(cm, dim=-1, descending=True, stable=True).indices
        ea, eb = cidx[:, topk - 1], cidx[:, topk]
        same = (lf.gather(1, ea[:, None]) == lf.gather(1, eb[:, None])).squeeze(1) & (b[ea] == b[eb])
        cgap = torch.where((cgap == 0) & same, inf, cgap)
    if topk_group < n_group:
        go = torch.from_numpy(gorder).long()
        ga, gb = go[:, topk_group - 1], go[:, topk_group]
        t2 = top2[..., :2] if gs > 1 else top2[..., :1]
        ar = torch.arange(T)
        same = (t2[ar, ga] == t2[ar, gb]).all(-1)
        ggap = torch.where((ggap == 0) & same, inf, ggap)
    margins = torch.minimum(ggap / gsorted[:, 0].abs().clamp_min(1e-30), cgap / csorted[:, 0].abs().clamp_min(1e-30))
    return w.contiguous(), torch.from_numpy(np.ascontiguousarray(ids)), margins
