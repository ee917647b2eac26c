"""Reference of the expert-parallel dispatch/combine steps — TEST INFRASTRUCTURE ONLY.

Plain torch on any device, used by ``tests/`` to check the CUDA kernels ``moe_ep_plan``,
``moe_ep_pack`` and ``moe_ep_combine`` and to drive ``ExpertParallelMoE``'s exchange logic on CPU
ranks (gloo), where the CUDA kernels cannot run. The reference operator has no multi-GPU mode;
the parity target of the expert-parallel path is the single-process oracle
(``oracle.moe_ref.fused_moe_ref``) applied to the concatenated tokens of all ranks.
"""
from __future__ import annotations

import torch

from oracle.moe_ref import fused_moe_ref


def plan_ref(topk_ids: torch.Tensor, expert_rank: torch.Tensor, world: int):
    """(token, rank) pairs sorted by rank then token: send_counts [W], send_pairs [n], pair_slot [T*W]."""
    T, k = topk_ids.shape
    owner = expert_rank.long()[topk_ids.long()]                      # [T, k]
    hit = torch.zeros((T, world), dtype=torch.bool, device=topk_ids.device)
    hit.scatter_(1, owner, True)
    keys = torch.where(hit, torch.arange(world, device=topk_ids.device), torch.full_like(owner[:, :1], -1).expand(T, world))
    flat = keys.reshape(-1)
    valid = flat >= 0
    order = torch.argsort(torch.where(valid, flat, world), stable=True)[: int(valid.sum())]
    send_counts = torch.bincount(flat[valid], minlength=world).to(torch.int32)
    pair_slot = torch.full((T * world,), -1, dtype=torch.int32, device=topk_ids.device)
    pair_slot[order] = torch.arange(order.numel(), dtype=torch.int32, device=topk_ids.device)
    return send_counts, order.to(torch.int32), pair_slot


def pack_ref(x, topk_ids, topk_weights, send_pairs, expert_rank, expert_local, world):
    t = send_pairs.long() // world
    r = send_pairs.long() % world
    ids = topk_ids.long()[t]                                          # [n, k]
    mine = expert_rank.long()[ids] == r.unsqueeze(1)
    send_ids = torch.where(mine, expert_local.long()[ids], torch.full_like(ids, -1)).to(torch.int32)
    return x[t].contiguous(), send_ids, topk_weights[t].to(torch.float32).contiguous()


def combine_ref(y_back, pair_slot, T, world, dtype):
    H = y_back.shape[1]
    out = torch.zeros((T, H), dtype=torch.float32, device=y_back.device)
    slots = pair_slot.view(T, world).long()
    for r in range(world):
        s = slots[:, r]
        m = s >= 0
        out[m] += y_back[s[m]].float()
    return out.to(dtype)


class RefPlan:
    def __init__(self, send_counts, send_pairs, pair_slot):
        self.send_counts, self.send_pairs, self.pair_slot = send_counts, send_pairs, pair_slot


class ReferenceOps:
    """Drop-in for ``muxi_race_b200.ep.CudaOps`` on CPU tensors (gloo ranks)."""

    def __init__(self, placement):
        self.world = placement.world
        self.expert_rank = placement.expert_rank
        self.expert_local = placement.expert_local

    def plan(self, topk_ids):
        return RefPlan(*plan_ref(topk_ids, self.expert_rank, self.world))

    def pack(self, x, topk_ids, topk_weights, plan):
        return pack_ref(x, topk_ids, topk_weights, plan.send_pairs, self.expert_rank, self.expert_local, self.world)

    def local_moe(self, x, ids, w, w13, w2):
        return fused_moe_ref(x, w13, w2, ids, w).to(x.dtype)

    def combine(self, y_back, plan, T, H, dtype, out=None):
        res = combine_ref(y_back, plan.pair_slot, T, self.world, dtype)
        if out is not None:
            out.copy_(res)
            return out
        return res
