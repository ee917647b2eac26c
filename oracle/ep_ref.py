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


# ----------------------------------------------------------------------------- peer-memory mode
def p2p_local_routes_ref(all_ids, expert_rank, expert_local, rank, T_max):
    """Virtual routes of the peer-memory mode for one rank: route r = (s * T_max + t) * k + j covers
    slot j of token t of rank s; local id = this rank's local index of that expert, -1 if another
    rank owns it or t is beyond rank s's token count (all_ids: one [T_s, k] tensor per rank)."""
    W = len(all_ids)
    k = all_ids[0].shape[1]
    local = torch.full((W * T_max * k,), -1, dtype=torch.int64)
    for s, ids in enumerate(all_ids):
        T_s = ids.shape[0]
        flat = ids.long().reshape(-1)
        own = expert_rank.long()[flat] == rank
        lid = torch.where(own, expert_local.long()[flat], torch.full_like(flat, -1))
        local[s * T_max * k: s * T_max * k + T_s * k] = lid
    return local


def p2p_partials_ref(all_x, all_ids, all_w, expert_rank, expert_local, rank, T_max, w13_local, w2_local):
    """Rank `rank`'s partial block y [W * T_max, H] (fp32): row s * T_max + t = sum over this rank's
    experts among token (s, t)'s top-k of weight * expert(x); rows without a local route are 0."""
    W = len(all_x)
    k = all_ids[0].shape[1]
    H = all_x[0].shape[1]
    local = p2p_local_routes_ref(all_ids, expert_rank, expert_local, rank, T_max).view(W, T_max, k)
    y = torch.zeros((W * T_max, H), dtype=torch.float32)
    for s in range(W):
        T_s = all_x[s].shape[0]
        if T_s == 0:
            continue
        ids = local[s, :T_s]
        w = torch.where(ids >= 0, all_w[s].float(), torch.zeros_like(all_w[s].float()))
        ids_c = ids.clamp(min=0)  # masked routes carry weight 0
        y[s * T_max: s * T_max + T_s] = fused_moe_ref(all_x[s], w13_local, w2_local, ids_c, w)
    return y


def p2p_combine_ref(partials, all_ids, expert_rank, rank, T_max, dtype):
    """out[t] of rank `rank` = sum, over the distinct owner ranks o of token t's experts in ascending
    order, of partials[o][rank * T_max + t] (fp32, then cast)."""
    ids = all_ids[rank].long()
    T = ids.shape[0]
    out = torch.zeros((T, partials[0].shape[1]), dtype=torch.float32)
    owners = expert_rank.long()[ids]  # [T, k]
    for o in range(len(partials)):
        m = (owners == o).any(dim=1)
        out[m] += partials[o][rank * T_max: rank * T_max + T][m].float()
    return out.to(dtype)


def p2p_push_ref(all_x, all_ids, all_w, expert_rank, expert_local, T_max, w13_by_rank, w2_by_rank):
    """Push combine: every owner o stores, for each virtual route r = (s * T_max + t) * k + j it owns,
    weight * expert(x) into slot t * k + j of home rank s's slot block (the destination map of the
    Stage2 epilogue in push mode: route r -> rank r // (T_max * k), slot r % (T_max * k)); the home
    then sums each token's slots j = 0..k-1 whose expert id is valid, in slot order. Returns one
    [T_s, H] fp32 output per rank and, to check that every slot has exactly one writer, the number
    of writes per slot of each rank."""
    W = len(all_x)
    k = all_ids[0].shape[1]
    H = all_x[0].shape[1]
    E = int(expert_rank.numel())
    slots = [torch.zeros((T_max * k, H), dtype=torch.float32) for _ in range(W)]
    writes = [torch.zeros(T_max * k, dtype=torch.int64) for _ in range(W)]
    for o in range(W):
        local = p2p_local_routes_ref(all_ids, expert_rank, expert_local, o, T_max)
        for r in torch.nonzero(local >= 0).flatten().tolist():
            home, slot = r // (T_max * k), r % (T_max * k)
            t, j = slot // k, slot % k
            x = all_x[home][t:t + 1]
            e_local = int(local[r])
            one = torch.zeros((1, 1), dtype=torch.int64)
            w = all_w[home][t:t + 1, j:j + 1].float()
            slots[home][slot] = fused_moe_ref(x, w13_by_rank[o][e_local:e_local + 1],
                                              w2_by_rank[o][e_local:e_local + 1], one, w)[0]
            writes[home][slot] += 1
    outs = []
    for s in range(W):
        ids = all_ids[s].long()
        T_s = ids.shape[0]
        out = torch.zeros((T_s, H), dtype=torch.float32)
        for t in range(T_s):
            for j in range(k):
                if 0 <= int(ids[t, j]) < E:
                    out[t] += slots[s][t * k + j]
        outs.append(out)
    return outs, writes
