"""Expert-parallel fused MoE over torch.distributed (one process per GPU, NCCL all-to-all).

The reference operator runs on one GPU (初审材料/源代码/submission.py:2098); this module shards
its experts across ranks. Rank r holds the weights of ``placement.local_experts(r)`` and its own
share of the tokens. A forward:

1. ``moe_ep_plan``     (token, rank) pairs for every rank that owns one of the token's top-k
                       experts, sorted by rank then token; send counts per rank;
2. counts exchange     ``all_to_all_single`` of W int32 counts, copied to the host once (the only
                       host synchronisation: NCCL needs split sizes on the host);
3. dispatch            ``moe_ep_pack`` gathers the token rows with destination-local expert ids
                       (-1 for experts owned elsewhere) and routing weights, then three
                       ``all_to_all_single`` calls move rows, ids and weights;
4. local fused MoE     ``fused_moe`` with the local experts; its Stage2 epilogue combines each
                       received token's local routes;
5. combine             the reverse ``all_to_all_single`` returns the partial rows, and
                       ``moe_ep_combine`` sums each token's partials in rank order.

Compute steps go through an ``ops`` object: the default uses the CUDA kernels of
``libmoe_b200.so``; tests of the exchange logic on CPU ranks (gloo) pass a reference
implementation instead. Every rank issues the same collectives in the same order.
"""
from __future__ import annotations

import heapq
from dataclasses import dataclass
from typing import Optional, Sequence

import torch
import torch.distributed as dist

from . import _lib
from .fused import _DTYPES, _ID_DTYPES, _W_DTYPES, _stream, _workspace, fused_moe


# ----------------------------------------------------------------------------- placement
@dataclass
class ExpertPlacement:
    """Owner rank and local index of every expert (int32 tensors [E] on the host)."""

    expert_rank: torch.Tensor
    expert_local: torch.Tensor
    world: int

    @property
    def num_experts(self) -> int:
        return int(self.expert_rank.numel())

    def local_experts(self, rank: int) -> list[int]:
        ids = torch.nonzero(self.expert_rank == rank).flatten()
        order = torch.argsort(self.expert_local[ids])
        return ids[order].tolist()

    @classmethod
    def contiguous(cls, num_experts: int, world: int) -> "ExpertPlacement":
        """Experts [r*E/W, (r+1)*E/W) on rank r."""
        if num_experts % world:
            raise ValueError("num_experts must be divisible by world")
        per = num_experts // world
        e = torch.arange(num_experts, dtype=torch.int32)
        return cls(e // per, e % per, world)

    @classmethod
    def balanced(cls, loads: Sequence[float], world: int) -> "ExpertPlacement":
        """Greedy longest-processing-time placement with E/W experts per rank: experts in decreasing
        load go to the least-loaded rank that still has room (loads from a calibration histogram)."""
        E = len(loads)
        if E % world:
            raise ValueError("num_experts must be divisible by world")
        cap = E // world
        order = sorted(range(E), key=lambda e: (-float(loads[e]), e))
        heap = [(0.0, r) for r in range(world)]
        count = [0] * world
        rank = torch.empty(E, dtype=torch.int32)
        local = torch.empty(E, dtype=torch.int32)
        for e in order:
            skipped = []
            while True:
                load, r = heapq.heappop(heap)
                if count[r] < cap:
                    break
                skipped.append((load, r))
            rank[e] = r
            local[e] = count[r]
            count[r] += 1
            heapq.heappush(heap, (load + float(loads[e]), r))
            for item in skipped:
                heapq.heappush(heap, item)
        return cls(rank, local, world)

    def max_over_mean_load(self, loads: Sequence[float]) -> float:
        per = torch.zeros(self.world, dtype=torch.float64)
        per.index_add_(0, self.expert_rank.long(), torch.as_tensor(loads, dtype=torch.float64))
        return float(per.max() / per.mean())


# ----------------------------------------------------------------------------- compute ops
@dataclass
class Plan:
    send_counts: torch.Tensor   # [W] int32 (device)
    send_pairs: torch.Tensor    # [T*W] int32
    pair_slot: torch.Tensor     # [T*W] int32
    meta: torch.Tensor          # [4] int32


class CudaOps:
    """Dispatch / combine kernels of libmoe_b200.so and the local fused MoE."""

    def __init__(self, placement: ExpertPlacement, device: torch.device):
        self.device = device
        self.world = placement.world
        self.E = placement.num_experts
        self.expert_rank = placement.expert_rank.to(device=device, dtype=torch.int32).contiguous()
        self.expert_local = placement.expert_local.to(device=device, dtype=torch.int32).contiguous()

    def plan(self, topk_ids: torch.Tensor) -> Plan:
        T, k = topk_ids.shape
        W = self.world
        i32 = dict(dtype=torch.int32, device=self.device)
        p = Plan(torch.empty(W, **i32), torch.empty(max(T * W, 1), **i32), torch.empty(max(T * W, 1), **i32),
                 torch.empty(4, **i32))
        offsets = torch.empty(W + 1, **i32)
        nbytes = _lib.lib().moe_ep_plan_workspace_bytes(T, W)
        ws = _workspace(("ep_plan", self.device, T, W, _stream(self.device)), nbytes, self.device)
        _lib.call("moe_ep_plan", topk_ids.data_ptr(), _ID_DTYPES[topk_ids.dtype], T, k, self.expert_rank.data_ptr(),
                  self.E, W, p.send_counts.data_ptr(), offsets.data_ptr(), p.send_pairs.data_ptr(),
                  p.pair_slot.data_ptr(), p.meta.data_ptr(), ws.data_ptr(), ws.numel(), _stream(self.device))
        return p

    def pack(self, x, topk_ids, topk_weights, plan: Plan):
        T, H = x.shape
        k = topk_ids.shape[1]
        cap = max(T * min(self.world, k), 1)
        send_x = torch.empty((cap, H), dtype=x.dtype, device=self.device)
        send_ids = torch.empty((cap, k), dtype=torch.int32, device=self.device)
        send_w = torch.empty((cap, k), dtype=torch.float32, device=self.device)
        _lib.call("moe_ep_pack", x.data_ptr(), topk_ids.data_ptr(), _ID_DTYPES[topk_ids.dtype], topk_weights.data_ptr(),
                  _W_DTYPES[topk_weights.dtype], self.expert_rank.data_ptr(), self.expert_local.data_ptr(), self.E,
                  plan.send_pairs.data_ptr(), plan.meta.data_ptr(), T, H, k, self.world, _DTYPES[x.dtype],
                  send_x.data_ptr(), send_ids.data_ptr(), send_w.data_ptr(), _stream(self.device))
        return send_x, send_ids, send_w

    def local_moe(self, x, ids, w, w13, w2):
        return fused_moe(x, w13, w2, ids, w)

    def combine(self, y_back, plan: Plan, T: int, H: int, dtype) -> torch.Tensor:
        out = torch.empty((T, H), dtype=dtype, device=self.device)
        _lib.call("moe_ep_combine", y_back.data_ptr() if y_back.numel() else None, plan.pair_slot.data_ptr(), T, H,
                  self.world, _DTYPES[dtype], out.data_ptr(), _stream(self.device))
        return out


# ----------------------------------------------------------------------------- the module
class ExpertParallelMoE:
    """Fused MoE with experts sharded over the ranks of ``group``.

    w_gate_up_local [E_local, 2I, H] and w_down_local [E_local, H, I] hold this rank's experts in
    ``placement.local_experts(rank)`` order. ``forward`` takes this rank's tokens.
    """

    def __init__(self, w_gate_up_local: torch.Tensor, w_down_local: torch.Tensor, placement: ExpertPlacement,
                 group: Optional[dist.ProcessGroup] = None, ops=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if placement.world != self.world:
            raise ValueError(f"placement is for {placement.world} ranks, group has {self.world}")
        n_local = len(placement.local_experts(self.rank))
        if w_gate_up_local.shape[0] != n_local or w_down_local.shape[0] != n_local:
            raise ValueError(f"rank {self.rank} owns {n_local} experts, weights hold {w_gate_up_local.shape[0]}")
        self.w13 = w_gate_up_local
        self.w2 = w_down_local
        self.placement = placement
        self.ops = ops if ops is not None else CudaOps(placement, w_gate_up_local.device)
        self.last_counts: Optional[tuple[list[int], list[int]]] = None
        self.last_recv_ids: Optional[torch.Tensor] = None  # for statistics (local routed rows)

    def _a2a(self, out, inp, out_splits, in_splits):
        dist.all_to_all_single(out, inp, output_split_sizes=out_splits, input_split_sizes=in_splits, group=self.group)

    def forward(self, hidden_states: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor) -> torch.Tensor:
        x = hidden_states
        T, H = x.shape
        k = topk_ids.shape[1]
        plan = self.ops.plan(topk_ids)
        send_x, send_ids, send_w = self.ops.pack(x, topk_ids, topk_weights, plan)

        recv_counts = torch.empty_like(plan.send_counts)
        dist.all_to_all_single(recv_counts, plan.send_counts, group=self.group)
        counts = torch.stack([plan.send_counts, recv_counts]).cpu()
        send_splits = [int(c) for c in counts[0]]
        recv_splits = [int(c) for c in counts[1]]
        n_send, n_recv = sum(send_splits), sum(recv_splits)
        if min(send_splits + recv_splits) < 0 or n_send > send_x.shape[0]:
            raise RuntimeError(f"rank {self.rank}: inconsistent exchange counts send={send_splits} recv={recv_splits}")
        self.last_counts = (send_splits, recv_splits)

        dev = x.device
        recv_x = torch.empty((n_recv, H), dtype=x.dtype, device=dev)
        recv_ids = torch.empty((n_recv, k), dtype=torch.int32, device=dev)
        recv_w = torch.empty((n_recv, k), dtype=torch.float32, device=dev)
        self._a2a(recv_x, send_x[:n_send], recv_splits, send_splits)
        self._a2a(recv_ids, send_ids[:n_send], recv_splits, send_splits)
        self._a2a(recv_w, send_w[:n_send], recv_splits, send_splits)

        self.last_recv_ids = recv_ids
        if n_recv > 0:
            y = self.ops.local_moe(recv_x, recv_ids, recv_w, self.w13, self.w2)
        else:
            y = torch.empty((0, H), dtype=x.dtype, device=dev)
        y_back = torch.empty((n_send, H), dtype=x.dtype, device=dev)
        self._a2a(y_back, y, send_splits, recv_splits)
        return self.ops.combine(y_back, plan, T, H, x.dtype)

    __call__ = forward
