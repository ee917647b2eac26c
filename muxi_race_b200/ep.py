"""Expert-parallel fused MoE over torch.distributed (one process per GPU, NCCL all-to-all).

The reference operator runs on one GPU (初审材料/源代码/submission.py:2098); this module shards
its experts across ranks. Rank r holds the weights of ``placement.local_experts(r)`` and its own
share of the tokens. A forward:

1. ``moe_ep_plan``     (token, rank) pairs for every rank that owns one of the token's top-k
                       experts, sorted by rank then token; send counts per rank;
2. counts exchange     ``all_to_all_single`` of W int32 counts, copied to the host once (the only
                       host synchronisation: NCCL needs split sizes on the host);
3. dispatch            ``moe_ep_pack`` gathers the token rows with destination-local expert ids
                       (-1 for experts owned elsewhere) and routing weights, then two
                       ``all_to_all_single`` calls move the rows and the [n, 2k] ids+weights;
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
import contextlib
import ctypes
from dataclasses import dataclass
from typing import Optional, Sequence

import torch
import torch.distributed as dist

from . import _lib
from ._lib import _c_void_p
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
        ws = _workspace(("ep_plan", self.device, _stream(self.device)), nbytes, self.device)
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

    def combine(self, y_back, plan: Plan, T: int, H: int, dtype, out=None) -> torch.Tensor:
        if out is None:
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
                 group: Optional[dist.ProcessGroup] = None, ops=None, chunks: int = 1, min_chunk_tokens: int = 512):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if placement.world != self.world:
            raise ValueError(f"placement is for {placement.world} ranks, group has {self.world}")
        n_local = len(placement.local_experts(self.rank))
        if w_gate_up_local.shape[0] != n_local or w_down_local.shape[0] != n_local:
            raise ValueError(f"rank {self.rank} owns {n_local} experts, weights hold {w_gate_up_local.shape[0]}")
        if chunks < 1:
            raise ValueError("chunks must be >= 1")
        self.w13 = w_gate_up_local
        self.w2 = w_down_local
        self.placement = placement
        self.ops = ops if ops is not None else CudaOps(placement, w_gate_up_local.device)
        self.chunks = chunks
        self.min_chunk_tokens = min_chunk_tokens
        self._comm_streams: dict = {}
        self.last_counts: Optional[tuple[list[int], list[int]]] = None
        self._last_recv_ids: list = []

    @property
    def last_recv_ids(self) -> Optional[torch.Tensor]:
        """Destination-local expert ids of the rows this rank received in the last forward."""
        if not self._last_recv_ids:
            return None
        return torch.cat(self._last_recv_ids)

    def _a2a(self, out, inp, out_splits, in_splits):
        dist.all_to_all_single(out, inp, output_split_sizes=out_splits, input_split_sizes=in_splits, group=self.group)

    def _comm_stream(self, device):
        st = self._comm_streams.get(device)
        if st is None:
            st = self._comm_streams[device] = torch.cuda.Stream(device=device)
        return st

    def forward(self, hidden_states: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor) -> torch.Tensor:
        """This rank's tokens are split into up to ``chunks`` contiguous chunks (at least
        ``min_chunk_tokens`` each). On GPUs the exchanges run on a communication stream: chunk
        c+1's dispatch overlaps chunk c's local MoE, and chunk c's return overlaps chunk c+1's
        local MoE. Every rank takes part in all ``chunks`` rounds of exchanges, with empty sends for
        chunks it does not have, so the collectives match across ranks whatever their token
        counts."""
        x = hidden_states
        T, H = x.shape
        k = topk_ids.shape[1]
        W = self.world
        C = max(1, min(self.chunks, T // max(self.min_chunk_tokens, 1)))
        bounds = [(T * c // C, T * (c + 1) // C) for c in range(C)]
        plans, packs = [], []
        for a, b in bounds:
            p = self.ops.plan(topk_ids[a:b])
            plans.append(p)
            packs.append(self.ops.pack(x[a:b], topk_ids[a:b], topk_weights[a:b], p))

        # one count exchange for all chunks: [W, C] per rank; also agrees on the chunk count
        dev = x.device
        send_counts = torch.zeros((W, self.chunks), dtype=torch.int32, device=dev)
        send_counts[:, :C] = torch.stack([p.send_counts for p in plans], dim=1)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        counts = torch.stack([send_counts, recv_counts]).cpu()
        send_splits = [[int(v) for v in counts[0, :, c]] for c in range(self.chunks)]
        recv_splits = [[int(v) for v in counts[1, :, c]] for c in range(self.chunks)]
        for c in range(self.chunks):
            n_send = sum(send_splits[c])
            cap = packs[c][0].shape[0] if c < C else 0
            if min(send_splits[c] + recv_splits[c]) < 0 or n_send > cap:
                raise RuntimeError(f"rank {self.rank}: inconsistent exchange counts send={send_splits[c]} "
                                   f"recv={recv_splits[c]} (chunk {c})")
        self.last_counts = ([sum(v) for v in zip(*send_splits)], [sum(v) for v in zip(*recv_splits)])
        # a chunk this rank does not have still takes part in every exchange (with empty sends)
        while len(packs) < self.chunks:
            packs.append((x[:0], topk_ids[:0].to(torch.int32), topk_weights[:0].float()))
            plans.append(None)
            bounds.append((T, T))

        cuda = x.is_cuda
        main = torch.cuda.current_stream(dev) if cuda else None
        comm = self._comm_stream(dev) if (cuda and self.chunks > 1) else main
        split = cuda and comm is not main

        def on(stream):
            return torch.cuda.stream(stream) if split else contextlib.nullcontext()

        def keep(t, stream):  # a tensor used on another stream than the one it was allocated on
            if split and t.numel():
                t.record_stream(stream)

        if split:
            comm.wait_stream(main)
        received = []
        with on(comm):
            for c in range(self.chunks):
                send_x, send_ids, send_w = packs[c]
                ss, rs = send_splits[c], recv_splits[c]
                n_send, n_recv = sum(ss), sum(rs)
                keep(send_x, comm)
                recv_x = torch.empty((n_recv, H), dtype=x.dtype, device=dev)
                self._a2a(recv_x, send_x[:n_send], rs, ss)
                # ids and weights travel together: one [n, 2k] int32 exchange (weights as fp32 bits)
                send_iw = torch.cat([send_ids[:n_send].to(torch.int32), send_w[:n_send].float().view(torch.int32)],
                                    dim=1)
                recv_iw = torch.empty((n_recv, 2 * k), dtype=torch.int32, device=dev)
                self._a2a(recv_iw, send_iw, rs, ss)
                keep(recv_x, main)
                keep(recv_iw, main)
                received.append((recv_x, recv_iw, comm.record_event() if split else None))

        out = torch.empty((T, H), dtype=x.dtype, device=dev)
        returned = []
        self._last_recv_ids = []
        for c in range(self.chunks):
            recv_x, recv_iw, ev = received[c]
            ss, rs = send_splits[c], recv_splits[c]
            if split:
                main.wait_event(ev)
            recv_ids = recv_iw[:, :k].contiguous()
            recv_w = recv_iw[:, k:].contiguous().view(torch.float32)
            self._last_recv_ids.append(recv_ids)
            if recv_x.shape[0] > 0:
                y = self.ops.local_moe(recv_x, recv_ids, recv_w, self.w13, self.w2)
            else:
                y = torch.empty((0, H), dtype=x.dtype, device=dev)
            keep(y, comm)
            ev_y = main.record_event() if split else None
            with on(comm):
                if split:
                    comm.wait_event(ev_y)
                y_back = torch.empty((sum(ss), H), dtype=x.dtype, device=dev)
                self._a2a(y_back, y, ss, rs)
                keep(y_back, main)
                returned.append((y_back, comm.record_event() if split else None))
        for c in range(self.chunks):
            a, b = bounds[c]
            y_back, ev = returned[c]
            if split:
                main.wait_event(ev)
            if b > a:
                self.ops.combine(y_back, plans[c], b - a, H, x.dtype, out=out[a:b])
        return out

    __call__ = forward


# ----------------------------------------------------------------------------- peer-memory mode
class PeerMemoryEP:
    """Expert-parallel fused MoE over NVLink peer memory (one process per GPU of one node).

    Same operator and weights as ``ExpertParallelMoE``; the exchange runs in the library's kernels
    instead of NCCL all-to-alls: every rank's region (staged inputs and the partial outputs it
    computes for all ranks' tokens) is mapped into every other rank by CUDA IPC. A forward issues,
    on the current stream and without host synchronisation: stage -> barrier -> compute (route,
    gather from the peers, Stage1 / Stage2) -> barrier -> combine (sum the owners' partials).
    ``max_tokens`` bounds the tokens per rank per forward; every rank must construct the module
    (collective: the IPC handles are exchanged through ``group``) and call ``forward`` the same
    number of times; ``close`` is collective too.

    ``combine="push"``: instead of the pull after the second barrier, Stage2's epilogue stores each
    route's weighted row into that route's slot in its token's home rank's region over NVLink
    (overlapping the GEMM; one writer per slot, no atomics); after the second barrier the home sums
    each token's slots locally in slot order.
    """

    def __init__(self, w_gate_up_local: torch.Tensor, w_down_local: torch.Tensor, placement: ExpertPlacement,
                 max_tokens: int, topk: int, group: Optional[dist.ProcessGroup] = None, combine: str = "pull"):
        if combine not in ("pull", "push"):
            raise ValueError("combine must be 'pull' or 'push'")
        self.push = combine == "push"
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if placement.world != self.world:
            raise ValueError(f"placement is for {placement.world} ranks, group has {self.world}")
        n_local = len(placement.local_experts(self.rank))
        if w_gate_up_local.shape[0] != n_local or w_down_local.shape[0] != n_local:
            raise ValueError(f"rank {self.rank} owns {n_local} experts, weights hold {w_gate_up_local.shape[0]}")
        if w_gate_up_local.dtype not in _DTYPES or not w_gate_up_local.is_cuda:
            raise ValueError("weights must be fp16/bf16 CUDA tensors")
        self.w13, self.w2 = w_gate_up_local.contiguous(), w_down_local.contiguous()
        self.device = self.w13.device
        self.dtype = self.w13.dtype
        self.H, self.I = int(self.w13.shape[2]), int(self.w2.shape[2])
        self.E_local, self.E = n_local, placement.num_experts
        self.T_max, self.k = int(max_tokens), int(topk)
        self.expert_rank = placement.expert_rank.to(device=self.device, dtype=torch.int32).contiguous()
        self.expert_local = placement.expert_local.to(device=self.device, dtype=torch.int32).contiguous()
        lib = _lib.lib()
        nbytes = lib.moe_ep_region_bytes(self.T_max, self.H, self.k, self.world)
        if nbytes == 0:
            raise ValueError("unsupported region shape")
        self._region = _c_void_p()
        _lib.call("moe_ep_region_alloc", nbytes, ctypes.byref(self._region))
        handle = (ctypes.c_char * 64)()
        _lib.call("moe_ep_ipc_get", self._region, handle)
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self._opened = []
        ptrs = []
        for q, h in enumerate(handles):
            if q == self.rank:
                ptrs.append(self._region.value)
                continue
            p = _c_void_p()
            _lib.call("moe_ep_ipc_open", ctypes.create_string_buffer(h, 64), ctypes.byref(p))
            self._opened.append(p)
            ptrs.append(p.value)
        self.regions = torch.tensor(ptrs, dtype=torch.int64, device=self.device)
        self._epoch = 0
        self._ws_bytes = lib.moe_ep_p2p_workspace_bytes(self.T_max, self.k, self.world, self.E_local, self.H, self.I,
                                                        _DTYPES[self.dtype])
        self._closed = False

    def _barrier(self, stream):
        self._epoch = (self._epoch + 1) & 0xFFFFFFFF
        _lib.call("moe_ep_p2p_barrier", self.regions.data_ptr(), self.rank, self.world, self._epoch, stream)

    def forward(self, hidden_states: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor) -> torch.Tensor:
        if self._closed:
            raise RuntimeError("module closed")
        x, ids, w = hidden_states.contiguous(), topk_ids.contiguous(), topk_weights.contiguous()
        T = int(x.shape[0])
        if T > self.T_max or x.shape[1] != self.H or ids.shape != (T, self.k) or w.shape != (T, self.k):
            raise ValueError(f"expected hidden_states [T <= {self.T_max}, {self.H}], topk ids/weights [T, {self.k}]")
        if x.dtype != self.dtype:
            raise ValueError("hidden_states dtype must match the weights")
        stream = _stream(self.device)
        dt = _DTYPES[self.dtype]
        _lib.call("moe_ep_p2p_stage", self._region, x.data_ptr(), ids.data_ptr(), _ID_DTYPES[ids.dtype], w.data_ptr(),
                  _W_DTYPES[w.dtype], T, self.T_max, self.H, self.k, self.world, dt, stream)
        if self.push:
            _lib.call("moe_ep_p2p_push_prepare", self._region, T, self.T_max, self.H, self.k, self.world, dt, stream)
        self._barrier(stream)
        ws = _workspace(("ep_p2p", self.device, self.T_max, self.k, self.world, self.E_local, stream), self._ws_bytes,
                        self.device)
        _lib.call("moe_ep_p2p_compute_push" if self.push else "moe_ep_p2p_compute", self.regions.data_ptr(),
                  self._region, self.rank, self.world, self.T_max, self.H, self.I, self.k,
                  self.expert_rank.data_ptr(), self.expert_local.data_ptr(), self.E, self.w13.data_ptr(),
                  self.w2.data_ptr(), self.E_local, dt, ws.data_ptr(), ws.numel(), stream)
        self._barrier(stream)
        out = torch.empty((T, self.H), dtype=self.dtype, device=self.device)
        if self.push:
            _lib.call("moe_ep_p2p_push_finish", self._region, T, self.T_max, self.H, self.k, self.world, self.E, dt,
                      out.data_ptr(), stream)
        else:
            _lib.call("moe_ep_p2p_combine", self.regions.data_ptr(), self.rank, self.world, T, self.T_max, self.H,
                      self.k, self.expert_rank.data_ptr(), self.E, dt, out.data_ptr(), stream)
        return out

    __call__ = forward

    def close(self) -> None:
        """Collective: after every rank's last forward has finished, unmap the peers and free."""
        if self._closed:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for p in self._opened:
            _lib.call("moe_ep_ipc_close", p)
        _lib.call("moe_ep_region_free", self._region)
        self._opened, self._closed = [], True
