"""Fused MoE on host (pinned) buffers with the transfers of consecutive calls overlapped.

A serving loop that keeps its activations in host memory pays, per call, a host->device copy of
the token rows and routing and a device->host copy of the result (about 118 MB per call at the
T=4096, H=7168 shape). Issued on the compute stream they add to every call; here they run on two
copy streams, double-buffered, so call i+1's upload and call i-1's download overlap call i's
kernels (PCIe / C2C copies in each direction run beside HBM-bound compute).

    pipe = HostPipeline(lambda x, ids, w, out: fused_moe(x, w13, w2, ids, w, out=out),
                        x_like, ids_like, w_like, out_like)
    for x_h, ids_h, w_h, out_h in batches:       # pinned host tensors
        pipe.submit([x_h, ids_h, w_h], out_h)
    pipe.synchronize()                             # every out_h is filled

Ordering per buffer slot: upload waits until the slot's previous call has consumed its inputs;
compute waits for its upload and for the slot's previous download; download waits for compute.
All waits are stream-event waits: nothing blocks the host except ``synchronize``. The caller keeps
each submitted host tensor unchanged (inputs) and unread (output) until ``synchronize`` returns.
"""
from __future__ import annotations

from typing import Callable, Sequence

import torch


class HostPipeline:
    def __init__(self, fn: Callable, input_likes: Sequence[torch.Tensor], out_like: torch.Tensor, depth: int = 2):
        """``fn(*device_inputs, device_out)`` runs one call on the current stream; the ``*_like``
        tensors give the device buffers' shapes, dtypes and device."""
        if depth < 1:
            raise ValueError("depth must be >= 1")
        dev = out_like.device
        if dev.type != "cuda":
            raise ValueError("HostPipeline needs CUDA tensors")
        self.fn = fn
        self.depth = depth
        self.dev = dev
        self.compute = torch.cuda.current_stream(dev)
        self.up = torch.cuda.Stream(dev)
        self.down = torch.cuda.Stream(dev)
        self.ins = [[torch.empty_like(t, device=dev) for t in input_likes] for _ in range(depth)]
        self.outs = [torch.empty_like(out_like, device=dev) for _ in range(depth)]
        self.consumed = [None] * depth   # compute of the slot's last call finished (inputs free)
        self.downloaded = [None] * depth  # the slot's last result left the device
        self.i = 0
        # the buffers live as long as the pipeline; on release the caching allocator must wait
        # for the copy streams' last use of them
        for slot in range(depth):
            for t in self.ins[slot]:
                t.record_stream(self.up)
            self.outs[slot].record_stream(self.down)

    def submit(self, host_inputs: Sequence[torch.Tensor], host_out: torch.Tensor) -> None:
        s = self.i % self.depth
        self.i += 1
        d_in, d_out = self.ins[s], self.outs[s]
        if self.consumed[s] is not None:
            self.up.wait_event(self.consumed[s])
        with torch.cuda.stream(self.up):
            for d, h in zip(d_in, host_inputs):
                d.copy_(h, non_blocking=True)
            up_ev = torch.cuda.Event()
            up_ev.record(self.up)
        self.compute.wait_event(up_ev)
        if self.downloaded[s] is not None:
            self.compute.wait_event(self.downloaded[s])
        with torch.cuda.stream(self.compute):
            self.fn(*d_in, d_out)
            done = torch.cuda.Event()
            done.record(self.compute)
        self.consumed[s] = done
        self.down.wait_event(done)
        with torch.cuda.stream(self.down):
            host_out.copy_(d_out, non_blocking=True)
            dn = torch.cuda.Event()
            dn.record(self.down)
        self.downloaded[s] = dn

    def join(self, stream: torch.cuda.Stream) -> None:
        """Make `stream` wait for every submitted call's download (device-side, no host block)."""
        for ev in self.downloaded:
            if ev is not None:
                stream.wait_event(ev)

    def synchronize(self) -> None:
        self.join(self.compute)
        self.compute.synchronize()
