"""Seeded inputs of the golden fixtures (CPU torch generators, reproducible on any host).

The fixtures in this directory hold the REFERENCE's outputs for these inputs (made by
``make_golden.py`` from the reference's own PyTorch code); the inputs themselves are regenerated
here and checked against the SHA-256 stored with each fixture.

Input recipes follow the reference harness:
* ``rb_*`` cases: ``make_group_sizes`` / ``make_inputs`` of 初审材料/源代码/benchmark/remote_bench.py:60-155
  (interleaved large/small experts; x ~ N(0,1); gate/up * 1/sqrt(I); down * 1/sqrt(H); fp32 routed
  weights ~ U[0,1)), at reduced hidden/intermediate sizes;
* ``rs_*`` cases: ``random_group_sizes`` / ``build_custom_inputs`` of race_stress2.py:15-80 (random
  per-expert sizes including empty experts; weights * 0.02; fp16 routed weights);
* ``fused_*`` cases: token-major inputs (softmax-top-k routing of N(0,1) logits).
"""
from __future__ import annotations

import hashlib
import math

import torch

BLOCK_M = 128

RUN_KERNEL_CASES = {
    # remote_bench CASES[0] verbatim: one expert, one partial block (127 valid rows)
    "rb_case0": dict(kind="rb", experts=1, hidden=128, intermediate=128, valid=127, high_experts=0, low_size=127,
                     seed=0),
    # remote_bench recipe, several experts, one of them spanning two blocks
    "rb_multi": dict(kind="rb", experts=4, hidden=128, intermediate=256, valid=400, high_experts=1, low_size=60,
                     seed=1),
    # race_stress2 recipe: random splits with empty experts, fp16 routed weights
    "rs_split": dict(kind="rs", experts=5, hidden=128, intermediate=192, valid=420, cap=200, seed=2),
    # K and N tails in both stages (H % 64 != 0, I % 128 != 0)
    "rs_odd": dict(kind="rs", experts=3, hidden=136, intermediate=200, valid=150, cap=140, seed=3),
}

FUSED_CASES = {
    # BASELINE cfg1: T=64, H=1024, I=512, E=8, top-2, fp16
    "fused_cfg1": dict(T=64, hidden=1024, intermediate=512, experts=8, topk=2, seed=0),
    # small, odd sizes, top-3 of 6
    "fused_odd": dict(T=37, hidden=136, intermediate=200, experts=6, topk=3, seed=5),
}

ALIGN_CASES = {
    "align_cfg1": dict(T=64, experts=8, topk=2, seed=0, skew=0.0),
    "align_t300": dict(T=300, experts=16, topk=4, seed=1, skew=0.0),
    "align_t1000": dict(T=1000, experts=64, topk=6, seed=2, skew=0.0),
    "align_skew": dict(T=2048, experts=32, topk=8, seed=3, skew=1.1),
}


def make_group_sizes(cfg) -> torch.Tensor:
    """remote_bench.py:60-75 restated."""
    high = cfg["high_experts"]
    low = cfg["experts"] - high
    sizes = [cfg["low_size"]] * low
    remaining = cfg["valid"] - sum(sizes)
    if high:
        q, r = divmod(remaining, high)
        sizes.extend([q + (i < r) for i in range(high)])
    else:
        assert remaining == 0
    sizes = sizes[::2] + sizes[1::2]
    assert len(sizes) == cfg["experts"] and sum(sizes) == cfg["valid"]
    assert sum(x > BLOCK_M for x in sizes) == high
    return torch.tensor(sizes, dtype=torch.int32)


def random_group_sizes(experts: int, valid: int, cap: int, gen: torch.Generator) -> torch.Tensor:
    """race_stress2.py:15-26 restated (per-expert cap as a parameter)."""
    sizes = []
    remaining = valid
    for _ in range(experts - 1):
        hi = min(remaining, cap)
        v = int(torch.randint(0, hi + 1, (1,), generator=gen).item())
        sizes.append(v)
        remaining -= v
    sizes.append(remaining)
    return torch.tensor(sizes, dtype=torch.int32)


def metadata(group_sizes: torch.Tensor):
    """remote_bench.py:82-101 restated: offsets, padded offsets, block -> expert map."""
    go = torch.cat([torch.zeros(1, dtype=torch.int32), torch.cumsum(group_sizes, 0, dtype=torch.int32)])
    padded = torch.div(group_sizes + BLOCK_M - 1, BLOCK_M, rounding_mode="floor") * BLOCK_M
    gpo = torch.cat([torch.zeros(1, dtype=torch.int32), torch.cumsum(padded, 0, dtype=torch.int32)])
    gidx = torch.repeat_interleave(torch.arange(group_sizes.numel(), dtype=torch.int32), padded // BLOCK_M)
    return go, gpo, gidx


def run_kernel_inputs(name: str):
    """(x, gate, up, down, routed, gs, go, gpo, gidx) on CPU for a RUN_KERNEL_CASES entry."""
    c = RUN_KERNEL_CASES[name]
    gen = torch.Generator(device="cpu")
    gen.manual_seed(1000 + c["seed"])
    E, H, I = c["experts"], c["hidden"], c["intermediate"]
    if c["kind"] == "rb":
        gs = make_group_sizes(c)
    else:
        gs = random_group_sizes(E, c["valid"], c["cap"], gen)
    go, gpo, gidx = metadata(gs)
    P = int(gpo[-1])
    if c["kind"] == "rb":
        x = torch.randn((P, H), generator=gen, dtype=torch.float16)
        gate = torch.randn((E, I, H), generator=gen, dtype=torch.float16).mul_(1.0 / math.sqrt(I))
        up = torch.randn((E, I, H), generator=gen, dtype=torch.float16).mul_(1.0 / math.sqrt(I))
        down = torch.randn((E, H, I), generator=gen, dtype=torch.float16).mul_(1.0 / math.sqrt(H))
        routed = torch.rand((int(gs.sum()),), generator=gen, dtype=torch.float32)
    else:
        x = torch.randn((P, H), generator=gen, dtype=torch.float16)
        gate = torch.randn((E, I, H), generator=gen, dtype=torch.float16) * 0.02
        up = torch.randn((E, I, H), generator=gen, dtype=torch.float16) * 0.02
        down = torch.randn((E, H, I), generator=gen, dtype=torch.float16) * 0.02
        routed = torch.rand((int(gs.sum()),), generator=gen, dtype=torch.float16)
    return x, gate, up, down, routed, gs, go, gpo, gidx


def routing(T: int, experts: int, topk: int, seed: int, skew: float = 0.0):
    """Softmax-top-k of N(0,1) logits (+ log-Zipf bias when skew > 0); ids int64, weights fp32."""
    gen = torch.Generator(device="cpu")
    gen.manual_seed(2000 + seed)
    logits = torch.randn((T, experts), generator=gen)
    if skew > 0:
        ranks = torch.randperm(experts, generator=gen).to(torch.float64) + 1.0
        pmf = ranks.pow(-skew)
        logits = logits + (pmf / pmf.sum()).log().to(torch.float32)
    probs = torch.softmax(logits, dim=-1)
    vals, ids = torch.topk(probs, topk, dim=-1)
    return ids.contiguous(), (vals / vals.sum(-1, keepdim=True)).contiguous()


def fused_inputs(name: str):
    """(hidden_states, w_gate_up, w_down, topk_ids, topk_weights) on CPU for a FUSED_CASES entry."""
    c = FUSED_CASES[name]
    T, H, I, E, k = c["T"], c["hidden"], c["intermediate"], c["experts"], c["topk"]
    ids, w = routing(T, E, k, c["seed"])
    gen = torch.Generator(device="cpu")
    gen.manual_seed(3000 + c["seed"])
    x = torch.randn((T, H), generator=gen).to(torch.float16)
    w13 = (torch.randn((E, 2 * I, H), generator=gen) * H ** -0.5).to(torch.float16)
    w2 = (torch.randn((E, H, I), generator=gen) * I ** -0.5).to(torch.float16)
    return x, w13, w2, ids, w


def align_inputs(name: str) -> torch.Tensor:
    c = ALIGN_CASES[name]
    ids, _ = routing(c["T"], c["experts"], c["topk"], c["seed"], c["skew"])
    return ids


def digest(*tensors) -> str:
    h = hashlib.sha256()
    for t in tensors:
        t = t.contiguous()
        h.update(str(t.dtype).encode())
        h.update(str(tuple(t.shape)).encode())
        h.update(t.view(torch.uint8).numpy().tobytes() if t.numel() else b"")
    return h.hexdigest()
