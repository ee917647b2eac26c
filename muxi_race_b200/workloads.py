"""Seeded synthetic inputs with the shapes and distributions of the benchmark configurations.

No dataset or checkpoint is involved: weights ~ N(0, (1/sqrt(fan_in))^2) (fan_in = H for gate/up,
I for down), hidden_states ~ N(0, 1), router logits ~ N(0, 1) -> softmax -> top-k -> weights
renormalised to sum to 1. The skewed expert-parallel configuration adds a Zipf(s) bias to the
logits in log form: expert with popularity rank r (a seeded permutation of the experts) gets
bias log(r^-s / H_{E,s}), which makes the top experts "hot" (they appear in most tokens' top-k).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch


@dataclass(frozen=True)
class MoeConfig:
    name: str
    T: int
    H: int
    I: int
    E: int
    topk: int
    dtype: torch.dtype
    int8: bool = False
    zipf_s: float = 0.0
    note: str = field(default="", compare=False)

    def flops(self, routes: int | None = None) -> float:
        """Algorithmic FLOPs: 2 * routed rows * 3 * H * I (padding rows excluded)."""
        r = self.T * self.topk if routes is None else routes
        return 2.0 * r * 3 * self.H * self.I

    def weight_bytes(self, active_experts: int | None = None) -> float:
        e = self.E if active_experts is None else active_experts
        return float(e) * 3 * self.H * self.I * (1 if self.int8 else 2)

    def io_bytes(self) -> float:
        return 2.0 * self.T * self.H * 2  # hidden_states in + out


CONFIGS = {
    "cfg1": MoeConfig("cfg1", 64, 1024, 512, 8, 2, torch.float16, note="small, CPU-runnable"),
    "cfg2": MoeConfig("cfg2", 1024, 4096, 14336, 8, 2, torch.bfloat16, note="Mixtral-style"),
    "cfg3": MoeConfig("cfg3", 4096, 7168, 2048, 256, 8, torch.float16, note="DeepSeek-V3-style, 1 GPU"),
    "cfg3_t128": MoeConfig("cfg3_t128", 128, 7168, 2048, 256, 8, torch.float16, note="decode-like"),
    "cfg4": MoeConfig("cfg4", 4096, 7168, 2048, 256, 8, torch.float16, int8=True, note="W8A8 of cfg3"),
    "cfg5": MoeConfig("cfg5", 32768, 7168, 2048, 256, 8, torch.float16, zipf_s=1.1, note="EP, Zipf-skewed"),
    # profiling case: cfg3's per-expert shape (about 128 rows per expert) with 32 experts, so a full
    # ncu capture holds ~3 GB on the device instead of 24 GB
    "cfg3_e32": MoeConfig("cfg3_e32", 512, 7168, 2048, 32, 8, torch.float16, note="cfg3 shape, 32 experts"),
    "cfg4_e32": MoeConfig("cfg4_e32", 512, 7168, 2048, 32, 8, torch.float16, int8=True, note="cfg4 shape, 32 experts"),
    # profiling case of the weight-streaming regime: cfg3_t128's ~4 rows per expert with 32 experts
    # (2.8 GB of weights, still far above L2)
    "cfg3_t128_e32": MoeConfig("cfg3_t128_e32", 16, 7168, 2048, 32, 8, torch.float16,
                               note="cfg3_t128 shape, 32 experts"),
}


def _gen(device, seed: int) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def make_weights(cfg: MoeConfig, seed: int = 0, device="cuda", experts=None):
    """w_gate_up [n, 2I, H] (gate rows then up rows) and w_down [n, H, I] in cfg.dtype.

    ``experts``: the global expert ids to build (default all E). Every expert has its own seed, so
    a rank of an expert-parallel group builds exactly its slice of the global weights.
    """
    ids = list(range(cfg.E)) if experts is None else list(experts)
    w13 = torch.empty((len(ids), 2 * cfg.I, cfg.H), dtype=cfg.dtype, device=device)
    w2 = torch.empty((len(ids), cfg.H, cfg.I), dtype=cfg.dtype, device=device)
    for i, e in enumerate(ids):  # one expert at a time in fp32 to bound the temporary
        g = _gen(device, seed * 1_000_003 + e)
        w13[i].copy_(torch.randn((2 * cfg.I, cfg.H), generator=g, device=device) * (cfg.H ** -0.5))
        w2[i].copy_(torch.randn((cfg.H, cfg.I), generator=g, device=device) * (cfg.I ** -0.5))
    return w13, w2


def make_hidden(cfg: MoeConfig, seed: int = 1, device="cuda", T: int | None = None) -> torch.Tensor:
    T = cfg.T if T is None else T
    return torch.randn((T, cfg.H), generator=_gen(device, seed), device=device).to(cfg.dtype)


ZIPF_SEED = 1000  # the expert popularity order is a property of the model, shared by every rank


def zipf_bias(E: int, s: float, seed: int = ZIPF_SEED, device="cpu") -> torch.Tensor:
    ranks = torch.randperm(E, generator=_gen("cpu", seed)).to(torch.float64) + 1.0
    pmf = ranks.pow(-s)
    pmf = pmf / pmf.sum()
    return pmf.log().to(torch.float32).to(device)


def make_router_logits(cfg: MoeConfig, seed: int = 2, device="cuda", T: int | None = None) -> torch.Tensor:
    """Router logits [T, E] fp32: N(0,1), plus the log-Zipf popularity bias when cfg.zipf_s > 0."""
    T = cfg.T if T is None else T
    logits = torch.randn((T, cfg.E), generator=_gen(device, seed), device=device)
    if cfg.zipf_s > 0:
        logits = logits + zipf_bias(cfg.E, cfg.zipf_s, device=device)
    return logits


def make_routing(cfg: MoeConfig, seed: int = 2, device="cuda", T: int | None = None, id_dtype=torch.int32):
    """topk_ids [T, k] (id_dtype) and topk_weights [T, k] fp32 from softmax-top-k of the logits of
    make_router_logits (same seed: same routing)."""
    logits = make_router_logits(cfg, seed, device, T)
    probs = torch.softmax(logits, dim=-1)
    vals, ids = torch.topk(probs, cfg.topk, dim=-1)
    weights = vals / vals.sum(dim=-1, keepdim=True)
    return ids.to(id_dtype).contiguous(), weights.to(torch.float32).contiguous()
