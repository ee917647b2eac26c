"""GPU: the fused MoE with the ordered (deterministic) top-k combine, moe_fused_ordered /
``fused_moe(..., deterministic=True)``.

Tolerance as the other fused tests: |out - ref_fp32| <= 1e-2 + 1e-2 * |ref|. Determinism:
repeated calls on the same inputs give identical bits.
"""
import os

import numpy as np
import pytest
import torch

import cases
from muxi_race_b200 import device_status, fused_moe
from oracle.moe_ref import fused_moe_ref

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
RTOL = ATOL = 1e-2


def within(out, ref, what):
    out, ref = out.float().cpu(), ref.float().cpu()
    err = (out - ref).abs()
    bad = err > ATOL + RTOL * ref.abs()
    assert int(bad.sum()) == 0, f"{what}: {int(bad.sum())}/{out.numel()} outside tolerance, max err {err.max():.3e}"


@pytest.mark.parametrize("name", sorted(cases.FUSED_CASES))
def test_ordered_matches_golden(cuda_device, name):
    x, w13, w2, ids, w = (t.to(cuda_device) for t in cases.fused_inputs(name))
    g = np.load(os.path.join(GOLDEN, f"fused_{name}.npz"))
    out = fused_moe(x, w13, w2, ids, w, deterministic=True)
    torch.cuda.synchronize()
    assert device_status() == 0
    within(out, torch.from_numpy(g["out_f32"]), name)


def make(T, E, k, H, I, dtype, seed, dev):
    g = torch.Generator(device="cpu").manual_seed(seed)
    logits = torch.randn((T, E), generator=g)
    vals, ids = torch.topk(torch.softmax(logits, -1), k, dim=-1)
    w = vals / vals.sum(-1, keepdim=True)
    x = torch.randn((T, H), generator=g).to(dtype)
    w13 = (torch.randn((E, 2 * I, H), generator=g) * H ** -0.5).to(dtype)
    w2 = (torch.randn((E, H, I), generator=g) * I ** -0.5).to(dtype)
    return [t.to(dev) for t in (x, w13, w2, ids.to(torch.int32), w)]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_ordered_is_bitwise_repeatable(cuda_device, dtype):
    x, w13, w2, ids, w = make(2048, 64, 8, 1024, 512, dtype, 7, cuda_device)
    first = fused_moe(x, w13, w2, ids, w, deterministic=True)
    for _ in range(3):
        again = fused_moe(x, w13, w2, ids, w, deterministic=True)
        assert torch.equal(again, first)
    torch.cuda.synchronize()
    assert device_status() == 0
    within(first, fused_moe_ref(x, w13, w2, ids, w), f"{dtype}")
    within(first, fused_moe(x, w13, w2, ids, w), f"{dtype} vs the atomic combine")


def test_ordered_skips_routes_outside_the_experts(cuda_device):
    """Ids outside [0, E) (as expert-parallel ranks pass for remote experts) contribute nothing."""
    x, w13, w2, ids, w = make(300, 16, 4, 256, 128, torch.float16, 8, cuda_device)
    ids[::3, 1] = -1
    ids[1::5, 0] = 16
    out = fused_moe(x, w13, w2, ids, w, deterministic=True)
    keep = (ids >= 0) & (ids < 16)
    ref = fused_moe_ref(x, w13, w2, torch.where(keep, ids, 0), torch.where(keep, w, 0.0))
    torch.cuda.synchronize()
    within(out, ref, "skipped routes")
