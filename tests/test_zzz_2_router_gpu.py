"""GPU: softmax top-k routing (moe_router_topk / fused_topk) and the fused MoE with device-side
routing (moe_fused_router / fused_moe_router) against the router oracle.

Ids bit-exact (the kernel and the oracle use the same total order: fp32 value, then ascending
expert id). Weights within rtol 1e-5 / atol 1e-6 of torch's fp32 softmax (the kernel computes
exp(l - max) over the selected logits with CUDA's expf). The fused output within the fused
tests' |out - ref| <= 1e-2 + 1e-2 * |ref| of the fp32 reference.
"""
import pytest
import torch

import cases
from muxi_race_b200 import device_status, fused_moe, fused_moe_router, fused_topk
from oracle.moe_ref import fused_moe_ref
from oracle.router_ref import router_topk_ref

pytestmark = pytest.mark.gpu
W_RTOL, W_ATOL = 1e-5, 1e-6


def check_routing(logits, k, renormalize, what):
    w, ids = fused_topk(logits, logits, k, renormalize)
    torch.cuda.synchronize()
    assert device_status() == 0
    w_ref, ids_ref = router_topk_ref(logits.cpu(), k, renormalize)
    assert ids.dtype == torch.int32 and w.dtype == torch.float32
    mism = (ids.cpu() != ids_ref).nonzero()
    assert mism.numel() == 0, f"{what}: {mism.shape[0]} id mismatches, first at {mism[0].tolist()}"
    torch.testing.assert_close(w.cpu(), w_ref, rtol=W_RTOL, atol=W_ATOL, msg=lambda m: f"{what}: {m}")


@pytest.mark.parametrize("T,E,k", [(1000, 8, 2), (513, 60, 4), (4096, 256, 8), (300, 1024, 32), (70, 32, 32),
                                   (129, 33, 1), (64, 5, 3)])
@pytest.mark.parametrize("renormalize", [True, False])
def test_router_fp32(cuda_device, T, E, k, renormalize):
    g = torch.Generator(device="cpu").manual_seed(T + 31 * E + k)
    logits = torch.randn((T, E), generator=g).to(cuda_device)
    check_routing(logits, k, renormalize, f"fp32 T={T} E={E} k={k} renorm={renormalize}")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_router_low_precision_logits(cuda_device, dtype):
    """fp16 / bf16 logits hold many equal values per token: the order of ties is part of the check."""
    g = torch.Generator(device="cpu").manual_seed(11)
    logits = torch.randn((2048, 256), generator=g).to(dtype).to(cuda_device)
    check_routing(logits, 8, True, f"{dtype}")


def test_router_ties_and_signed_zeros(cuda_device):
    g = torch.Generator(device="cpu").manual_seed(12)
    logits = torch.randint(-2, 3, (500, 64), generator=g).float()  # five distinct values
    logits[::7] = 0.0
    logits[::7, 1::2] = -0.0
    check_routing(logits.to(cuda_device), 8, True, "ties")
    check_routing(logits.to(cuda_device), 8, False, "ties, no renormalisation")


def test_router_empty(cuda_device):
    logits = torch.zeros((0, 16), device=cuda_device)
    w, ids = fused_topk(logits, logits, 4)
    assert w.shape == (0, 4) and ids.shape == (0, 4)


@pytest.mark.parametrize("name", sorted(cases.FUSED_CASES))
def test_fused_moe_router(cuda_device, name):
    c = cases.FUSED_CASES[name]
    x, w13, w2, _, _ = (t.to(cuda_device) for t in cases.fused_inputs(name))
    g = torch.Generator(device="cpu").manual_seed(2000 + c["seed"])
    logits = torch.randn((c["T"], c["experts"]), generator=g).to(cuda_device)
    out, w, ids = fused_moe_router(x, w13, w2, logits, c["topk"], return_routing=True)
    torch.cuda.synchronize()
    assert device_status() == 0
    w_ref, ids_ref = router_topk_ref(logits.cpu(), c["topk"])
    assert torch.equal(ids.cpu(), ids_ref)
    torch.testing.assert_close(w.cpu(), w_ref, rtol=W_RTOL, atol=W_ATOL)
    ref = fused_moe_ref(x, w13, w2, ids_ref.to(cuda_device), w_ref.to(cuda_device))
    err = (out.float() - ref.float()).abs()
    assert bool((err <= 1e-2 + 1e-2 * ref.float().abs()).all()), f"{name}: max err {err.max().item():.3e}"
    # the same routing through fused_moe gives the same result up to the combine's summation order
    out2 = fused_moe(x, w13, w2, ids, w)
    torch.testing.assert_close(out, out2, rtol=1e-2, atol=1e-2)


def test_fused_moe_router_cfg3_routing(cuda_device):
    """cfg3's router shape (T=4096, E=256, top-8) through the fused path at a small hidden size:
    the returned routing is bit-exact and the output matches the fp32 reference."""
    T, E, k, H, I = 4096, 256, 8, 256, 128
    g = torch.Generator(device="cpu").manual_seed(21)
    logits = torch.randn((T, E), generator=g)
    x = torch.randn((T, H), generator=g).half()
    w13 = (torch.randn((E, 2 * I, H), generator=g) * H ** -0.5).half()
    w2 = (torch.randn((E, H, I), generator=g) * I ** -0.5).half()
    d = cuda_device
    out, w, ids = fused_moe_router(x.to(d), w13.to(d), w2.to(d), logits.to(d), k, return_routing=True)
    torch.cuda.synchronize()
    assert device_status() == 0
    w_ref, ids_ref = router_topk_ref(logits, k)
    assert torch.equal(ids.cpu(), ids_ref)
    ref = fused_moe_ref(x.to(d), w13.to(d), w2.to(d), ids_ref.to(d), w_ref.to(d))
    err = (out.float() - ref.float()).abs()
    assert bool((err <= 1e-2 + 1e-2 * ref.float().abs()).all()), f"max err {err.max().item():.3e}"
