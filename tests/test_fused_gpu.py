"""GPU: token-major fused MoE (align + Stage1 + Stage2 with the fused top-k combine).

Tolerance: |out - ref_fp32| <= 1e-2 + 1e-2 * |ref| for fp16/bf16 outputs.
"""
import os

import numpy as np
import pytest
import torch

import cases
from muxi_race_b200 import device_status, fused_moe
from muxi_race_b200.workloads import CONFIGS, make_hidden, make_routing, make_weights
from oracle.moe_ref import fused_moe_ref

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
RTOL = ATOL = 1e-2


def assert_within(out, ref, rtol=RTOL, atol=ATOL, what=""):
    out = out.float().cpu()
    ref = ref.float().cpu()
    err = (out - ref).abs()
    bad = err > atol + rtol * ref.abs()
    n = int(bad.sum())
    if n:
        i = bad.nonzero()[0].tolist()
        raise AssertionError(f"{what}: {n}/{out.numel()} outside tolerance (max err {err.max():.3e}), "
                             f"first {i}: out={out[tuple(i)]} ref={ref[tuple(i)]}")


@pytest.mark.parametrize("name", sorted(cases.FUSED_CASES))
def test_fused_matches_golden(cuda_device, name):
    x, w13, w2, ids, w = (t.to(cuda_device) for t in cases.fused_inputs(name))
    g = np.load(os.path.join(GOLDEN, f"fused_{name}.npz"))
    out = fused_moe(x, w13, w2, ids, w)
    torch.cuda.synchronize()
    assert device_status() == 0
    assert_within(out, torch.from_numpy(g["out_f32"]), what=name)


@pytest.mark.parametrize("id_dtype", [torch.int32, torch.int64])
@pytest.mark.parametrize("w_dtype", [torch.float32, torch.float16])
def test_fused_cfg1_dtypes(cuda_device, id_dtype, w_dtype):
    cfg = CONFIGS["cfg1"]
    w13, w2 = make_weights(cfg, seed=0, device=cuda_device)
    x = make_hidden(cfg, device=cuda_device)
    ids, w = make_routing(cfg, device=cuda_device, id_dtype=id_dtype)
    w = w.to(w_dtype)
    out = fused_moe(x, w13, w2, ids, w)
    ref = fused_moe_ref(x, w13, w2, ids, w)
    torch.cuda.synchronize()
    assert_within(out, ref, what=f"cfg1 ids={id_dtype} w={w_dtype}")


def test_fused_bf16_mixtral_shape(cuda_device):
    """cfg2 shape (H=4096, I=14336, E=8, top-2, bf16) at T=256."""
    cfg = CONFIGS["cfg2"]
    w13, w2 = make_weights(cfg, seed=0, device=cuda_device)
    x = make_hidden(cfg, device=cuda_device, T=256)
    ids, w = make_routing(cfg, device=cuda_device, T=256)
    out = fused_moe(x, w13, w2, ids, w)
    ref = fused_moe_ref(x, w13, w2, ids, w)
    torch.cuda.synchronize()
    assert out.dtype == torch.bfloat16
    assert_within(out, ref, what="cfg2 bf16")


@pytest.mark.parametrize("T", [4096, 128])
def test_fused_deepseek_shape_full(cuda_device, T):
    """cfg3 at full size (T=4096) and the decode-like T=128, against an fp32 torch reference on GPU."""
    cfg = CONFIGS["cfg3"]
    w13, w2 = make_weights(cfg, seed=0, device=cuda_device)
    x = make_hidden(cfg, device=cuda_device, T=T)
    ids, w = make_routing(cfg, device=cuda_device, T=T)
    out = fused_moe(x, w13, w2, ids, w)
    torch.cuda.synchronize()
    assert device_status() == 0
    ref = fused_moe_ref(x, w13, w2, ids, w)
    assert_within(out, ref, what=f"cfg3 T={T}")
    # size-independent property: repeated calls stay within the nondeterminism of the fp16
    # red.add combine (order of adds only), well inside the tolerance
    out2 = fused_moe(x, w13, w2, ids, w)
    torch.cuda.synchronize()
    assert_within(out2, out.float(), rtol=2e-3, atol=2e-3, what="repeat")


def test_fused_edge_cases(cuda_device):
    dev = cuda_device
    E, H, I = 4, 128, 128
    g = torch.Generator(device=dev).manual_seed(3)
    w13 = (torch.randn((E, 2 * I, H), generator=g, device=dev) * H ** -0.5).half()
    w2 = (torch.randn((E, H, I), generator=g, device=dev) * I ** -0.5).half()
    # T = 0
    out = fused_moe(torch.empty((0, H), dtype=torch.float16, device=dev), w13, w2,
                    torch.empty((0, 2), dtype=torch.int32, device=dev), torch.empty((0, 2), device=dev))
    assert out.shape == (0, H)
    # every token routed to the same expert (one expert spans many blocks), top-1
    x = torch.randn((300, H), generator=g, device=dev).half()
    ids = torch.full((300, 1), 2, dtype=torch.int32, device=dev)
    w = torch.ones((300, 1), device=dev)
    out = fused_moe(x, w13, w2, ids, w)
    torch.cuda.synchronize()
    assert_within(out, fused_moe_ref(x, w13, w2, ids, w), what="single hot expert")
    # a token that routes twice to the same expert gets both contributions
    ids = torch.tensor([[1, 1], [0, 3]], dtype=torch.int32, device=dev)
    w = torch.tensor([[0.25, 0.75], [0.5, 0.5]], device=dev)
    out = fused_moe(x[:2], w13, w2, ids, w)
    torch.cuda.synchronize()
    assert_within(out, fused_moe_ref(x[:2], w13, w2, ids, w), what="duplicate expert in top-k")
