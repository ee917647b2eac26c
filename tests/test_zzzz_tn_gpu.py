"""GPU: the operand-swapped grouped GEMM (tile "tn": expert weight rows as the MMA's M side, an
expert's tokens as its N side, padded to 16 rows instead of 128) against the CPU oracle.

The configuration is forced per stage with ``set_tile`` on the fused path (fp16, bf16, int8,
fp8), on shapes with empty experts, experts with 1..15 rows (a 16-column MMA), experts with more
than 256 rows (several token chunks), a Stage1 feature tile that is cut by I (I = 200: 3 tiles of
64 and one of 8) and a Stage2 output tile cut by H (H = 576: 4 tiles of 128 and one of 64).
Tolerance: fp16/bf16 |out - ref_fp32| <= 1e-2 + 1e-2 * |ref| against ``fused_moe_ref``; the
8-bit kinds relative L2 < 1e-2 against the exact quantised model (``fused_moe_int8_ref`` /
``fused_moe_fp8_ref``), the bound of the int8 and fp8 route tests.
"""
import math

import pytest
import torch

from muxi_race_b200 import (_lib, device_status, fused_moe, fused_moe_fp8, fused_moe_int8, quantize_rows_fp8,
                            quantize_rows_int8)
from oracle.moe_ref import fused_moe_fp8_ref, fused_moe_int8_ref, fused_moe_ref

pytestmark = pytest.mark.gpu


@pytest.fixture
def stage(request):
    _lib.set_tile(request.param, "tn")
    yield request.param
    _lib.set_tile(0, None)


def skewed_routing(T, E, k, seed, dev, empty=(2,)):
    g = torch.Generator().manual_seed(seed)
    p = torch.tensor([1.0 / (1 + e) ** 0.8 for e in range(E)])
    for e in empty:
        p[e] = 0
    ids = torch.stack([torch.multinomial(p, k, replacement=False, generator=g) for _ in range(T)])
    w = torch.rand((T, k), generator=g) + 0.1
    return ids.to(torch.int32).to(dev), (w / w.sum(-1, keepdim=True)).to(dev)


def weights(E, H, I, dtype, seed, dev):
    g = torch.Generator().manual_seed(seed)
    w13 = (torch.randn((E, 2 * I, H), generator=g) / math.sqrt(H)).to(dtype).to(dev)
    w2 = (torch.randn((E, H, I), generator=g) / math.sqrt(I)).to(dtype).to(dev)
    return w13, w2


def assert_within(out, ref, what):
    out, ref = out.float().cpu(), ref.float().cpu()
    err = (out - ref).abs()
    bad = err > 1e-2 + 1e-2 * ref.abs()
    assert int(bad.sum()) == 0, f"{what}: {int(bad.sum())}/{out.numel()} outside tolerance (max err {err.max():.3e})"


SHAPES = [  # dtype, H, I, T, E, k
    (torch.float16, 1024, 512, 600, 8, 3),
    (torch.bfloat16, 768, 384, 600, 8, 3),
    (torch.float16, 512, 200, 300, 8, 2),
    (torch.bfloat16, 576, 320, 300, 8, 2),
    (torch.float16, 512, 256, 9, 8, 2),
]
SHAPE_IDS = ["f16_h1024", "bf16_h768", "f16_i200", "bf16_h576", "f16_t9"]


@pytest.mark.parametrize("stage", [1, 2, 0], indirect=True, ids=["stage1", "stage2", "both"])
@pytest.mark.parametrize("dtype,H,I,T,E,k", SHAPES, ids=SHAPE_IDS)
def test_tn_fused(cuda_device, stage, dtype, H, I, T, E, k):
    w13, w2 = weights(E, H, I, dtype, 11, cuda_device)
    x = torch.randn((T, H), generator=torch.Generator().manual_seed(12)).to(dtype).to(cuda_device)
    ids, w = skewed_routing(T, E, k, 13, cuda_device)
    out = torch.full((T, H), float("nan"), dtype=dtype, device=cuda_device)
    fused_moe(x, w13, w2, ids, w, out=out)
    torch.cuda.synchronize()
    assert device_status() == 0
    assert_within(out, fused_moe_ref(x.cpu(), w13.cpu(), w2.cpu(), ids.cpu(), w.cpu()), f"tn stage {stage}")


@pytest.mark.parametrize("stage", [1, 2, 0], indirect=True, ids=["stage1", "stage2", "both"])
@pytest.mark.parametrize("kind", ["int8", "fp8"])
def test_tn_8bit(cuda_device, stage, kind):
    E, H, I, T, k = 8, 512, 256, 700, 2
    w13, w2 = weights(E, H, I, torch.float16, 21, cuda_device)
    x = torch.randn((T, H), generator=torch.Generator().manual_seed(22)).half().to(cuda_device)
    ids, w = skewed_routing(T, E, k, 23, cuda_device)
    quant, fused_q, exact_ref = ((quantize_rows_fp8, fused_moe_fp8, fused_moe_fp8_ref) if kind == "fp8" else
                                 (quantize_rows_int8, fused_moe_int8, fused_moe_int8_ref))
    w13q, w13s = quant(w13)
    w2q, w2s = quant(w2)
    out = fused_q(x, w13q, w13s, w2q, w2s, ids, w)
    torch.cuda.synchronize()
    assert device_status() == 0
    exact = exact_ref(x.cpu(), w13q.cpu(), w13s.cpu(), w2q.cpu(), w2s.cpu(), ids.cpu(), w.cpu(),
                      out_dtype=torch.float16)
    rel = ((out.float().cpu() - exact).norm() / exact.norm()).item()
    assert rel < 1e-2, (kind, stage, rel)
