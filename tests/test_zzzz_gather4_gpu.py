"""GPU: Stage1 with the TMA tile::gather4 A path (``set_a_path("gather")``: the token rows are
gathered inside the GEMM from ``hidden_states``, 32 four-row loads per 128-row block, no stacked
copy) against the CPU oracle.

Covered: fp16 and bf16 (``fused_moe_ref``, |out - ref| <= 1e-2 + 1e-2 |ref|), the int8 and fp8
routes (exact quantised models, relative L2 < 1e-2), every Stage1 configuration built for the
path (one- and two-block groups, 4 and 8 epilogue warps), experts with zero, one, two and three
blocks, token counts that are not multiples of 4, the ordered combine, and a call on the default
path afterwards in the same process (the workspace follows the selection).
"""
import math

import pytest
import torch

from muxi_race_b200 import (_lib, device_status, fused_moe, fused_moe_fp8, fused_moe_int8, quantize_rows_fp8,
                            quantize_rows_int8)
from oracle.moe_ref import fused_moe_fp8_ref, fused_moe_int8_ref, fused_moe_ref

pytestmark = pytest.mark.gpu


@pytest.fixture
def gather_path():
    _lib.set_a_path("gather")
    yield
    _lib.set_a_path(None)
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


@pytest.mark.parametrize("tile", ["256a4b5e8", "256a4b5", "256x2a3b4e8", "256x2a3b4"])
@pytest.mark.parametrize("dtype,H,I,T", [(torch.float16, 1024, 512, 601), (torch.bfloat16, 768, 384, 333)])
def test_gather4_fused(cuda_device, gather_path, tile, dtype, H, I, T):
    _lib.set_tile(1, tile)
    E, k = 8, 3
    w13, w2 = weights(E, H, I, dtype, 11, cuda_device)
    x = torch.randn((T, H), generator=torch.Generator().manual_seed(12)).to(dtype).to(cuda_device)
    ids, w = skewed_routing(T, E, k, 13, cuda_device)
    out = torch.full((T, H), float("nan"), dtype=dtype, device=cuda_device)
    fused_moe(x, w13, w2, ids, w, out=out)
    torch.cuda.synchronize()
    assert device_status() == 0
    assert_within(out, fused_moe_ref(x.cpu(), w13.cpu(), w2.cpu(), ids.cpu(), w.cpu()), f"gather4 {tile}")


def test_gather4_ordered_then_default_path(cuda_device, gather_path):
    E, H, I, T, k = 8, 512, 256, 77, 2
    w13, w2 = weights(E, H, I, torch.float16, 5, cuda_device)
    x = torch.randn((T, H), generator=torch.Generator().manual_seed(6)).half().to(cuda_device)
    ids, w = skewed_routing(T, E, k, 7, cuda_device)
    ref = fused_moe_ref(x.cpu(), w13.cpu(), w2.cpu(), ids.cpu(), w.cpu())
    assert_within(fused_moe(x, w13, w2, ids, w, deterministic=True), ref, "gather4 ordered")
    _lib.set_a_path(None)
    assert_within(fused_moe(x, w13, w2, ids, w), ref, "default path after gather4")
    torch.cuda.synchronize()
    assert device_status() == 0


@pytest.mark.parametrize("kind", ["int8", "fp8"])
def test_gather4_8bit(cuda_device, gather_path, kind):
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
    assert rel < 1e-2, (kind, rel)
