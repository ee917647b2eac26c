"""GPU: packed weights (moe_pack_weights / moe_fused_packed).

Packing is checked bit for bit: the 16-bit kinds against gate/up rows stacked with torch, the
8-bit kinds against the library's own per-row quantisers applied to the stacked weights (both
quantisers are checked bit-exact against the oracle's in their own tests). The fused call on
packed weights is checked against the CPU oracle: fp16/bf16 against ``fused_moe_ref`` with
|a - b| <= 1e-2 + 1e-2 |b|; the 8-bit kinds against the exact quantised model
(``fused_moe_int8_ref`` / ``fused_moe_fp8_ref``) at relative L2 < 1e-2, the bound of the int8 and
fp8 route tests. It also matches the unpacked entry point on the same weights.
"""
import pytest
import torch

from muxi_race_b200 import (device_status, fused_moe, fused_moe_fp8, fused_moe_int8, quantize_rows_fp8,
                            quantize_rows_int8)
from muxi_race_b200.packed import fused_moe_packed, pack_weights, packed_layout
from oracle.moe_ref import fused_moe_fp8_ref, fused_moe_int8_ref, fused_moe_ref

pytestmark = pytest.mark.gpu


def weights(E, H, I, dtype, dev, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    gate = (torch.randn((E, I, H), generator=g) * H ** -0.5).to(dtype).to(dev)
    up = (torch.randn((E, I, H), generator=g) * H ** -0.5).to(dtype).to(dev)
    down = (torch.randn((E, H, I), generator=g) * I ** -0.5).to(dtype).to(dev)
    return gate, up, down


def routing(T, E, k, dev, seed=1):
    g = torch.Generator(device="cpu").manual_seed(seed)
    vals, ids = torch.topk(torch.softmax(torch.randn((T, E), generator=g), -1), k, dim=-1)
    return ids.to(torch.int32).to(dev), (vals / vals.sum(-1, keepdim=True)).to(dev)


@pytest.mark.parametrize("kind", ["fp16", "bf16", "int8", "fp8"])
def test_pack_and_run(cuda_device, kind):
    E, H, I, T, k = 8, 512, 256, 300, 2
    dtype = torch.bfloat16 if kind == "bf16" else torch.float16
    gate, up, down = weights(E, H, I, dtype, cuda_device)
    w13 = torch.cat([gate, up], dim=1).contiguous()
    p = pack_weights(gate, up, down, kind)
    off, total = packed_layout(E, H, I, kind)
    torch.cuda.synchronize()
    assert device_status() == 0 and p.blob.numel() == total
    b = p.blob
    x = torch.randn((T, H), generator=torch.Generator(device="cpu").manual_seed(2)).to(dtype).to(cuda_device)
    ids, w = routing(T, E, k, cuda_device)
    if kind in ("fp16", "bf16"):
        assert torch.equal(b[off[0]:off[0] + w13.numel() * 2].view(dtype).view_as(w13), w13)
        assert torch.equal(b[off[2]:off[2] + down.numel() * 2].view(dtype).view_as(down), down)
        out = fused_moe_packed(x, p, ids, w)
        torch.cuda.synchronize()
        assert device_status() == 0
        oracle = fused_moe_ref(x.cpu(), w13.cpu(), down.cpu(), ids.cpu(), w.cpu())
        err = (out.float().cpu() - oracle).abs()
        assert bool((err <= 1e-2 + 1e-2 * oracle.abs()).all()), f"max err {float(err.max()):.3e}"
        ref = fused_moe(x, w13, down, ids, w)
        err = (out.float() - ref.float()).abs()
        assert bool((err <= 1e-2 + 1e-2 * ref.float().abs()).all())
        return
    quant = quantize_rows_fp8 if kind == "fp8" else quantize_rows_int8
    q13, s13 = quant(w13)
    q2, s2 = quant(down)
    assert torch.equal(b[off[0]:off[0] + q13.numel()], q13.view(torch.uint8).reshape(-1))
    assert torch.equal(b[off[1]:off[1] + s13.numel() * 4].view(torch.float32), s13.reshape(-1))
    assert torch.equal(b[off[2]:off[2] + q2.numel()], q2.view(torch.uint8).reshape(-1))
    assert torch.equal(b[off[3]:off[3] + s2.numel() * 4].view(torch.float32), s2.reshape(-1))
    out = fused_moe_packed(x, p, ids, w)
    torch.cuda.synchronize()
    assert device_status() == 0
    exact_ref = fused_moe_fp8_ref if kind == "fp8" else fused_moe_int8_ref
    exact = exact_ref(x.cpu(), q13.cpu(), s13.cpu(), q2.cpu(), s2.cpu(), ids.cpu(), w.cpu(), out_dtype=dtype)
    rel = ((out.float().cpu() - exact).norm() / exact.norm()).item()
    assert rel < 1e-2, f"vs the exact quantised model: {rel}"
    fused_q = fused_moe_fp8 if kind == "fp8" else fused_moe_int8
    ref = fused_q(x, q13, s13, q2, s2, ids, w)
    rel = ((out.float() - ref.float()).norm() / ref.float().norm()).item()
    assert rel < 1e-2, rel
