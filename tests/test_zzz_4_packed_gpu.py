"""GPU: packed weights (moe_pack_weights / moe_fused_packed).

Packing is checked bit for bit: the 16-bit kinds against gate/up rows stacked with torch, the
8-bit kinds against the library's own per-row quantisers applied to the stacked weights. The
fused call on packed weights is checked against the unpacked entry point with the same weights
(fp16/bf16: |a - b| <= 1e-2 + 1e-2 |b|; 8-bit kinds: relative L2 < 1e-2, the run-to-run spread
of the atomic top-k combine).

The file name sorts after the other GPU test files, so a run that stops at the first failure has
run them all.
"""
import pytest
import torch

from muxi_race_b200 import (device_status, fused_moe, fused_moe_fp8, fused_moe_int8, quantize_rows_fp8,
                            quantize_rows_int8)
from muxi_race_b200.packed import fused_moe_packed, pack_weights, packed_layout

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
        ref = fused_moe(x, w13, down, ids, w)
        out = fused_moe_packed(x, p, ids, w)
        torch.cuda.synchronize()
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
    fused_q = fused_moe_fp8 if kind == "fp8" else fused_moe_int8
    ref = fused_q(x, q13, s13, q2, s2, ids, w)
    out = fused_moe_packed(x, p, ids, w)
    torch.cuda.synchronize()
    assert device_status() == 0
    rel = ((out.float() - ref.float()).norm() / ref.float().norm()).item()
    assert rel < 1e-2, rel
