"""GPU: every grouped-GEMM tile configuration, forced with ``set_tile``, against the oracle.

The per-call choice picks a configuration from the expected blocks per expert; this file runs
each configuration (single-CTA, two-block groups, k-block-spanning weight boxes and token-row
boxes (``ka``), BN = 128 (in Stage2 too: 128x2a4b6e8), CTA pairs) on shapes that exercise empty experts, one-, two- and three-block experts, partial column
tiles and both element types, for the fused, int8 and reference drop-in paths.
Tolerance: |out - ref_fp32| <= 1e-2 + 1e-2 * |ref| (int8: relative L2 <= 5e-2 vs the fp reference).
"""
import math

import pytest
import torch

from muxi_race_b200 import _lib, device_status, fused_moe, fused_moe_int8, quantize_rows_int8, run_kernel
from oracle.moe_ref import fused_moe_ref, run_kernel_ref_f32

pytestmark = pytest.mark.gpu

TILES = ["256a4b5", "256x2a3b4", "256a4b5e8", "256x2a3b4e8", "512a2b3", "256a2b2c2", "256a6b4", "256a6b2k2",
         "128x2a3b4k2", "128x2a3b8", "256x2a3b2k2", "p256a6b8", "p256a7b7", "p256a4b10", "128x2a4b6e8",
         "256a3b4e8ka2", "256a2b3e8ka4", "256a3b2e8k2ka2", "256a2b6e8", "256a3b5e8", "256x2a2b5e8",
         "256a5b4e8", "256a6b4e8", "256x2a4b3e8"]


@pytest.fixture
def tile(request):
    _lib.set_tile(0, request.param)
    yield request.param
    _lib.set_tile(0, None)


def assert_within(out, ref, what, rtol=1e-2, atol=1e-2):
    out = out.float().cpu()
    ref = ref.float().cpu()
    err = (out - ref).abs()
    bad = err > atol + rtol * ref.abs()
    n = int(bad.sum())
    if n:
        i = bad.nonzero()[0].tolist()
        raise AssertionError(f"{what}: {n}/{out.numel()} outside tolerance (max err {err.max():.3e}), "
                             f"first {i}: out={out[tuple(i)]} ref={ref[tuple(i)]}")


def skewed_routing(T, E, k, seed, dev, empty=(2,)):
    """top-k ids drawn from a skewed expert distribution (some experts get three blocks, some one,
    the `empty` ones none) and renormalised weights."""
    g = torch.Generator().manual_seed(seed)
    p = torch.tensor([1.0 / (1 + e) ** 0.8 for e in range(E)])
    for e in empty:
        p[e] = 0
    ids = torch.stack([torch.multinomial(p, k, replacement=False, generator=g) for _ in range(T)])
    w = torch.rand((T, k), generator=g) + 0.1
    w = w / w.sum(-1, keepdim=True)
    return ids.to(torch.int32).to(dev), w.to(dev)


def weights(E, H, I, dtype, seed, dev):
    g = torch.Generator().manual_seed(seed)
    w13 = (torch.randn((E, 2 * I, H), generator=g) / math.sqrt(H)).to(dtype).to(dev)
    w2 = (torch.randn((E, H, I), generator=g) / math.sqrt(I)).to(dtype).to(dev)
    return w13, w2


@pytest.mark.parametrize("tile", TILES, indirect=True)
@pytest.mark.parametrize("dtype,H,I", [(torch.float16, 1024, 512), (torch.bfloat16, 768, 384)])
def test_fused_tile(cuda_device, tile, dtype, H, I):
    E, T, k = 8, 600, 3
    w13, w2 = weights(E, H, I, dtype, 11, cuda_device)
    x = torch.randn((T, H), generator=torch.Generator().manual_seed(12)).to(dtype).to(cuda_device)
    ids, w = skewed_routing(T, E, k, 13, cuda_device)
    out = fused_moe(x, w13, w2, ids, w)
    torch.cuda.synchronize()
    assert device_status() == 0
    assert_within(out, fused_moe_ref(x, w13, w2, ids, w), what=f"{tile} {dtype}")


@pytest.mark.parametrize("tile", TILES, indirect=True)
def test_fused_int8_tile(cuda_device, tile):
    E, H, I, T, k = 8, 512, 256, 700, 2
    w13, w2 = weights(E, H, I, torch.float16, 21, cuda_device)
    x = torch.randn((T, H), generator=torch.Generator().manual_seed(22)).half().to(cuda_device)
    ids, w = skewed_routing(T, E, k, 23, cuda_device)
    w13q, w13s = quantize_rows_int8(w13)
    w2q, w2s = quantize_rows_int8(w2)
    out = fused_moe_int8(x, w13q, w13s, w2q, w2s, ids, w)
    torch.cuda.synchronize()
    assert device_status() == 0
    ref = fused_moe_ref(x, w13, w2, ids, w)
    rel = ((out.float() - ref).norm() / ref.norm()).item()
    assert rel <= 5e-2, (tile, rel)


@pytest.mark.parametrize("tile", TILES, indirect=True)
def test_run_kernel_tile(cuda_device, tile):
    """The reference drop-in with separate gate/up tensors: empty, one-, two- and three-block experts."""
    E, H, I = 6, 512, 384
    gs = torch.tensor([300, 0, 129, 40, 256, 128], dtype=torch.int32)
    go = torch.cat([torch.zeros(1, dtype=torch.int32), torch.cumsum(gs, 0, dtype=torch.int32)])
    padded = (gs + 127) // 128 * 128
    gpo = torch.cat([torch.zeros(1, dtype=torch.int32), torch.cumsum(padded, 0, dtype=torch.int32)])
    gidx = torch.repeat_interleave(torch.arange(E, dtype=torch.int32), padded // 128)
    P, R = int(gpo[-1]), int(go[-1])
    g = torch.Generator().manual_seed(31)
    x = torch.randn((P, H), generator=g).half()
    gate = (torch.randn((E, I, H), generator=g) / math.sqrt(H)).half()
    up = (torch.randn((E, I, H), generator=g) / math.sqrt(H)).half()
    down = (torch.randn((E, H, I), generator=g) / math.sqrt(I)).half()
    routed = torch.rand((R,), generator=g)
    ref = run_kernel_ref_f32(x, gate, up, down, routed, gs, go, gpo, gidx)
    d = [t.to(cuda_device) for t in (x, gate, up, down, routed, gs, go, gpo, gidx)]
    out = torch.full((P, H), float("nan"), dtype=torch.float16, device=cuda_device)
    run_kernel(*d, out)
    torch.cuda.synchronize()
    assert device_status() == 0
    assert_within(out, ref, what=tile)


def test_set_tile_rejects_unknown_names():
    with pytest.raises(_lib.MoeError):
        _lib.set_tile(1, "no-such-tile")
    with pytest.raises(_lib.MoeError):
        _lib.set_tile(3, "256a4b5")
    _lib.set_tile(0, "auto")
