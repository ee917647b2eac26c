"""GPU: M = 64 MMAs for an expert's last block when it holds at most 64 valid rows
(``MOE_B200_M64_TAIL=1``, read at each launch) against the CPU oracle.

The routing gives experts 0, 1..64, 65..127, 128, 129..192 and more rows, so one-block experts
with a half block, two-block groups whose second block is a half block, and full blocks all occur;
every single-CTA Stage1 / Stage2 configuration that groups one or two blocks is forced in turn.
Checked: fp16 / bf16 ``fused_moe`` against ``fused_moe_ref`` (|out - ref| <= 1e-2 + 1e-2 |ref|),
the int8 and fp8 routes against their exact quantised models (relative L2 < 1e-2), and the
reference drop-in ``run_kernel`` (its Stage1 uses the half blocks, its padded-store Stage2 keeps
M = 128 and writes zero pad rows) against ``run_kernel_ref_f32`` with its pad rows zero.
"""
import math
import os

import pytest
import torch

from muxi_race_b200 import (_lib, device_status, fused_moe, fused_moe_fp8, fused_moe_int8, quantize_rows_fp8,
                            quantize_rows_int8, run_kernel)
from oracle.moe_ref import fused_moe_fp8_ref, fused_moe_int8_ref, fused_moe_ref, run_kernel_ref_f32

pytestmark = pytest.mark.gpu

# rows per expert: empty, 1, 64 (half), 65, 127, 128, 129 (second block: 1 row), 192 (64), 193, 301
SIZES = [0, 1, 64, 65, 127, 128, 129, 192, 193, 301]


@pytest.fixture
def m64():
    old = os.environ.get("MOE_B200_M64_TAIL")
    os.environ["MOE_B200_M64_TAIL"] = "1"
    yield
    if old is None:
        os.environ.pop("MOE_B200_M64_TAIL", None)
    else:
        os.environ["MOE_B200_M64_TAIL"] = old
    _lib.set_tile(0, None)


def routing_with_sizes(sizes, k, seed, dev):
    """Top-k ids with exactly sizes[e] routes to expert e (k distinct experts per token)."""
    g = torch.Generator().manual_seed(seed)
    E = len(sizes)
    R = sum(sizes)
    assert R % k == 0
    T = R // k
    left = list(sizes)
    ids = torch.empty((T, k), dtype=torch.int64)
    for t in range(T):  # greedy: the k experts with the most routes left, random tie order
        order = sorted(range(E), key=lambda e: (-left[e], float(torch.rand(1, generator=g))))
        pick = order[:k]
        for e in pick:
            left[e] -= 1
        ids[t] = torch.tensor(pick)
    assert all(v == 0 for v in left)
    w = torch.rand((T, k), generator=g) + 0.1
    return ids.to(torch.int32).to(dev), (w / w.sum(-1, keepdim=True)).to(dev), T


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


@pytest.mark.parametrize("tile", ["256a4b5e8", "256x2a3b4e8", "256a4b5", "256x2a3b4"])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_m64_tail_fused(cuda_device, m64, tile, dtype):
    _lib.set_tile(0, tile)
    E, H, I, k = len(SIZES), 512, 256, 2
    ids, w, T = routing_with_sizes(SIZES, k, 3, cuda_device)
    w13, w2 = weights(E, H, I, dtype, 4, cuda_device)
    x = torch.randn((T, H), generator=torch.Generator().manual_seed(5)).to(dtype).to(cuda_device)
    out = torch.full((T, H), float("nan"), dtype=dtype, device=cuda_device)
    fused_moe(x, w13, w2, ids, w, out=out)
    torch.cuda.synchronize()
    assert device_status() == 0
    assert_within(out, fused_moe_ref(x.cpu(), w13.cpu(), w2.cpu(), ids.cpu(), w.cpu()), f"m64 {tile} {dtype}")


@pytest.mark.parametrize("kind", ["int8", "fp8"])
def test_m64_tail_8bit(cuda_device, m64, kind):
    E, H, I, k = len(SIZES), 512, 256, 2
    ids, w, T = routing_with_sizes(SIZES, k, 6, cuda_device)
    w13, w2 = weights(E, H, I, torch.float16, 7, cuda_device)
    x = torch.randn((T, H), generator=torch.Generator().manual_seed(8)).half().to(cuda_device)
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


def test_m64_tail_run_kernel(cuda_device, m64):
    E, H, I = len(SIZES), 512, 384
    gs = torch.tensor(SIZES, dtype=torch.int32)
    go = torch.cat([torch.zeros(1, dtype=torch.int32), torch.cumsum(gs, 0, dtype=torch.int32)])
    padded = (gs + 127) // 128 * 128
    gpo = torch.cat([torch.zeros(1, dtype=torch.int32), torch.cumsum(padded, 0, dtype=torch.int32)])
    gidx = torch.repeat_interleave(torch.arange(E, dtype=torch.int32), padded // 128)
    P, R = int(gpo[-1]), int(go[-1])
    g = torch.Generator().manual_seed(9)
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
    assert_within(out, ref, "run_kernel with half blocks")
    o = out.cpu()
    for e, n in enumerate(SIZES):
        assert torch.count_nonzero(o[int(gpo[e]) + n:int(gpo[e + 1])]) == 0, f"pad rows of expert {e}"
