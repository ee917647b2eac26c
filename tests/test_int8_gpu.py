"""GPU: W8A8 int8 route.

Two checks: (1) against an exact model of the quantised computation (``fused_moe_int8_ref``:
the same quantisers, exact integer GEMMs): relative L2 error < 1e-2; (2) against the fp16/bf16
reference operator: the north star's 5e-2 relative bound, taken as the relative L2 error
||out - ref||_2 / ||ref||_2 <= 5e-2, plus an elementwise sanity bound |out - ref| <= 0.1 * max|ref|
that catches localised corruption (quantisation error is not elementwise-relative near zero).
"""
import pytest
import torch

from muxi_race_b200 import fused_moe_int8, quantize_rows_int8
from muxi_race_b200.workloads import CONFIGS, MoeConfig, make_hidden, make_routing, make_weights
from oracle.moe_ref import fused_moe_int8_ref, fused_moe_ref, quantize_rows_ref

pytestmark = pytest.mark.gpu


def test_quantize_rows_bit_exact(cuda_device):
    g = torch.Generator(device=cuda_device).manual_seed(0)
    w = (torch.randn((3, 96, 256), generator=g, device=cuda_device) * 0.05).half()
    w[1, 5] = 0  # an all-zero row
    q, s = quantize_rows_int8(w)
    qr, sr = quantize_rows_ref(w)
    torch.cuda.synchronize()
    assert torch.equal(q, qr)
    torch.testing.assert_close(s, sr, rtol=0, atol=0)


def int8_case(cfg, T, dev):
    w13, w2 = make_weights(cfg, seed=0, device=dev)
    x = make_hidden(cfg, device=dev, T=T)
    ids, w = make_routing(cfg, device=dev, T=T)
    w13q, w13s = quantize_rows_int8(w13)
    w2q, w2s = quantize_rows_int8(w2)
    return x, w13, w2, w13q, w13s, w2q, w2s, ids, w


@pytest.mark.parametrize("cfg,T", [
    (MoeConfig("small", 0, 512, 256, 8, 2, torch.float16), 200),
    (MoeConfig("small_bf16", 0, 256, 384, 6, 3, torch.bfloat16), 77),
    (CONFIGS["cfg4"], 512),
], ids=lambda v: v.name if isinstance(v, MoeConfig) else f"T{v}")
def test_fused_int8(cuda_device, cfg, T):
    x, w13, w2, w13q, w13s, w2q, w2s, ids, w = int8_case(cfg, T, cuda_device)
    out = fused_moe_int8(x, w13q, w13s, w2q, w2s, ids, w)
    torch.cuda.synchronize()
    exact = fused_moe_int8_ref(x, w13q, w13s, w2q, w2s, ids, w, out_dtype=cfg.dtype)
    # (1) vs the exact quantised model: differences come only from fp32 rounding order and the
    # low-precision combine (and rare one-step requantisation flips)
    rel_exact = ((out.float() - exact).norm() / exact.norm()).item()
    assert rel_exact < 1e-2, rel_exact
    # (2) vs the fp16/bf16 reference operator
    ref = fused_moe_ref(x, w13, w2, ids, w)
    err = (out.float() - ref).abs()
    rel = ((out.float() - ref).norm() / ref.norm()).item()
    print(f"int8 {cfg.name}: rel_l2 vs exact model {rel_exact:.2e}, vs fp reference {rel:.2e}, "
          f"max err / max|ref| {float(err.max() / ref.abs().max()):.2e}")
    assert rel <= 5e-2, rel
    assert float(err.max()) <= 0.1 * float(ref.abs().max())
