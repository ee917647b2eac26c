"""GPU: the fp8 (e4m3) route, moe_quantize_rows_fp8 / moe_fused_fp8.

Checks: (1) the quantiser is bit-exact against ``quantize_rows_fp8_ref``; (2) the fused output
against the exact model of the quantised computation (``fused_moe_fp8_ref``: same quantisers,
exact float64 GEMMs of the e4m3 values): relative L2 error < 1e-2; (3) against the fp16/bf16
reference operator: relative L2 error <= 1e-1 — e4m3 keeps 3 fraction bits and the route
quantises four operands (activations, gate/up weights, the intermediate, down weights), which
the CPU oracle puts at about 6.5e-2 on the cfg1 case — plus an elementwise sanity bound
|out - ref| <= 0.2 * max|ref| that catches localised corruption.
"""
import pytest
import torch

from muxi_race_b200 import device_status, fused_moe_fp8, quantize_rows_fp8
from muxi_race_b200.workloads import CONFIGS, MoeConfig, make_hidden, make_routing, make_weights
from oracle.moe_ref import fused_moe_fp8_ref, fused_moe_ref, quantize_rows_fp8_ref

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_quantize_rows_fp8_bit_exact(cuda_device, dtype):
    g = torch.Generator(device=cuda_device).manual_seed(0)
    w = (torch.randn((3, 96, 256), generator=g, device=cuda_device) * 0.05).to(dtype)
    w[1, 5] = 0  # an all-zero row
    w[2, 7, :16] = torch.tensor([1e-6, -3e-5, 2e-4, 0.5] * 4, dtype=dtype)  # subnormal e4m3 results
    q, s = quantize_rows_fp8(w)
    qr, sr = quantize_rows_fp8_ref(w)
    torch.cuda.synchronize()
    assert device_status() == 0
    assert torch.equal(q.view(torch.uint8), qr.view(torch.uint8))
    torch.testing.assert_close(s, sr, rtol=0, atol=0)


def fp8_case(cfg, T, dev):
    w13, w2 = make_weights(cfg, seed=0, device=dev)
    x = make_hidden(cfg, device=dev, T=T)
    ids, w = make_routing(cfg, device=dev, T=T)
    w13q, w13s = quantize_rows_fp8(w13)
    w2q, w2s = quantize_rows_fp8(w2)
    return x, w13, w2, w13q, w13s, w2q, w2s, ids, w


@pytest.mark.parametrize("cfg,T", [
    (MoeConfig("small", 0, 512, 256, 8, 2, torch.float16), 200),
    (MoeConfig("small_bf16", 0, 256, 384, 6, 3, torch.bfloat16), 77),
    (MoeConfig("two_block_groups", 0, 1024, 512, 4, 2, torch.float16), 1500),
    (CONFIGS["cfg4"], 512),
], ids=lambda v: v.name if isinstance(v, MoeConfig) else f"T{v}")
def test_fused_fp8(cuda_device, cfg, T):
    x, w13, w2, w13q, w13s, w2q, w2s, ids, w = fp8_case(cfg, T, cuda_device)
    out = fused_moe_fp8(x, w13q, w13s, w2q, w2s, ids, w)
    torch.cuda.synchronize()
    assert device_status() == 0
    exact = fused_moe_fp8_ref(x, w13q, w13s, w2q, w2s, ids, w, out_dtype=cfg.dtype)
    rel_exact = ((out.float() - exact).norm() / exact.norm()).item()
    assert rel_exact < 1e-2, rel_exact
    ref = fused_moe_ref(x, w13, w2, ids, w)
    err = (out.float() - ref).abs()
    rel = ((out.float() - ref).norm() / ref.norm()).item()
    print(f"fp8 {cfg.name}: rel_l2 vs exact model {rel_exact:.2e}, vs fp reference {rel:.2e}, "
          f"max err / max|ref| {float(err.max() / ref.abs().max()):.2e}")
    assert rel <= 1e-1, rel
    assert float(err.max()) <= 0.2 * float(ref.abs().max())
