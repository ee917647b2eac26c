"""CPU: the fp8 (e4m3) oracle — per-row quantisation bounds, saturation, and the fp8 fused route
against the fp32 reference operator."""
import torch

import cases
from oracle.moe_ref import fused_moe_fp8_ref, fused_moe_ref, quantize_rows_fp8_ref


def test_quantize_rows_fp8_bounds():
    g = torch.Generator().manual_seed(3)
    w = (torch.randn((64, 256), generator=g) * torch.logspace(-3, 2, 64).unsqueeze(1)).half()
    w[5] = 0
    q, s = quantize_rows_fp8_ref(w)
    assert q.dtype == torch.float8_e4m3fn and s.shape == (64,)
    qf = q.float()
    assert not torch.isnan(qf).any()
    wf = w.float()
    amax = wf.abs().amax(-1)
    # the largest element of each non-zero row lands on +-448
    nz = amax > 0
    assert torch.equal(qf.abs().amax(-1)[nz], torch.full((int(nz.sum()),), 448.0))
    assert torch.equal(s[5:6], torch.zeros(1)) and torch.equal(qf[5], torch.zeros(256))
    # e4m3 keeps 3 fraction bits: relative error <= 2^-4 for normals, absolute <= 2^-10 below 2^-6
    deq = qf * s.unsqueeze(1)
    err = (deq - wf).abs()
    bound = torch.maximum(wf.abs() * 2.0 ** -4, s.unsqueeze(1) * 2.0 ** -10)
    assert bool((err <= bound * (1 + 1e-6)).all())


def test_quantize_rows_fp8_rounds_to_nearest_even():
    # rows scaled so that amax -> 448 exactly: 1 * 448/448; values between e4m3 neighbours
    w = torch.tensor([[448.0, 9.0, 9.5, 10.0, 10.5, 11.0, -9.5, 0.0009765625, 0.001]])
    q, s = quantize_rows_fp8_ref(w)
    assert float(s[0]) == 1.0
    # e4m3 spacing in [8, 16) is 1: 9.5 and 10.5 are ties -> even significands 10 and 10
    assert q.float()[0].tolist() == [448.0, 9.0, 10.0, 10.0, 10.0, 11.0, -10.0, 0.0, 0.001953125]


def test_fp8_route_close_to_fp32_reference():
    """e4m3 keeps 3 fraction bits and the route quantises four operands: about 6.5e-2 relative
    L2 error on this case (int8: 2.5e-2), inside the 1e-1 bound the GPU tests use."""
    name = "fused_cfg1"
    x, w13, w2, ids, w = cases.fused_inputs(name)
    w13_q, w13_s = quantize_rows_fp8_ref(w13)
    w2_q, w2_s = quantize_rows_fp8_ref(w2)
    out8 = fused_moe_fp8_ref(x, w13_q, w13_s, w2_q, w2_s, ids, w)
    ref = fused_moe_ref(x, w13, w2, ids, w)
    rel = (out8 - ref).norm() / ref.norm()
    assert float(rel) < 1e-1, float(rel)
