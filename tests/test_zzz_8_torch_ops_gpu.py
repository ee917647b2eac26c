"""GPU: the PyTorch operator registrations (torch.ops.muxi_race_b200.*) run the library's kernels:
same results as the Python entry points (|a - b| <= 1e-2 + 1e-2 |b| where the atomic combine is
involved; identical bits for run_kernel and the router).
"""
import pytest
import torch

import cases
import muxi_race_b200.torch_ops  # noqa: F401
from muxi_race_b200 import device_status, fused_moe, fused_topk, run_kernel

pytestmark = pytest.mark.gpu


def test_torch_ops_match_entry_points(cuda_device):
    d = cuda_device
    x, w13, w2, ids, w = (t.to(d) for t in cases.fused_inputs("fused_cfg1"))
    out = torch.ops.muxi_race_b200.fused_moe(x, w13, w2, ids, w)
    ref = fused_moe(x, w13, w2, ids, w)
    torch.cuda.synchronize()
    err = (out.float() - ref.float()).abs()
    assert bool((err <= 1e-2 + 1e-2 * ref.float().abs()).all())

    logits = torch.randn((100, 16), generator=torch.Generator(device="cpu").manual_seed(4)).to(d)
    tw, tid = torch.ops.muxi_race_b200.fused_topk(logits, 4, True)
    rw, rid = fused_topk(logits, logits, 4, True)
    assert torch.equal(tid, rid) and torch.equal(tw, rw)

    name = sorted(cases.RUN_KERNEL_CASES)[0]
    inputs = [t.to(d) for t in cases.run_kernel_inputs(name)]
    o1 = torch.empty((inputs[0].shape[0], inputs[0].shape[1]), dtype=torch.float16, device=d)
    o2 = torch.empty_like(o1)
    torch.ops.muxi_race_b200.run_kernel(*inputs, o1)
    run_kernel(*inputs, o2)
    torch.cuda.synchronize()
    assert device_status() == 0
    assert torch.equal(o1, o2)
