"""GPU: group-limited sigmoid routing (moe_router_grouped_topk / grouped_topk, the DeepSeek-V3
router) against ``router_grouped_ref``.

The kernel's sigmoid (CUDA expf) and torch's may differ in the last bit, which can swap two
candidates whose scores are within rounding of each other; so ids are compared bit for bit on the
tokens whose selection boundaries are clear (relative margin > 1e-5, checked to be >= 99% of
them), weights there within rtol 1e-5 / atol 1e-6, and on every token the structural properties
hold (distinct ids, at most topk_group groups, weights summing to the scale). A boundary between
candidates with identical inputs (frequent with bf16 logits) is not a near-tie: both sides compute
the same score for both and break the tie by the lower id.
"""
import pytest
import torch

from muxi_race_b200 import device_status, grouped_topk
from oracle.router_ref import router_grouped_ref

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("E,n_group,topk_group,k", [(256, 8, 4, 8), (64, 4, 2, 6), (96, 3, 3, 5), (33, 11, 5, 3)])
@pytest.mark.parametrize("with_bias", [False, True])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_grouped_router(cuda_device, E, n_group, topk_group, k, with_bias, dtype):
    T, scale = 4096, 2.5
    g = torch.Generator(device="cpu").manual_seed(E * 7 + k)
    logits = torch.randn((T, E), generator=g).to(dtype)
    bias = (torch.randn(E, generator=g) * 0.05) if with_bias else None
    w, ids = grouped_topk(logits.to(cuda_device), logits.to(cuda_device), k, True, n_group, topk_group,
                          bias.to(cuda_device) if bias is not None else None, scale)
    torch.cuda.synchronize()
    assert device_status() == 0
    w_ref, ids_ref, margins = router_grouped_ref(logits, k, n_group, topk_group, bias, True, scale)
    w, ids = w.cpu(), ids.cpu()
    sure = margins > 1e-5
    assert int(sure.sum()) >= 0.99 * T
    assert torch.equal(ids[sure], ids_ref[sure])
    torch.testing.assert_close(w[sure], w_ref[sure], rtol=1e-5, atol=1e-6)
    gsz = E // n_group
    for t in range(0, T, 97):
        assert ids[t].unique().numel() == k and bool(((ids[t] >= 0) & (ids[t] < E)).all())
        assert (ids[t].long() // gsz).unique().numel() <= topk_group
    torch.testing.assert_close(w.sum(-1), torch.full((T,), scale), rtol=1e-5, atol=1e-5)
