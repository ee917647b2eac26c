"""GPU: HostPipeline (fused MoE on pinned host buffers, transfers of consecutive calls overlapped
with compute) gives every call the result of a direct ``fused_moe`` on the same inputs: different
token rows and routing per call, more calls than buffer slots, results compared after one final
synchronize. Tolerance: the fused tests' |a - b| <= 1e-2 + 1e-2 |b| (the top-k combine's atomic
order differs between runs).
"""
import pytest
import torch

from muxi_race_b200 import device_status, fused_moe
from muxi_race_b200.host_pipeline import HostPipeline

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("depth", [1, 2, 3])
def test_host_pipeline_matches_direct_calls(cuda_device, depth):
    T, H, I, E, k, n_calls = 256, 512, 256, 8, 2, 7
    g = torch.Generator(device="cpu").manual_seed(depth)
    w13 = (torch.randn((E, 2 * I, H), generator=g) * H ** -0.5).half().to(cuda_device)
    w2 = (torch.randn((E, H, I), generator=g) * I ** -0.5).half().to(cuda_device)
    calls = []
    for _ in range(n_calls):
        x = torch.randn((T, H), generator=g).half().pin_memory()
        vals, ids = torch.topk(torch.softmax(torch.randn((T, E), generator=g), -1), k, dim=-1)
        w = (vals / vals.sum(-1, keepdim=True)).pin_memory()
        calls.append((x, ids.to(torch.int32).pin_memory(), w, torch.empty((T, H), dtype=torch.float16).pin_memory()))
    fn = lambda xx, ii, ww, oo: fused_moe(xx, w13, w2, ii, ww, out=oo)  # noqa: E731
    x0, i0, w0, _ = calls[0]
    pipe = HostPipeline(fn, [x0.to(cuda_device), i0.to(cuda_device), w0.to(cuda_device)],
                        torch.empty((T, H), dtype=torch.float16, device=cuda_device), depth=depth)
    for x, ids, w, out_h in calls:
        pipe.submit([x, ids, w], out_h)
    pipe.synchronize()
    assert device_status() == 0
    for n, (x, ids, w, out_h) in enumerate(calls):
        ref = fused_moe(x.to(cuda_device), w13, w2, ids.to(cuda_device), w.to(cuda_device)).cpu().float()
        err = (out_h.float() - ref).abs()
        assert bool((err <= 1e-2 + 1e-2 * ref.abs()).all()), f"call {n}: max err {err.max().item():.3e}"
