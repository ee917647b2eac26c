"""GPU: a fused MoE call captured into a CUDA graph (GraphedMoE) and replayed on new inputs
written into the captured buffers gives the direct call's result (|a - b| <= 1e-2 + 1e-2 |b|:
the top-k combine's atomic order differs between runs), for the token-major call and the
reference drop-in.
"""
import pytest
import torch

from muxi_race_b200 import device_status, fused_moe
from muxi_race_b200.graphs import GraphedMoE

pytestmark = pytest.mark.gpu


def close(a, b):
    err = (a.float() - b.float()).abs()
    return bool((err <= 1e-2 + 1e-2 * b.float().abs()).all())


def test_graphed_fused_moe_replays(cuda_device):
    T, H, I, E, k = 64, 1024, 512, 8, 2  # a decode-sized call
    g = torch.Generator(device="cpu").manual_seed(0)
    d = cuda_device
    w13 = (torch.randn((E, 2 * I, H), generator=g) * H ** -0.5).half().to(d)
    w2 = (torch.randn((E, H, I), generator=g) * I ** -0.5).half().to(d)

    def inputs():
        x = torch.randn((T, H), generator=g).half()
        vals, ids = torch.topk(torch.softmax(torch.randn((T, E), generator=g), -1), k, dim=-1)
        return x.to(d), ids.to(torch.int32).to(d), (vals / vals.sum(-1, keepdim=True)).to(d)

    x, ids, w = inputs()
    out = torch.empty((T, H), dtype=torch.float16, device=d)
    gm = GraphedMoE(lambda xx, ii, ww, oo: fused_moe(xx, w13, w2, ii, ww, out=oo), x, ids, w, out)
    for _ in range(3):
        nx, nids, nw = inputs()
        x.copy_(nx)
        ids.copy_(nids)
        w.copy_(nw)
        gm.replay()
        ref = fused_moe(nx, w13, w2, nids, nw)
        torch.cuda.synchronize()
        assert device_status() == 0
        assert close(out, ref)


def test_graphed_run_kernel_replays(cuda_device):
    import math

    import cases
    from muxi_race_b200 import run_kernel

    d = cuda_device
    c = dict(experts=4, hidden=512, intermediate=256, valid=400, high_experts=1, low_size=60)
    gs = cases.make_group_sizes(c)
    go, gpo, gidx = cases.metadata(gs)
    P, E, H, I = int(gpo[-1]), c["experts"], c["hidden"], c["intermediate"]
    g = torch.Generator(device="cpu").manual_seed(1)
    gate = (torch.randn((E, I, H), generator=g) / math.sqrt(H)).half().to(d)
    up = (torch.randn((E, I, H), generator=g) / math.sqrt(H)).half().to(d)
    down = (torch.randn((E, H, I), generator=g) / math.sqrt(I)).half().to(d)
    meta = [t.to(d) for t in (gs, go, gpo, gidx)]
    x = torch.randn((P, H), generator=g).half().to(d)
    routed = torch.rand((c["valid"],), generator=g).to(d)
    out = torch.empty((P, H), dtype=torch.float16, device=d)
    gm = GraphedMoE(lambda xx, rr, oo: run_kernel(xx, gate, up, down, rr, *meta, oo), x, routed, out)
    for _ in range(2):
        nx = torch.randn((P, H), generator=g).half().to(d)
        nr = torch.rand((c["valid"],), generator=g).to(d)
        x.copy_(nx)
        routed.copy_(nr)
        gm.replay()
        ref = torch.empty_like(out)
        run_kernel(nx, gate, up, down, nr, *meta, ref)
        torch.cuda.synchronize()
        assert device_status() == 0
        assert torch.equal(out, ref)  # the padded-store path has no atomics: identical bits
