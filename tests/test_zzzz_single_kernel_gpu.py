"""GPU: the single-kernel MoE (Stage1 and Stage2 in one cooperative launch, selected with
``moe_set_single_kernel`` / ``_lib.set_single_kernel``; forced on here, automatic by default)
against the CPU oracle and against the two stage launches.

Checked:
- the reference drop-in ``run_kernel`` on the golden fixtures (the reference's own outputs) and on
  random group splits with empty experts and multi-block experts (race_stress2.py's recipe),
  against ``run_kernel_ref_f32`` with its pad rows zero, and bit for bit equal to the two launches
  (both run the same tiles; the padded-store Stage2 has no atomics);
- ``fused_moe`` (fp16 and bf16) on skewed routings with empty, one-block and many-block experts,
  against ``fused_moe_ref`` (|out - ref| <= 1e-2 + 1e-2 |ref|), including a call with fewer Stage1
  units than SMs (a grid smaller than the GPU);
- repeated calls on one workspace (the per-block counts are cleared by every call);
- a single-kernel call captured into a CUDA graph and replayed on new inputs;
- the device status word stays clear (bit 3 would mean a Stage2 unit gave up waiting for its rows).
"""
import math
import os

import numpy as np
import pytest
import torch

import cases
from muxi_race_b200 import _lib, device_status, fused_moe, run_kernel
from muxi_race_b200.graphs import GraphedMoE
from oracle.moe_ref import fused_moe_ref, run_kernel_ref_f32

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture
def single():
    _lib.set_tile(0, None)
    _lib.set_single_kernel(True)
    yield
    _lib.set_single_kernel(None)


def assert_within(out, ref, what):
    out, ref = out.float().cpu(), ref.float().cpu()
    err = (out - ref).abs()
    bad = err > 1e-2 + 1e-2 * ref.abs()
    assert int(bad.sum()) == 0, f"{what}: {int(bad.sum())}/{out.numel()} outside tolerance (max err {err.max():.3e})"


def check_padding_zero(out, gs, gpo):
    gs, gpo = gs.tolist(), gpo.tolist()
    for e, n in enumerate(gs):
        assert torch.count_nonzero(out[gpo[e] + n:gpo[e + 1]]) == 0, f"pad rows of expert {e} not zero"


def run_both(d, P, H):
    """run_kernel through the single kernel, then through the two launches."""
    out1 = torch.full((P, H), float("nan"), dtype=torch.float16, device=d[0].device)
    run_kernel(*d, out1)
    torch.cuda.synchronize()
    assert device_status() == 0
    _lib.set_single_kernel(False)
    out2 = torch.full((P, H), float("nan"), dtype=torch.float16, device=d[0].device)
    run_kernel(*d, out2)
    torch.cuda.synchronize()
    _lib.set_single_kernel(True)
    return out1, out2


@pytest.mark.parametrize("name", sorted(cases.RUN_KERNEL_CASES))
def test_single_run_kernel_golden(cuda_device, single, name):
    inputs = cases.run_kernel_inputs(name)
    g = np.load(os.path.join(GOLDEN, f"run_kernel_{name}.npz"))
    d = [t.to(cuda_device) for t in inputs]
    out, two = run_both(d, d[0].shape[0], d[0].shape[1])
    assert_within(out, torch.from_numpy(g["out_f32"]), name)
    assert_within(out, torch.from_numpy(g["out"]).float(), name + " vs the reference's fp16 output")
    check_padding_zero(out.cpu(), inputs[5], inputs[7])
    assert torch.equal(out, two), f"{name}: single kernel differs from the two launches"


@pytest.mark.parametrize("seed", range(6))
def test_single_run_kernel_random_splits(cuda_device, single, seed):
    gen = torch.Generator().manual_seed(500 + seed)
    E, H, I = 12, 512, 384
    gs = cases.random_group_sizes(E, 2600, 700, gen)  # empty experts and experts of up to 6 blocks
    go, gpo, gidx = cases.metadata(gs)
    P, R = int(gpo[-1]), int(go[-1])
    x = torch.randn((P, H), generator=gen).half()
    gate = (torch.randn((E, I, H), generator=gen) / math.sqrt(H)).half()
    up = (torch.randn((E, I, H), generator=gen) / math.sqrt(H)).half()
    down = (torch.randn((E, H, I), generator=gen) / math.sqrt(I)).half()
    routed = torch.rand((R,), generator=gen)
    ref = run_kernel_ref_f32(x, gate, up, down, routed, gs, go, gpo, gidx)
    d = [t.to(cuda_device) for t in (x, gate, up, down, routed, gs, go, gpo, gidx)]
    out, two = run_both(d, P, H)
    assert_within(out, ref, f"random split {seed}")
    check_padding_zero(out.cpu(), gs, gpo)
    assert torch.equal(out, two), f"split {seed}: single kernel differs from the two launches"


def test_single_run_kernel_contest_shape(cuda_device, single):
    """Contest case 2 (remote_bench.py:27: H=7168, I=2048, E=32, 4544 valid rows), fp32 torch
    reference on the GPU; 3 calls on one workspace give the same bits."""
    c = dict(experts=32, hidden=7168, intermediate=2048, valid=4544, high_experts=22, low_size=112)
    dev = cuda_device
    gs = cases.make_group_sizes(c)
    go, gpo, gidx = cases.metadata(gs)
    P, E, H, I = int(gpo[-1]), c["experts"], c["hidden"], c["intermediate"]
    g = torch.Generator(device=dev).manual_seed(2)
    x = torch.randn((P, H), generator=g, device=dev).half()
    gate = (torch.randn((E, I, H), generator=g, device=dev) / math.sqrt(I)).half()
    up = (torch.randn((E, I, H), generator=g, device=dev) / math.sqrt(I)).half()
    down = (torch.randn((E, H, I), generator=g, device=dev) / math.sqrt(H)).half()
    routed = torch.rand((c["valid"],), generator=g, device=dev)
    meta = [t.to(dev) for t in (gs, go, gpo, gidx)]
    d = [x, gate, up, down, routed, *meta]
    out, two = run_both(d, P, H)
    ref = run_kernel_ref_f32(x, gate, up, down, routed, *meta)
    assert_within(out, ref, "contest case 2")
    assert torch.equal(out, two)
    again = torch.empty_like(out)
    for _ in range(3):
        run_kernel(*d, again)
    torch.cuda.synchronize()
    assert device_status() == 0
    assert torch.equal(again, out)


def skewed_routing(T, E, k, seed, skew=1.2, empty=3):
    """Top-k of logits with a log-Zipf expert bias; the last `empty` experts get no routes."""
    g = torch.Generator().manual_seed(seed)
    logits = torch.randn((T, E), generator=g)
    ranks = torch.randperm(E, generator=g).double() + 1.0
    logits = logits + ranks.pow(-skew).log().float() * 1.5
    logits[:, E - empty:] = -1e9
    vals, ids = torch.topk(torch.softmax(logits, -1), k, dim=-1)
    return ids.to(torch.int32), vals / vals.sum(-1, keepdim=True)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["fp16", "bf16"])
@pytest.mark.parametrize("T,E,k,H,I", [(3, 4, 2, 256, 128), (700, 16, 4, 1024, 512), (1536, 24, 6, 768, 640)],
                         ids=["tiny", "mid", "skew6"])
def test_single_fused(cuda_device, single, dtype, T, E, k, H, I):
    ids, w = skewed_routing(T, E, k, seed=T + E, empty=1 if E < 8 else 3)
    g = torch.Generator().manual_seed(7 * T + E)
    x = torch.randn((T, H), generator=g).to(dtype)
    w13 = (torch.randn((E, 2 * I, H), generator=g) / math.sqrt(H)).to(dtype)
    w2 = (torch.randn((E, H, I), generator=g) / math.sqrt(I)).to(dtype)
    ref = fused_moe_ref(x, w13, w2, ids, w)
    d = cuda_device
    xd, w13d, w2d, idsd, wd = x.to(d), w13.to(d), w2.to(d), ids.to(d), w.to(d)
    out = torch.full((T, H), float("nan"), dtype=dtype, device=d)
    for _ in range(2):  # the second call re-uses the cached workspace: its counts start from zero again
        fused_moe(xd, w13d, w2d, idsd, wd, out=out)
        torch.cuda.synchronize()
        assert device_status() == 0
        assert_within(out, ref, f"single fused T={T} E={E} {dtype}")


def test_single_graph_replay(cuda_device, single):
    T, H, I, E, k = 256, 1024, 512, 8, 2
    g = torch.Generator().manual_seed(11)
    d = cuda_device
    w13 = (torch.randn((E, 2 * I, H), generator=g) * H ** -0.5).half().to(d)
    w2 = (torch.randn((E, H, I), generator=g) * I ** -0.5).half().to(d)

    def inputs():
        x = torch.randn((T, H), generator=g).half()
        vals, ids = torch.topk(torch.softmax(torch.randn((T, E), generator=g), -1), k, dim=-1)
        return x, ids.to(torch.int32), vals / vals.sum(-1, keepdim=True)

    x, ids, w = [t.to(d) for t in inputs()]
    out = torch.empty((T, H), dtype=torch.float16, device=d)
    gm = GraphedMoE(lambda xx, ii, ww, oo: fused_moe(xx, w13, w2, ii, ww, out=oo), x, ids, w, out)
    for _ in range(3):
        nx, nids, nw = inputs()
        x.copy_(nx.to(d))
        ids.copy_(nids.to(d))
        w.copy_(nw.to(d))
        gm.replay()
        torch.cuda.synchronize()
        assert device_status() == 0
        assert_within(out, fused_moe_ref(nx, w13.cpu(), w2.cpu(), nids, nw), "graph replay")
