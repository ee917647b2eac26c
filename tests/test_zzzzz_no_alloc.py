"""GPU: moe_run_kernel_noalloc, the reference drop-in for callers that cannot allocate.

A caller such as the contest's online judge, which binds ``run_kernel`` through the C ABI, passes
only the operator's own tensors, so it cannot hand the operator a scratch buffer. ``moe_run_kernel_noalloc`` keeps the
Stage1 intermediate in the library's static device buffer instead. This test calls it through
the C ABI twice in a row (different inputs, so the second call runs over the first call's leftover
buffer contents) and checks each output against the existing ``moe_run_kernel`` entry point with
a caller-allocated workspace and against the CPU oracle ``run_kernel_ref_f32`` (the reference's own
PyTorch operator), with the tolerance of the other run_kernel tests (|a - b| <= 1e-2 + 1e-2 * |b|).
It also checks that a problem too large for the buffer is refused.

The file name sorts after every other test file (``test_zzzzz_`` > ``test_zzzz_``), so a run that
stops at the first failure has run every other test before this one.
"""
import math

import pytest
import torch

import cases
from muxi_race_b200 import _lib
from oracle.moe_ref import run_kernel_ref_f32

pytestmark = pytest.mark.gpu
RTOL = ATOL = 1e-2


def make_case(seed, dev):
    gen = torch.Generator().manual_seed(seed)
    E, H, I = 6, 512, 384
    gs = cases.random_group_sizes(E, 700, 300, gen)
    go, gpo, gidx = cases.metadata(gs)
    P = int(gpo[-1])
    x = torch.randn((P, H), generator=gen).half()
    gate = (torch.randn((E, I, H), generator=gen) / math.sqrt(H)).half()
    up = (torch.randn((E, I, H), generator=gen) / math.sqrt(H)).half()
    down = (torch.randn((E, H, I), generator=gen) / math.sqrt(I)).half()
    routed = torch.rand((int(gs.sum()),), generator=gen)
    return [t.to(dev) for t in (x, gate, up, down, routed, gs, go, gpo, gidx)], (P, H, I, E)


def args_of(t, dims):
    x, gate, up, down, routed, gs, go, gpo, gidx = t
    P, H, I, E = dims
    return ([x.data_ptr(), gate.data_ptr(), up.data_ptr(), down.data_ptr(), routed.data_ptr(), _lib.MOE_F32,
             gs.data_ptr(), go.data_ptr(), gpo.data_ptr(), gidx.data_ptr()],
            [P, H, I, E, routed.numel(), gidx.numel(), _lib.MOE_F16])


def test_noalloc_matches_workspace_entry_point_twice(cuda_device):
    lib = _lib.lib()
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    for seed in (31, 32):  # two calls in a row on the shared static buffer
        t, dims = make_case(seed, cuda_device)
        ptrs, sizes = args_of(t, dims)
        P, H, I, _ = dims
        out_static = torch.full((P, H), float("nan"), dtype=torch.float16, device=cuda_device)
        out_ref = torch.full((P, H), float("nan"), dtype=torch.float16, device=cuda_device)
        _lib.check("moe_run_kernel_noalloc",
                   lib.moe_run_kernel_noalloc(*ptrs, out_static.data_ptr(), *sizes, stream))
        nbytes = lib.moe_run_kernel_workspace_bytes(P, I, _lib.MOE_F16)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=cuda_device)
        _lib.check("moe_run_kernel",
                   lib.moe_run_kernel(*ptrs, out_ref.data_ptr(), *sizes, ws.data_ptr(), nbytes, stream))
        torch.cuda.synchronize()
        a, b = out_static.float().cpu(), out_ref.float().cpu()
        assert not torch.isnan(a).any()
        bad = (a - b).abs() > ATOL + RTOL * b.abs()
        assert int(bad.sum()) == 0, f"seed {seed}: {int(bad.sum())} elements differ from moe_run_kernel"
        oracle = run_kernel_ref_f32(*[v.cpu() for v in t])
        bad = (a - oracle).abs() > ATOL + RTOL * oracle.abs()
        assert int(bad.sum()) == 0, f"seed {seed}: {int(bad.sum())} elements differ from the oracle"


def test_noalloc_refuses_problems_larger_than_its_buffer(cuda_device):
    lib = _lib.lib()
    # 65536 padded rows x I = 2048 needs 256 MiB > 64 MiB: refused before any pointer is used
    rc = lib.moe_run_kernel_noalloc(*([None] * 5), _lib.MOE_F32, *([None] * 5), 65536, 7168, 2048, 64, 60000, 512,
                                    _lib.MOE_F16, None)
    assert rc == -5
    assert b"static buffer" in lib.moe_last_error()
