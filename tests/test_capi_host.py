"""CPU: the C-ABI library loads, exports every declared symbol, and host-side checks run without a GPU."""
import ctypes
import os
import re

import pytest
import torch

from muxi_race_b200 import _lib
from muxi_race_b200.workloads import CONFIGS

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "moe_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"MOE_API\s+[\w\s\*]+?\b(moe_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_symbols()
    for expected in ("moe_run_kernel", "moe_align", "moe_fused", "moe_fused_int8", "moe_quantize_rows_int8"):
        assert expected in names


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    for name in declared_symbols():
        assert hasattr(lib, name), f"{name} declared in moe_b200.h but not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_version_and_pure_host_queries():
    lib = _lib.lib()
    assert b"sm_100a" in lib.moe_version()
    # moe_max_padded_rows: sum_e ceil(n_e / bm) * bm <= R + min(E, R) * (bm - 1), rounded to bm
    assert lib.moe_max_padded_rows(0, 8, 128) == 0
    assert lib.moe_max_padded_rows(1, 8, 128) == 128
    assert lib.moe_max_padded_rows(128, 8, 128) == 1152
    assert lib.moe_max_padded_rows(32768, 256, 128) == 65280
    # U, then the block groups + count and the single kernel's per-block counts (256 bytes each)
    assert lib.moe_run_kernel_workspace_bytes(256, 2048, _lib.MOE_F16) == 256 * 2048 * 2 + 256 + 256
    # the Stage1 intermediate U [P_max, I] dominates (token rows are gathered inside Stage1)
    assert lib.moe_fused_workspace_bytes(4096, 8, 256, 7168, 2048, _lib.MOE_F16) >= 65280 * 2048 * 2


def test_invalid_arguments_fail_before_any_launch():
    lib = _lib.lib()
    # odd hidden size is rejected by the argument check (no device pointer is touched)
    rc = lib.moe_run_kernel(*([None] * 5), _lib.MOE_F32, *([None] * 5), 128, 100, 64, 1, 1, 1, _lib.MOE_F16, None, 0,
                            None)
    assert rc == -1 and b"multiples of 8" in lib.moe_last_error()
    rc = lib.moe_run_kernel(*([None] * 5), _lib.MOE_F32, *([None] * 5), 256, 128, 64, 1, 1, 1, _lib.MOE_F16, None, 0,
                            None)
    assert rc == -1 and b"num_blocks_m" in lib.moe_last_error()
    rc = lib.moe_align(None, _lib.MOE_I32, 10, 2000, 128, *([None] * 7), None, 0, None)
    assert rc == -1 and b"num_experts" in lib.moe_last_error()
    for fn in ("moe_fused", "moe_fused_ordered"):
        with pytest.raises(_lib.MoeError, match="MOE_ERR_INVALID_ARG"):
            _lib.call(fn, *([None] * 4), _lib.MOE_I8, None, _lib.MOE_F32, None, 4, 128, 128, 8, 2, _lib.MOE_F16,
                      None, 0, None)
    # the ordered combine's workspace adds the padded Stage2 rows and the raw-order weights
    T, k, E, H, I = 4096, 8, 256, 7168, 2048
    extra = lib.moe_fused_ordered_workspace_bytes(T, k, E, H, I, _lib.MOE_F16) - lib.moe_fused_workspace_bytes(
        T, k, E, H, I, _lib.MOE_F16)
    assert extra >= lib.moe_max_padded_rows(T * k, E, 128) * H * 2 + T * k * 4


def test_router_argument_checks():
    """moe_router_topk / moe_fused_router refuse bad arguments before touching a device pointer;
    no tokens is a no-op."""
    lib = _lib.lib()
    cases = [((_lib.MOE_F32, 8, 256, 33), b"topk"), ((_lib.MOE_F32, 8, 4, 5), b"topk"),
             ((_lib.MOE_F32, 8, 2000, 8), b"num_experts"), ((_lib.MOE_I8, 8, 256, 8), b"fp32, fp16 or bf16"),
             ((_lib.MOE_F16, -1, 256, 8), b"token count")]
    for (dt, T, E, k), msg in cases:
        rc = lib.moe_router_topk(None, dt, T, E, k, 1, None, None, None)
        assert rc == -1 and msg in lib.moe_last_error(), (dt, T, E, k, lib.moe_last_error())
        rc = lib.moe_fused_router(None, None, None, None, dt, 1, None, None, None, T, 128, 128, E, k, _lib.MOE_F16,
                                  None, 0, None)
        assert rc == -1 and msg in lib.moe_last_error(), (dt, T, E, k, lib.moe_last_error())
    assert lib.moe_router_topk(None, _lib.MOE_F32, 0, 256, 8, 1, None, None, None) == 0
    # grouped routing: groups must divide the experts, topk_group <= groups, topk within reach
    for (E, ng, tg, k), msg in [((256, 7, 4, 8), b"divide"), ((256, 8, 9, 8), b"topk_group"),
                                ((256, 64, 1, 8), b"num_expert_group"), ((64, 8, 1, 9), b"topk")]:
        rc = lib.moe_router_grouped_topk(None, _lib.MOE_F32, None, 8, E, ng, tg, k, 1, 1.0, None, None, None)
        assert rc == -1 and msg in lib.moe_last_error(), (E, ng, tg, k, lib.moe_last_error())
    assert lib.moe_router_grouped_topk(None, _lib.MOE_F32, None, 0, 256, 8, 4, 8, 1, 2.5, None, None, None) == 0
    rc = lib.moe_router_topk(None, _lib.MOE_F32, 4, 256, 8, 1, None, None, None)
    assert rc == -1 and b"null" in lib.moe_last_error()


def test_python_entry_points_reject_cpu_tensors():
    from muxi_race_b200 import fused_moe, run_kernel

    x = torch.zeros(128, 64, dtype=torch.float16)
    w = torch.zeros(1, 64, 64, dtype=torch.float16)
    meta = [torch.zeros(n, dtype=torch.int32) for n in (1, 2, 2, 1)]
    with pytest.raises(ValueError, match="CUDA"):
        run_kernel(x, w, w, w, torch.zeros(4), *meta, torch.zeros_like(x))
    with pytest.raises(ValueError):
        fused_moe(x, torch.zeros(1, 128, 64, dtype=torch.float16), w, torch.zeros(128, 1, dtype=torch.int32),
                  torch.zeros(128, 1))


def test_workload_algorithmic_work():
    c = CONFIGS["cfg3"]
    assert c.flops() == pytest.approx(2.886e12, rel=1e-3)
    assert c.weight_bytes() == pytest.approx(22.55e9, rel=1e-3)
    assert CONFIGS["cfg4"].weight_bytes() == pytest.approx(11.27e9, rel=1e-3)


def test_set_tile_host():
    """Tile selection is host state: known names and "auto" are accepted, unknown ones refused."""
    _lib.set_tile(0, "p256a6b8")
    _lib.set_tile(1, "256a4b5")
    _lib.set_tile(2, None)
    _lib.set_tile(0, "auto")
    with pytest.raises(_lib.MoeError):
        _lib.set_tile(2, "256a4b5x")
    with pytest.raises(_lib.MoeError):
        _lib.set_tile(-1, "auto")


def test_peer_memory_ep_host_checks():
    """Peer-memory expert parallelism: region and workspace sizes, and argument checks that fail
    before any CUDA call."""
    lib = _lib.lib()
    T, H, k, W = 4096, 7168, 8, 8
    region = lib.moe_ep_region_bytes(T, H, k, W)
    # flags + count, x [T, H], ids and weights [T, k], partials [W * T, H], each 256-byte aligned
    assert region >= T * H * 2 + 2 * T * k * 4 + W * T * H * 2
    assert region % 256 == 0 and region < T * H * 2 + 2 * T * k * 4 + W * T * H * 2 + 8192
    assert lib.moe_ep_region_bytes(T, H, k, 33) == 0 and lib.moe_ep_region_bytes(0, H, k, W) == 0
    ws = lib.moe_ep_p2p_workspace_bytes(T, k, W, 32, H, 2048, _lib.MOE_F16)
    # the local pipeline over W * T virtual tokens plus the local ids and weights of every route
    assert ws >= lib.moe_fused_workspace_bytes(W * T, k, 32, H, 2048, _lib.MOE_F16) + 2 * 4 * W * T * k
    assert lib.moe_ep_p2p_workspace_bytes(T, k, 0, 32, H, 2048, _lib.MOE_F16) == 0
    # more tokens than the region holds, a world above 32, a rank outside the world
    rc = lib.moe_ep_p2p_stage(None, None, None, _lib.MOE_I32, None, _lib.MOE_F32, T + 1, T, H, k, W, _lib.MOE_F16,
                              None)
    assert rc == -1 and b"max_tokens" in lib.moe_last_error()
    rc = lib.moe_ep_p2p_stage(None, None, None, _lib.MOE_I32, None, _lib.MOE_F32, 1, T, H, k, 33, _lib.MOE_F16, None)
    assert rc == -1 and b"world" in lib.moe_last_error()
    assert lib.moe_ep_p2p_barrier(None, 0, W, 1, None) == -1
    rc = lib.moe_ep_p2p_combine(None, 8, W, 4, T, H, k, None, 256, _lib.MOE_F16, None, None)
    assert rc == -1
    rc = lib.moe_ep_p2p_compute(None, None, 0, W, T, H, 2048, k, None, None, 256, None, None, 32, _lib.MOE_F16, None,
                                0, None)
    assert rc == -1 and b"regions" in lib.moe_last_error()
    assert lib.moe_ep_region_alloc(0, None) == -1
    # push combine entry points: the same checks, no device pointer touched
    rc = lib.moe_ep_p2p_compute_push(None, None, 0, W, T, H, 2048, k, None, None, 256, None, None, 32, _lib.MOE_F16,
                                     None, 0, None)
    assert rc == -1 and b"regions" in lib.moe_last_error()
    assert lib.moe_ep_p2p_push_prepare(None, T + 1, T, H, k, W, _lib.MOE_F16, None) == -1
    assert lib.moe_ep_p2p_push_prepare(None, 0, T, H, k, W, _lib.MOE_F16, None) == -1  # null region
    assert lib.moe_ep_p2p_push_finish(None, 4, T, H, k, W, 64, _lib.MOE_F32, None, None) == -1
    assert b"dtype" in lib.moe_last_error()


def test_host_pipeline_needs_cuda_tensors():
    from muxi_race_b200.host_pipeline import HostPipeline

    with pytest.raises(ValueError, match="CUDA"):
        HostPipeline(lambda *a: None, [torch.zeros(4)], torch.zeros(4))
    with pytest.raises(ValueError, match="depth"):
        HostPipeline(lambda *a: None, [torch.zeros(4)], torch.zeros(4), depth=0)


def test_python_argument_checks_without_a_gpu():
    """Shape and dtype errors of the Python entry points are reported before any device work."""
    from muxi_race_b200 import fused_moe, fused_topk
    from muxi_race_b200.packed import PackedWeights, fused_moe_packed, packed_layout

    x = torch.zeros(16, 64, dtype=torch.float16)
    w13 = torch.zeros(4, 64, 64, dtype=torch.float16)   # 2I = 64 -> I = 32
    w2 = torch.zeros(4, 64, 32, dtype=torch.float16)
    ids = torch.zeros(16, 2, dtype=torch.int32)
    w = torch.zeros(16, 2)
    with pytest.raises(ValueError, match="w_down shape"):
        fused_moe(x, w13, torch.zeros(4, 64, 16, dtype=torch.float16), ids, w)
    with pytest.raises(ValueError, match="topk_ids and topk_weights"):
        fused_moe(x, w13, w2, ids, torch.zeros(16, 3))
    with pytest.raises(ValueError, match="topk"):
        fused_topk(x, torch.zeros(16, 8), 9)
    _, total = packed_layout(4, 64, 32, "fp16")
    p = PackedWeights(torch.zeros(total, dtype=torch.uint8), 4, 64, 32, "fp16")
    with pytest.raises(ValueError, match="hidden size"):
        fused_moe_packed(torch.zeros(16, 128, dtype=torch.float16), p, ids, w)


def test_a_path_selection_sizes_the_workspace():
    """The gather4 A path reads token rows in place: no stacked copy in the workspace."""
    lib = _lib.lib()
    args = (4096, 8, 256, 7168, 2048, _lib.MOE_F16)
    try:
        _lib.set_a_path("tma")
        stacked = lib.moe_fused_workspace_bytes(*args)
        _lib.set_a_path("gather")
        in_place = lib.moe_fused_workspace_bytes(*args)
        assert stacked - in_place >= 65280 * 7168 * 2  # the [P_max, H] stacked rows
        with pytest.raises(_lib.MoeError, match="MOE_ERR_INVALID_ARG"):
            _lib.set_a_path("no-such-path")
    finally:
        _lib.set_a_path(None)


def test_single_kernel_switch():
    """moe_set_single_kernel takes 0 (two launches), 1 (single kernel) or 2 (automatic); anything
    else is refused."""
    lib = _lib.lib()
    try:
        for mode in (1, 0, 2):
            assert lib.moe_set_single_kernel(mode) == 0
        for bad in (3, -1):
            with pytest.raises(_lib.MoeError, match="MOE_ERR_INVALID_ARG"):
                _lib.call("moe_set_single_kernel", bad)
        assert b"0, 1 or 2" in lib.moe_last_error()
    finally:
        _lib.set_single_kernel(None)
