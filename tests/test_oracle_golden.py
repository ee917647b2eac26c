"""CPU: pin the oracle against the golden fixtures made from the reference's own PyTorch code."""
import os

import numpy as np
import pytest
import torch

import cases
from oracle.moe_ref import align_ref, fused_moe_ref, run_kernel_ref

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    return np.load(os.path.join(GOLDEN, name), allow_pickle=False)


@pytest.mark.parametrize("name", sorted(cases.RUN_KERNEL_CASES))
def test_run_kernel_oracle_matches_reference(name):
    inputs = cases.run_kernel_inputs(name)
    g = load(f"run_kernel_{name}.npz")
    assert str(g["digest"]) == cases.digest(*inputs), "regenerated inputs drifted from the fixture"
    x = inputs[0]
    out = torch.full((x.shape[0], x.shape[1]), float("nan"), dtype=torch.float16)
    run_kernel_ref(*inputs, out)
    ref = torch.from_numpy(g["out"])
    # same fp32 arithmetic as the reference; allow one fp16 ulp for BLAS blocking differences
    torch.testing.assert_close(out, ref, rtol=1e-3, atol=1e-4)
    exact = (out == ref).float().mean().item()
    assert exact > 0.99, f"only {exact:.4f} of elements bit-identical"
    # padding rows are exactly zero
    gs, gpo = inputs[5].tolist(), inputs[7].tolist()
    for e, n in enumerate(gs):
        assert torch.count_nonzero(out[gpo[e] + n:gpo[e + 1]]) == 0


@pytest.mark.parametrize("name", sorted(cases.FUSED_CASES))
def test_fused_oracle_matches_reference(name):
    x, w13, w2, ids, w = cases.fused_inputs(name)
    g = load(f"fused_{name}.npz")
    assert str(g["digest"]) == cases.digest(x, w13, w2, ids, w)
    out = fused_moe_ref(x, w13, w2, ids, w)
    torch.testing.assert_close(out, torch.from_numpy(g["out_f32"]), rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("name", sorted(cases.ALIGN_CASES))
def test_align_oracle_matches_reference(name):
    ids = cases.align_inputs(name)
    g = load(f"align_{name}.npz")
    assert str(g["digest"]) == cases.digest(ids)
    c = cases.ALIGN_CASES[name]
    a = align_ref(ids.numpy(), c["experts"])
    for key in ("group_sizes", "group_offsets", "group_padded_offsets", "group_idx_for_bx", "sorted_route_ids"):
        np.testing.assert_array_equal(a[key], g[key], err_msg=key)
    # route_slot is the inverse permutation of sorted_route_ids on valid rows
    R = ids.numel()
    valid = a["sorted_route_ids"] < R
    np.testing.assert_array_equal(a["route_slot"][a["sorted_route_ids"][valid]], np.nonzero(valid)[0])


def test_align_oracle_skips_out_of_range_ids():
    ids = np.array([3, -1, 0, 7, 3, 8, 0, 3], dtype=np.int64)  # E = 8: -1 and 8 skipped
    a = align_ref(ids, 8, block_m=4)
    assert a["group_sizes"].tolist() == [2, 0, 0, 3, 0, 0, 0, 1]
    assert a["group_padded_offsets"].tolist() == [0, 4, 4, 4, 8, 8, 8, 8, 12]
    assert a["sorted_route_ids"].tolist() == [2, 6, 8, 8, 0, 4, 7, 8, 3, 8, 8, 8]
    assert a["route_slot"].tolist() == [4, -1, 0, 8, 5, -1, 1, 6]
    assert a["group_idx_for_bx"].tolist() == [0, 3, 7]
