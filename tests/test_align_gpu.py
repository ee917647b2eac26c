"""GPU: device routing alignment is bit-exact against the reference construction."""
import os

import numpy as np
import pytest
import torch

import cases
from muxi_race_b200 import moe_align
from oracle.moe_ref import align_ref

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
KEYS = ("group_sizes", "group_offsets", "group_padded_offsets")


def check_alignment(al, ref, R):
    for key in KEYS:
        np.testing.assert_array_equal(getattr(al, key).cpu().numpy(), ref[key], err_msg=key)
    P = al.padded_rows()
    assert P == ref["padded_rows"]
    nblk = al.num_blocks()
    np.testing.assert_array_equal(al.group_idx_for_bx[:nblk].cpu().numpy(), ref["group_idx_for_bx"])
    np.testing.assert_array_equal(al.sorted_route_ids[:P].cpu().numpy(), ref["sorted_route_ids"])
    np.testing.assert_array_equal(al.route_slot[:R].cpu().numpy(), ref["route_slot"])
    assert int(al.meta[2]) == int(ref["group_offsets"][-1])


@pytest.mark.parametrize("name", sorted(cases.ALIGN_CASES))
def test_align_matches_golden(cuda_device, name):
    ids = cases.align_inputs(name)
    g = np.load(os.path.join(GOLDEN, f"align_{name}.npz"))
    E = cases.ALIGN_CASES[name]["experts"]
    for dt in (torch.int64, torch.int32):
        al = moe_align(ids.to(dt).reshape(-1).to(cuda_device), E)
        torch.cuda.synchronize()
        for key in KEYS + ("sorted_route_ids",):
            got = getattr(al, key).cpu().numpy()
            if key == "sorted_route_ids":
                got = got[: al.padded_rows()]
            np.testing.assert_array_equal(got, g[key], err_msg=key)
        np.testing.assert_array_equal(al.group_idx_for_bx[: al.num_blocks()].cpu().numpy(), g["group_idx_for_bx"])


@pytest.mark.parametrize("T,E,k,skew,seed", [
    (1, 8, 1, 0.0, 0),            # single route
    (5, 1024, 3, 0.0, 1),         # E at the shared-memory limit, mostly empty experts
    (4096, 256, 8, 0.0, 2),       # cfg3 routing
    (128, 256, 8, 0.0, 3),        # decode-like: many empty experts
    (32768, 256, 8, 1.1, 4),      # cfg5 routing, Zipf-skewed (R = 262144, many chunks)
    (3000, 7, 5, 0.0, 5),         # few experts, multi-block groups
])
def test_align_random_and_large(cuda_device, T, E, k, skew, seed):
    ids, _ = cases.routing(T, E, k, seed, skew)
    al = moe_align(ids.reshape(-1).to(cuda_device), E)
    torch.cuda.synchronize()
    check_alignment(al, align_ref(ids.numpy(), E), T * k)


def test_align_skips_out_of_range_ids_and_other_block_sizes(cuda_device):
    gen = torch.Generator().manual_seed(7)
    ids = torch.randint(-3, 20, (5000,), generator=gen)  # E = 16: -3..-1 and 16..19 skipped
    for bm in (128, 64, 1):
        al = moe_align(ids.to(cuda_device), 16, block_m=bm)
        torch.cuda.synchronize()
        ref = align_ref(ids.numpy(), 16, block_m=bm)
        for key in KEYS:
            np.testing.assert_array_equal(getattr(al, key).cpu().numpy(), ref[key], err_msg=f"{key} bm={bm}")
        P = al.padded_rows()
        np.testing.assert_array_equal(al.sorted_route_ids[:P].cpu().numpy(), ref["sorted_route_ids"])
        np.testing.assert_array_equal(al.route_slot[:5000].cpu().numpy(), ref["route_slot"])


def test_align_is_deterministic(cuda_device):
    ids, _ = cases.routing(8192, 64, 8, 11)
    d = ids.reshape(-1).to(cuda_device)
    first = moe_align(d, 64)
    ref = first.sorted_route_ids.clone()
    for _ in range(5):
        again = moe_align(d, 64)
        assert torch.equal(again.sorted_route_ids[: first.padded_rows()], ref[: first.padded_rows()])
