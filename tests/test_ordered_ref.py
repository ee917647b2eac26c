"""CPU: the ordered combine's decomposition, restated with numpy/torch on the oracle's alignment.

The device path runs Stage2 in the padded-store form (row p = routed row scaled by
raw[group_offsets[e] + p - group_padded_offsets[e]]) after permuting the token-major weights into
that raw order (raw_weights_kernel), then sums each token's rows in route order. This test checks
the two index maps against the reference's own definitions: the raw order equals the stable
argsort of the flat ids (the order run_kernel's routed weights use, remote_bench.py:82-101), and
padded store + in-order sum equals the fused operator, with ids outside [0, E) skipped.
"""
import numpy as np
import pytest
import torch

from oracle.moe_ref import align_ref, fused_moe_ref, run_kernel_ref


def raw_weights(al, tw_flat, R):
    """raw[go[e] + i] = tw[sorted[gpo[e] + i]] for every valid padded row (the kernel's map)."""
    raw = np.zeros(R, dtype=np.float32)
    gidx, go, gpo, srt = al["group_idx_for_bx"], al["group_offsets"], al["group_padded_offsets"], al["sorted_route_ids"]
    for p in range(al["padded_rows"]):
        route = int(srt[p])
        if route >= R:
            continue
        e = int(gidx[p // 128])
        raw[int(go[e]) + p - int(gpo[e])] = tw_flat[route]
    return raw


@pytest.mark.parametrize("T,E,k,invalid", [(50, 6, 2, False), (200, 16, 4, True), (129, 3, 3, True)])
def test_ordered_decomposition(T, E, k, invalid):
    g = torch.Generator().manual_seed(T + E)
    H, I = 64, 32
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(torch.int64)
    if invalid:
        ids[::5, 0] = -1
        ids[1::7, -1] = E
    tw = torch.rand((T, k), generator=g)
    x = torch.randn((T, H), generator=g)
    w13 = torch.randn((E, 2 * I, H), generator=g) * H ** -0.5
    w2 = torch.randn((E, H, I), generator=g) * I ** -0.5
    R = T * k
    al = align_ref(ids.numpy(), E)
    flat = ids.reshape(-1).numpy()
    valid = (flat >= 0) & (flat < E)
    raw = raw_weights(al, tw.reshape(-1).numpy(), R)
    # the raw order is the stable argsort of the valid ids
    order = np.argsort(np.where(valid, flat, E), kind="stable")[: int(valid.sum())]
    assert np.array_equal(raw[: order.size], tw.reshape(-1).numpy()[order])
    # padded store with the raw weights, then the in-order per-token sum
    P = al["padded_rows"]
    srt = torch.from_numpy(al["sorted_route_ids"].astype(np.int64))
    stacked = torch.zeros((P, H))
    rows = srt < R
    stacked[rows] = x[srt[rows] // k]
    y = torch.zeros((P, H))
    t = lambda a: torch.from_numpy(np.asarray(a))  # noqa: E731
    run_kernel_ref(stacked, w13[:, :I], w13[:, I:], w2, t(raw[: max(order.size, 1)]), t(al["group_sizes"]),
                   t(al["group_offsets"]), t(al["group_padded_offsets"]), t(al["group_idx_for_bx"]), y)
    slot = al["route_slot"].reshape(T, k)
    out = torch.zeros((T, H))
    for tok in range(T):
        for j in range(k):  # route order
            if slot[tok, j] >= 0:
                out[tok] += y[int(slot[tok, j])]
    keep = torch.from_numpy(valid.reshape(T, k))
    ref = fused_moe_ref(x, w13, w2, torch.where(keep, ids, 0), torch.where(keep, tw, 0.0))
    torch.testing.assert_close(out, ref, rtol=1e-4, atol=1e-5)
