"""CPU: the peer-memory expert-parallel decomposition (virtual routes, per-owner partial blocks,
pull-combine over the owners; and the push combine's destination map) reproduces the
single-process oracle, with a different token count
on every simulated rank and a skewed placement. The CUDA kernels of the mode are checked against
the oracle on GPUs (tests/test_ep_gpu.py); this pins the decomposition they implement."""
import torch

from muxi_race_b200.ep import ExpertPlacement
from oracle.ep_ref import p2p_combine_ref, p2p_local_routes_ref, p2p_partials_ref, p2p_push_ref
from oracle.moe_ref import fused_moe_ref


def test_p2p_decomposition_matches_oracle():
    W, E, H, I, k = 3, 12, 64, 32, 3
    T = [20, 7, 13]
    T_max = max(T) + 2
    g = torch.Generator().manual_seed(5)
    w13 = torch.randn((E, 2 * I, H), generator=g) * H ** -0.5
    w2 = torch.randn((E, H, I), generator=g) * I ** -0.5
    xs = [torch.randn((t, H), generator=g) for t in T]
    ids = [torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(t)]) for t in T]
    ws = [torch.softmax(torch.randn((t, k), generator=g), -1) for t in T]
    loads = torch.bincount(torch.cat(ids).flatten(), minlength=E).float().tolist()
    placement = ExpertPlacement.balanced(loads, W)
    partials = []
    for o in range(W):
        mine = placement.local_experts(o)
        partials.append(p2p_partials_ref(xs, ids, ws, placement.expert_rank, placement.expert_local, o, T_max,
                                         w13[mine], w2[mine]))
        # every virtual route of a real token is owned by exactly one rank
        local = p2p_local_routes_ref(ids, placement.expert_rank, placement.expert_local, o, T_max)
        assert local.numel() == W * T_max * k
    owned = sum((p2p_local_routes_ref(ids, placement.expert_rank, placement.expert_local, o, T_max) >= 0).long()
                for o in range(W))
    assert int(owned.sum()) == sum(t * k for t in T) and int(owned.max()) == 1
    for r in range(W):
        out = p2p_combine_ref(partials, ids, placement.expert_rank, r, T_max, torch.float32)
        ref = fused_moe_ref(xs[r], w13, w2, ids[r], ws[r])
        torch.testing.assert_close(out, ref, rtol=1e-5, atol=1e-5)

    # push combine: each owner stores its routes' rows into per-route slots of the home rank, which
    # sums its tokens' slots; every slot of a real route has exactly one writer
    pushed, writes = p2p_push_ref(xs, ids, ws, placement.expert_rank, placement.expert_local, T_max,
                                  [w13[placement.local_experts(o)] for o in range(W)],
                                  [w2[placement.local_experts(o)] for o in range(W)])
    for r in range(W):
        torch.testing.assert_close(pushed[r], fused_moe_ref(xs[r], w13, w2, ids[r], ws[r]), rtol=1e-5, atol=1e-5)
        assert int(writes[r].max()) <= 1 and int(writes[r].sum()) == int(((ids[r] >= 0) & (ids[r] < E)).sum())
