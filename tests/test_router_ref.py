"""CPU: the router oracle (softmax top-k with a total selection order) against torch's own
softmax -> top-k -> renormalise, and its tie and signed-zero order."""
import numpy as np
import pytest
import torch

import cases
from oracle.router_ref import order_keys, router_ids_ref, router_topk_ref


def tie_free(logits: torch.Tensor, k: int) -> bool:
    """No two of each token's k+1 largest logits are equal (torch.topk's order is then unique)."""
    top = torch.topk(logits.float(), min(k + 1, logits.shape[1]), dim=-1).values
    return bool((top[:, 1:] != top[:, :-1]).all())


@pytest.mark.parametrize("T,E,k", [(512, 8, 2), (1000, 60, 4), (777, 256, 8), (64, 1024, 32), (33, 5, 5)])
def test_oracle_matches_torch_softmax_topk(T, E, k):
    g = torch.Generator().manual_seed(T * 7 + E)
    logits = torch.randn((T, E), generator=g)
    assert tie_free(logits, k)
    probs = torch.softmax(logits, -1)
    vals, ids = torch.topk(probs, k, dim=-1)
    w, ids_ref = router_topk_ref(logits, k, renormalize=True)
    assert torch.equal(ids_ref.long(), ids)
    assert torch.equal(w, vals / vals.sum(-1, keepdim=True))
    w_raw, _ = router_topk_ref(logits, k, renormalize=False)
    assert torch.equal(w_raw, vals)


def test_oracle_reproduces_the_workload_routing():
    """The seeded routing of the fused test cases (tests/golden/cases.py) is the oracle's output."""
    for T, E, k, seed in [(300, 16, 2, 0), (200, 256, 8, 1)]:
        ids, w = cases.routing(T, E, k, seed)
        gen = torch.Generator(device="cpu")
        gen.manual_seed(2000 + seed)
        logits = torch.randn((T, E), generator=gen)
        w_ref, ids_ref = router_topk_ref(logits, k)
        assert torch.equal(ids_ref.long(), ids)
        assert torch.equal(w_ref, w)


def test_ties_rank_lower_expert_first():
    logits = torch.tensor([[1.0, 3.0, 3.0, 2.0, 3.0], [0.0, -0.0, 0.0, -1.0, -0.0]])
    ids = router_ids_ref(logits, 4)
    assert ids[0].tolist() == [1, 2, 4, 3]
    # +0 ranks above -0; equal zeros by ascending id
    assert ids[1].tolist() == [0, 2, 1, 4]


def test_order_keys_are_monotone():
    vals = torch.tensor([-float("inf"), -3.5, -1e-30, -0.0, 0.0, 1e-30, 2.0, float("inf")])
    keys = order_keys(vals[None, :])[0].astype(np.int64)
    assert (np.diff(keys) > 0).all()


def test_low_precision_logits_order_by_value():
    g = torch.Generator().manual_seed(5)
    logits = torch.randn((256, 64), generator=g).to(torch.bfloat16)  # many equal values
    ids = router_ids_ref(logits, 8)
    f = logits.float()
    for t in range(logits.shape[0]):
        sel = f[t, ids[t].long()]
        assert (sel[:-1] >= sel[1:]).all()
        # every unselected logit is below the last selected one, or equal with a larger id
        last_v, last_e = sel[-1].item(), int(ids[t, -1])
        rest = [e for e in range(64) if e not in set(ids[t].tolist())]
        for e in rest:
            assert f[t, e].item() < last_v or (f[t, e].item() == last_v and e > last_e)


def grouped_plain(logits, topk, n_group, topk_group, bias, scale):
    """Group-limited sigmoid routing written the plain torch way (topk + masks), for comparison."""
    T, E = logits.shape
    scores = torch.sigmoid(logits)
    sfc = scores + bias
    gscore = sfc.view(T, n_group, -1).topk(2, dim=-1).values.sum(-1)
    gidx = torch.topk(gscore, topk_group, dim=-1).indices
    gmask = torch.zeros((T, n_group), dtype=torch.bool).scatter_(1, gidx, True)
    emask = gmask.unsqueeze(-1).expand(T, n_group, E // n_group).reshape(T, E)
    ids = torch.topk(sfc.masked_fill(~emask, float("-inf")), topk, dim=-1).indices
    w = scores.gather(1, ids)
    return w / (w.sum(-1, keepdim=True) + 1e-20) * scale, ids


@pytest.mark.parametrize("T,E,n_group,topk_group,k", [(300, 256, 8, 4, 8), (200, 64, 4, 2, 6), (100, 96, 3, 3, 5)])
def test_grouped_oracle_matches_plain_torch(T, E, n_group, topk_group, k):
    from oracle.router_ref import router_grouped_ref

    g = torch.Generator().manual_seed(E + k)
    logits = torch.randn((T, E), generator=g)
    bias = torch.randn(E, generator=g) * 0.05
    w, ids, margins = router_grouped_ref(logits, k, n_group, topk_group, bias, True, 2.5)
    w_p, ids_p = grouped_plain(logits, k, n_group, topk_group, bias, 2.5)
    sure = margins > 1e-6  # tokens without a boundary near-tie (nearly all of them)
    assert int(sure.sum()) >= 0.95 * T
    assert torch.equal(ids.long()[sure], ids_p[sure])  # both descending by biased score
    torch.testing.assert_close(w[sure], w_p[sure])
    torch.testing.assert_close(w.sum(-1), torch.full((T,), 2.5))
    # every chosen expert lies in one of the topk_group chosen groups
    assert max(torch.unique(ids[t].long() // (E // n_group)).numel() for t in range(T)) <= topk_group
