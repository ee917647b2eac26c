"""GPU: variants of the peer-memory expert-parallel path on one rank, against the oracle
(|out - ref| <= 1e-2 + 1e-2 |ref|), including a forward with fewer tokens: the push combine
(Stage2 adds into the home rank's region; home-side zeroing and copy-out), and the per-route and
bulk-copy token gathers (MOE_B200_EP_GATHER=route / bulk; the deduplicating gather is the default
that the other peer-memory tests run). The 2-4 GPU version of the push combine is
``test_ep_multi_gpu_matches_oracle[p2p_push]``.
"""
import json
import multiprocessing as mp

import pytest

from test_ep_gpu import _ep_worker, _free_port

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mode,gather", [("p2p_push", ""), ("p2p", "route"), ("p2p_push", "route"), ("p2p", "bulk")])
def test_ep_p2p_variants_single_rank_match_oracle(cuda_device, tmp_path, mode, gather):
    ctx = mp.get_context("spawn")
    port = _free_port()
    env = {"MOE_B200_EP_GATHER": gather} if gather else {}
    p = ctx.Process(target=_ep_worker, args=(0, 1, port, str(tmp_path), 300, 32, 1024, 512, 8, 1.1, mode, env))
    p.start()
    p.join(timeout=600)
    if p.is_alive():
        p.kill()
        pytest.fail(f"the single-rank {mode} / gather={gather or 'route'} run did not finish")
    r = json.load(open(tmp_path / "rank0.json"))
    assert "error" not in r, r.get("trace")
    assert r["bad"] == 0 and r["status"] == 0, r
    assert r["repeat_max_diff"] < 2e-2, r
