"""GPU: variants of the peer-memory expert-parallel path on one rank, against the oracle
(|out - ref| <= 1e-2 + 1e-2 |ref|), including a forward with fewer tokens: the push combine
(Stage2 adds into the home rank's region; home-side zeroing and copy-out), and the per-route and
bulk-copy token gathers (MOE_B200_EP_GATHER=route / bulk; the deduplicating gather is the default
that the other peer-memory tests run), and the fused gather (MOE_B200_EP_GATHER=fused: Stage1's
gather warps copy the rows while the weights stream). The 2-4 GPU version of the push combine is
``test_ep_multi_gpu_matches_oracle[p2p_push]``; the fused gather runs on 2-4 GPUs below.
"""
import json
import multiprocessing as mp
import os

import pytest
import torch

from test_ep_gpu import _ep_worker, _free_port

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mode,gather", [("p2p_push", ""), ("p2p", "route"), ("p2p_push", "route"), ("p2p", "bulk"),
                                         ("p2p", "fused"), ("p2p_push", "fused")])
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


@pytest.mark.parametrize("mode", ["p2p", "p2p_push"])
@pytest.mark.parametrize("skew", [0.0, 1.1])
def test_ep_fused_gather_multi_gpu_matches_oracle(cuda_device, tmp_path, skew, mode):
    """The fused token gather on 2-4 GPUs: every rank's Stage1 gather warps read the token rows
    over NVLink from all ranks' regions while its weights stream; against the oracle, with a
    forward where every rank has a different token count."""
    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("expert parallelism needs at least 2 GPUs")
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    ctx = mp.get_context("spawn")
    port = _free_port()
    env = {"MOE_B200_EP_GATHER": "fused"}
    procs = [ctx.Process(target=_ep_worker, args=(r, world, port, str(tmp_path), 256, 64, 1024, 512, 8, skew, mode, env))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
        if p.is_alive():
            p.kill()
            pytest.fail("an expert-parallel rank did not finish")
    for r in range(world):
        res = json.load(open(tmp_path / f"rank{r}.json"))
        assert "error" not in res, res.get("trace")
        assert res["bad"] == 0 and res["status"] == 0, res
        assert res["repeat_max_diff"] < 2e-2, res
