"""GPU: the peer-memory expert-parallel path with the push combine (Stage2 adds into the home
rank's region) on one rank: routing, gather, grouped GEMMs with the push epilogue, the home-side
zeroing and copy-out, against the oracle (|out - ref| <= 1e-2 + 1e-2 |ref|), including a forward
with fewer tokens. The 2-4 GPU version is ``test_ep_multi_gpu_matches_oracle[p2p_push]``.

The file name sorts after the other GPU test files, so a run that stops at the first failure has
run them all.
"""
import json
import multiprocessing as mp

import pytest

from test_ep_gpu import _ep_worker, _free_port

pytestmark = pytest.mark.gpu


def test_ep_p2p_push_single_rank_matches_oracle(cuda_device, tmp_path):
    ctx = mp.get_context("spawn")
    port = _free_port()
    p = ctx.Process(target=_ep_worker, args=(0, 1, port, str(tmp_path), 300, 32, 1024, 512, 8, 1.1, "p2p_push"))
    p.start()
    p.join(timeout=600)
    if p.is_alive():
        p.kill()
        pytest.fail("the single-rank push-combine run did not finish")
    r = json.load(open(tmp_path / "rank0.json"))
    assert "error" not in r, r.get("trace")
    assert r["bad"] == 0 and r["status"] == 0, r
    assert r["repeat_max_diff"] < 2e-2, r
