"""CPU (gloo, world_size 2): the expert-parallel exchange logic of ``ExpertParallelMoE``.

The CUDA compute steps are replaced by the reference ops (oracle/ep_ref.py) so that the
collectives, split bookkeeping and combine order run on CPU ranks. Failures are injected on the
host: a rank that raises before a collective, and an inconsistent count plan.
"""
import json
import os
import socket
import traceback

import pytest
import torch
import torch.multiprocessing as mp

from muxi_race_b200.ep import ExpertParallelMoE, ExpertPlacement

WORLD = 2
E, H, I, K, T_PER_RANK = 8, 64, 32, 2, 24


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _global_problem(seed=0):
    g = torch.Generator().manual_seed(seed)
    T = T_PER_RANK * WORLD
    x = torch.randn((T, H), generator=g)
    w13 = torch.randn((E, 2 * I, H), generator=g) * H ** -0.5
    w2 = torch.randn((E, H, I), generator=g) * I ** -0.5
    logits = torch.randn((T, E), generator=g)
    vals, ids = torch.topk(torch.softmax(logits, -1), K, dim=-1)
    return x, w13, w2, ids, vals / vals.sum(-1, keepdim=True)


def _placement(kind):
    if kind == "contiguous":
        return ExpertPlacement.contiguous(E, WORLD)
    loads = torch.arange(E, 0, -1).tolist()
    return ExpertPlacement.balanced(loads, WORLD)


def _worker(rank, port, out_dir, kind, fault, chunks=1, cut=T_PER_RANK):
    import datetime

    import torch.distributed as dist

    from oracle.ep_ref import ReferenceOps

    result = {"rank": rank}
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=WORLD,
                                timeout=datetime.timedelta(seconds=10))
        x, w13, w2, ids, w = _global_problem()
        placement = _placement(kind)
        mine = placement.local_experts(rank)
        ops = ReferenceOps(placement)
        if fault == "bad_counts" and rank == 1:
            real_plan = ops.plan

            def bad_plan(topk_ids):
                p = real_plan(topk_ids)
                p.send_counts = p.send_counts.clone()
                p.send_counts[0] = -5
                return p

            ops.plan = bad_plan
        moe = ExpertParallelMoE(w13[mine].contiguous(), w2[mine].contiguous(), placement, ops=ops, chunks=chunks,
                                min_chunk_tokens=8)
        sl = slice(0, cut) if rank == 0 else slice(cut, WORLD * T_PER_RANK)
        if fault == "rank_raises" and rank == 1:
            raise RuntimeError("injected failure on rank 1 before the exchange")
        out = moe(x[sl].contiguous(), ids[sl].contiguous(), w[sl].contiguous())
        result["out"] = out.tolist()
        result["counts"] = moe.last_counts
        dist.barrier()
        dist.destroy_process_group()
    except Exception as exc:  # reported to the test, never hangs: the group timeout bounds every wait
        result["error"] = f"{type(exc).__name__}: {exc}"
        result["trace"] = traceback.format_exc()[-2000:]
    with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
        json.dump(result, f)


def _run(tmp_path, kind="contiguous", fault=None, chunks=1, cut=T_PER_RANK):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, str(tmp_path), kind, fault, chunks, cut))
             for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            pytest.fail("a rank did not finish within 120 s")
    return [json.load(open(tmp_path / f"rank{r}.json")) for r in range(WORLD)]


@pytest.mark.parametrize("kind,chunks,cut", [("contiguous", 1, T_PER_RANK), ("balanced", 1, T_PER_RANK),
                                              ("balanced", 3, 30)])
def test_ep_matches_single_process_oracle(tmp_path, kind, chunks, cut):
    """chunks=3 with 30 / 18 tokens per rank: rank 0 runs three chunks, rank 1 two (plus one round of
    empty sends), so the chunked exchange must line up across ranks with different chunk counts."""
    from oracle.moe_ref import fused_moe_ref

    res = _run(tmp_path, kind, chunks=chunks, cut=cut)
    for r in res:
        assert "error" not in r, r.get("trace")
    x, w13, w2, ids, w = _global_problem()
    ref = fused_moe_ref(x, w13, w2, ids, w)
    got = torch.cat([torch.tensor(r["out"]) for r in res])
    torch.testing.assert_close(got, ref, rtol=1e-4, atol=1e-5)
    # every rank sent to / received from every rank; what one sends the other receives
    (s0, r0), (s1, r1) = res[0]["counts"], res[1]["counts"]
    assert s0[1] == r1[0] and s1[0] == r0[1]


def test_ep_rank_failure_surfaces_as_error(tmp_path):
    res = _run(tmp_path, fault="rank_raises")
    assert "injected failure" in res[1]["error"]
    assert "error" in res[0], "the surviving rank must get an error, not a hang or a silent result"


def test_ep_inconsistent_counts_are_rejected(tmp_path):
    res = _run(tmp_path, fault="bad_counts")
    assert any("inconsistent exchange counts" in r.get("error", "") for r in res)
    assert all("error" in r for r in res)


def test_balanced_placement_evens_load():
    loads = [1000.0 / (i + 1) ** 1.1 for i in range(256)]
    contiguous = ExpertPlacement.contiguous(256, 8)
    balanced = ExpertPlacement.balanced(loads, 8)
    assert sorted(balanced.expert_rank.bincount().tolist()) == [32] * 8
    # with 32 experts per rank, the hottest expert's rank carries it plus at least the 31 coldest
    srt = sorted(loads)
    bound = max(1.0, (max(loads) + sum(srt[:31])) / (sum(loads) / 8))
    assert balanced.max_over_mean_load(loads) <= bound + 0.02
    assert balanced.max_over_mean_load(loads) < contiguous.max_over_mean_load(loads)
    mild = [1.0 / (i + 1) ** 0.5 for i in range(256)]
    assert ExpertPlacement.balanced(mild, 8).max_over_mean_load(mild) < 1.05
