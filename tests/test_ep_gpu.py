"""GPU: expert-parallel kernels (1 GPU, bit-exact against oracle/ep_ref.py) and the full
expert-parallel fused MoE over NCCL (needs >= 2 GPUs; skipped otherwise).

Multi-GPU parity: each rank's output equals the single-process fp32 oracle on the concatenated
tokens of all ranks, within |err| <= 1e-2 + 1e-2 * |ref|.
"""
import datetime
import json
import os
import socket
import traceback

import pytest
import torch
import torch.multiprocessing as mp

from muxi_race_b200.ep import CudaOps, ExpertParallelMoE, ExpertPlacement, PeerMemoryEP
from oracle.ep_ref import combine_ref, pack_ref, plan_ref

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world,E,k,T", [(2, 8, 2, 37), (8, 256, 8, 512), (4, 64, 6, 1000), (1, 16, 4, 64)])
def test_ep_plan_pack_combine_exact(cuda_device, world, E, k, T):
    g = torch.Generator().manual_seed(world * 1000 + E)
    logits = torch.randn((T, E), generator=g)
    ids = torch.topk(logits, k, dim=-1).indices
    w = torch.rand((T, k), generator=g)
    x = torch.randn((T, 128), generator=g).half()
    placement = ExpertPlacement.balanced(torch.rand(E, generator=g).tolist(), world) if world > 1 else \
        ExpertPlacement.contiguous(E, 1)
    ops = CudaOps(placement, cuda_device)
    for id_dtype in (torch.int32, torch.int64):
        d_ids = ids.to(id_dtype).to(cuda_device)
        plan = ops.plan(d_ids)
        send_x, send_ids, send_w = ops.pack(x.to(cuda_device), d_ids, w.to(cuda_device), plan)
        torch.cuda.synchronize()
        counts, pairs, slots = plan_ref(ids, placement.expert_rank, world)
        n = int(counts.sum())
        assert torch.equal(plan.send_counts.cpu(), counts)
        assert int(plan.meta[2]) == n
        assert torch.equal(plan.send_pairs[:n].cpu(), pairs)
        assert torch.equal(plan.pair_slot[: T * world].cpu(), slots)
        rx, rids, rw = pack_ref(x, ids, w, pairs, placement.expert_rank, placement.expert_local, world)
        assert torch.equal(send_x[:n].cpu(), rx)
        assert torch.equal(send_ids[:n].cpu(), rids)
        assert torch.equal(send_w[:n].cpu(), rw)
    y = torch.randn((n, 128), generator=g).half()
    out = ops.combine(y.to(cuda_device), plan, T, 128, torch.float16)
    torch.cuda.synchronize()
    torch.testing.assert_close(out.cpu().float(), combine_ref(y, slots, T, world, torch.float16).float(), rtol=0, atol=0)


# ----------------------------------------------------------------------------- multi-GPU
def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _ep_worker(rank, world, port, out_dir, T_per_rank, E, H, I, k, skew, mode="nccl", env=None):
    import torch.distributed as dist

    os.environ.update(env or {})  # library switches (read on first use, in this process only)

    from muxi_race_b200.workloads import MoeConfig, make_hidden, make_routing, make_weights
    from oracle.moe_ref import fused_moe_ref

    res = {"rank": rank}
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=120), device_id=dev)
        cfg = MoeConfig("ep_test", T_per_rank * world, H, I, E, k, torch.float16, zipf_s=skew)
        w13, w2 = make_weights(cfg, seed=0, device=dev)           # same global weights on every rank
        x = make_hidden(cfg, seed=1, device=dev)                   # global tokens; each rank takes its slice
        ids, w = make_routing(cfg, seed=2, device=dev)
        loads = torch.bincount(ids.flatten().long(), minlength=E).float().cpu().tolist()
        placement = ExpertPlacement.balanced(loads, world)
        mine = placement.local_experts(rank)
        sl = slice(rank * T_per_rank, (rank + 1) * T_per_rank)
        if mode in ("p2p", "p2p_push"):
            moe = PeerMemoryEP(w13[mine].contiguous(), w2[mine].contiguous(), placement, max_tokens=T_per_rank, topk=k,
                               combine="push" if mode == "p2p_push" else "pull")
        else:
            moe = ExpertParallelMoE(w13[mine].contiguous(), w2[mine].contiguous(), placement)
        out = moe(x[sl].contiguous(), ids[sl].contiguous(), w[sl].contiguous())
        out2 = moe(x[sl].contiguous(), ids[sl].contiguous(), w[sl].contiguous())
        ref = fused_moe_ref(x[sl], w13, w2, ids[sl], w[sl])
        # a forward with a different token count on every rank (rank r drops its last 13 * r + 1)
        cut = slice(rank * T_per_rank, (rank + 1) * T_per_rank - 13 * rank - 1)
        out3 = moe(x[cut].contiguous(), ids[cut].contiguous(), w[cut].contiguous())
        ref3 = fused_moe_ref(x[cut], w13, w2, ids[cut], w[cut])
        torch.cuda.synchronize()
        err = (out.float() - ref).abs()
        err3 = (out3.float() - ref3).abs()
        res["bad"] = int((err > 1e-2 + 1e-2 * ref.abs()).sum()) + int((err3 > 1e-2 + 1e-2 * ref3.abs()).sum())
        res["max_err"] = max(float(err.max()), float(err3.max()))
        res["repeat_max_diff"] = float((out2.float() - out.float()).abs().max())
        res["counts"] = moe.last_counts if mode == "nccl" else None
        from muxi_race_b200 import device_status
        res["status"] = device_status()
        if mode != "nccl":
            moe.close()
        dist.barrier()
        dist.destroy_process_group()
    except Exception as exc:
        res["error"] = f"{type(exc).__name__}: {exc}"
        res["trace"] = traceback.format_exc()[-3000:]
    with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
        json.dump(res, f)


@pytest.mark.parametrize("mode", ["nccl", "p2p", "p2p_push"])
@pytest.mark.parametrize("skew", [0.0, 1.1])
def test_ep_multi_gpu_matches_oracle(cuda_device, tmp_path, skew, mode):
    """NCCL all-to-all mode and peer-memory mode against the single-process oracle, including a
    forward where every rank has a different token count."""
    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("expert parallelism needs at least 2 GPUs")
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    ctx = mp.get_context("spawn")
    port = _free_port()
    args = (world, port, str(tmp_path), 256, 64, 1024, 512, 8, skew, mode)
    procs = [ctx.Process(target=_ep_worker, args=(r,) + args) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
        if p.is_alive():
            p.kill()
            pytest.fail("an expert-parallel rank did not finish")
    res = [json.load(open(tmp_path / f"rank{r}.json")) for r in range(world)]
    for r in res:
        assert "error" not in r, r.get("trace")
        assert r["bad"] == 0, r
        assert r["repeat_max_diff"] < 2e-2, r
        assert r["status"] == 0, r
    if mode != "nccl":
        return
    # what rank a sends to rank b, rank b receives from rank a
    for a in range(world):
        for b in range(world):
            assert res[a]["counts"][0][b] == res[b]["counts"][1][a]


def test_ep_p2p_single_rank_matches_oracle(cuda_device, tmp_path):
    """The peer-memory path with one rank (its own region only): routing, gather, grouped GEMMs,
    partial rows and the pull-combine against the oracle on one GPU."""
    ctx = mp.get_context("spawn")
    port = _free_port()
    p = ctx.Process(target=_ep_worker, args=(0, 1, port, str(tmp_path), 300, 32, 1024, 512, 8, 1.1, "p2p"))
    p.start()
    p.join(timeout=600)
    if p.is_alive():
        p.kill()
        pytest.fail("the single-rank peer-memory run did not finish")
    r = json.load(open(tmp_path / "rank0.json"))
    assert "error" not in r, r.get("trace")
    assert r["bad"] == 0 and r["status"] == 0, r
    assert r["repeat_max_diff"] < 2e-2, r
