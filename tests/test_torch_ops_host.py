"""CPU: the PyTorch operator registrations exist and propagate shapes on meta tensors (no GPU)."""
import torch

import muxi_race_b200.torch_ops  # noqa: F401 - registers torch.ops.muxi_race_b200.*


def test_ops_registered():
    for name in ("fused_moe", "fused_moe_int8", "fused_moe_fp8", "fused_topk", "grouped_topk", "run_kernel"):
        assert hasattr(torch.ops.muxi_race_b200, name), name


def test_meta_shapes():
    T, H, I, E, k = 64, 256, 128, 8, 2
    m = dict(device="meta")
    x = torch.empty((T, H), dtype=torch.float16, **m)
    w13 = torch.empty((E, 2 * I, H), dtype=torch.float16, **m)
    w2 = torch.empty((E, H, I), dtype=torch.float16, **m)
    ids = torch.empty((T, k), dtype=torch.int32, **m)
    w = torch.empty((T, k), dtype=torch.float32, **m)
    out = torch.ops.muxi_race_b200.fused_moe(x, w13, w2, ids, w)
    assert out.shape == (T, H) and out.dtype == torch.float16 and out.device.type == "meta"
    q13 = torch.empty((E, 2 * I, H), dtype=torch.int8, **m)
    q2 = torch.empty((E, H, I), dtype=torch.int8, **m)
    s13 = torch.empty((E, 2 * I), dtype=torch.float32, **m)
    s2 = torch.empty((E, H), dtype=torch.float32, **m)
    assert torch.ops.muxi_race_b200.fused_moe_int8(x, q13, s13, q2, s2, ids, w).shape == (T, H)
    logits = torch.empty((T, E), dtype=torch.float32, **m)
    tw, tid = torch.ops.muxi_race_b200.fused_topk(logits, k, True)
    assert tw.shape == (T, k) and tw.dtype == torch.float32 and tid.dtype == torch.int32
    gw, gi = torch.ops.muxi_race_b200.grouped_topk(logits, k, True, 4, 2, None, 2.5)
    assert gw.shape == (T, k) and gi.dtype == torch.int32


def test_export_keeps_the_op_as_one_node():
    """torch.export traces a model that calls the op on meta tensors (no GPU): the op stays one
    opaque graph node next to the surrounding aten ops."""
    class Block(torch.nn.Module):
        def forward(self, x, w13, w2, ids, w):
            return torch.ops.muxi_race_b200.fused_moe(x, w13, w2, ids, w) * 2

    m = dict(device="meta")
    args = (torch.empty(64, 256, dtype=torch.float16, **m), torch.empty(8, 256, 256, dtype=torch.float16, **m),
            torch.empty(8, 256, 128, dtype=torch.float16, **m), torch.empty(64, 2, dtype=torch.int32, **m),
            torch.empty(64, 2, **m))
    ep = torch.export.export(Block(), args)
    targets = [str(n.target) for n in ep.graph.nodes if n.op == "call_function"]
    assert targets.count("muxi_race_b200.fused_moe.default") == 1, targets
