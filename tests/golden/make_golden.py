"""Generate the golden fixtures from the REFERENCE's own code (run once, where the reference is mounted).

    python tests/golden/make_golden.py [/path/to/muxi_race]

What runs here is the reference, not a restatement:
* the operator: the official PyTorch implementation embedded in
  ``xpuoj_data/problem1_contest5.json`` (section "PyTorch 参考实现"), extracted as text and
  executed as-is (CPU, fp32 arithmetic, fp16 output);
* the fp32 checker ``reference()`` of ``初审材料/源代码/benchmark/race_stress2.py:29-48``;
* the harness helpers ``make_group_sizes`` (``remote_bench.py:60-75``) and ``random_group_sizes``
  (``race_stress2.py:15-26``), extracted from the source files with ``ast`` and run to confirm that
  ``cases.py`` restates them exactly;
* the routing metadata construction of ``remote_bench.py:83-101`` (bincount -> cumsum -> ceil ->
  repeat_interleave), executed from the extracted source lines.

Outputs: ``run_kernel_<case>.npz``, ``fused_<case>.npz``, ``align_<case>.npz`` in this directory,
each with the SHA-256 of the regenerated inputs. Nothing at test time reads the reference.
"""
from __future__ import annotations

import ast
import json
import os
import re
import sys
import textwrap

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import cases  # noqa: E402

if len(sys.argv) < 2:
    sys.exit("usage: python tests/golden/make_golden.py <reference checkout>")
REF = sys.argv[1]
BENCH = os.path.join(REF, "初审材料", "源代码", "benchmark")


def reference_run_kernel():
    spec = json.load(open(os.path.join(REF, "xpuoj_data", "problem1_contest5.json")))
    sections = spec["localizedContentsOfLocale"]["contentSections"]
    text = next(s["text"] for s in sections if s["sectionTitle"] == "PyTorch 参考实现")
    code = re.search(r"```python\n(.*?)```", text, re.S).group(1)
    ns: dict = {}
    exec(compile(code, "problem1_contest5.json:PyTorch-reference", "exec"), ns)
    return ns["run_kernel"]


def extract_functions(path: str, names: list[str], extra_globals: dict) -> dict:
    src = open(path).read()
    tree = ast.parse(src)
    ns = dict(extra_globals)
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and node.name in names:
            exec(compile(ast.Module([node], []), path, "exec"), ns)
    return ns


def reference_metadata_fn():
    """The metadata lines of remote_bench.make_inputs (:83-101), executed verbatim."""
    src = open(os.path.join(BENCH, "remote_bench.py")).read().splitlines()
    body = textwrap.dedent("\n".join(src[82:101]))  # lines 83..101
    assert "group_offsets_cpu" in body and "group_idx_cpu" in body, body

    def run(group_sizes_cpu, experts):
        ns = dict(torch=torch, BLOCK_M=cases.BLOCK_M, cfg={"experts": experts}, group_sizes_cpu=group_sizes_cpu)
        exec(body, ns)
        return ns["group_offsets_cpu"], ns["group_padded_offsets_cpu"], ns["group_idx_cpu"]

    return run


def main():
    ref_run_kernel = reference_run_kernel()
    ref_meta = reference_metadata_fn()
    rb = extract_functions(os.path.join(BENCH, "remote_bench.py"), ["make_group_sizes"],
                           dict(torch=torch, BLOCK_M=cases.BLOCK_M))
    rs = extract_functions(os.path.join(BENCH, "race_stress2.py"), ["random_group_sizes", "reference"],
                           dict(torch=torch, BLOCK_M=cases.BLOCK_M))

    # --- the restated harness helpers must agree with the reference's own
    for name, c in cases.RUN_KERNEL_CASES.items():
        if c["kind"] == "rb":
            assert torch.equal(rb["make_group_sizes"](c), cases.make_group_sizes(c)), name
    for seed in range(5):
        g1, g2 = torch.Generator(), torch.Generator()
        g1.manual_seed(seed)
        g2.manual_seed(seed)
        ref_sizes = rs["random_group_sizes"](dict(experts=7, valid=900), g1)
        assert torch.equal(ref_sizes, cases.random_group_sizes(7, 900, 400, g2)), seed

    # --- run_kernel golden outputs
    for name in cases.RUN_KERNEL_CASES:
        x, gate, up, down, routed, gs, go, gpo, gidx = cases.run_kernel_inputs(name)
        rgo, rgpo, rgidx = ref_meta(gs, gs.numel())
        assert torch.equal(rgo, go) and torch.equal(rgpo, gpo) and torch.equal(rgidx, gidx), name
        out = torch.empty((x.shape[0], x.shape[1]), dtype=torch.float16)
        ref_run_kernel(x, gate, up, down, routed, gs, go, gpo, gidx, out)
        cfg = dict(hidden=x.shape[1], experts=gs.numel())
        out32 = rs["reference"]((x, gate, up, down, routed, gs, go, gpo, gidx), cfg, x.shape[0], "cpu")
        assert torch.allclose(out.float(), out32, rtol=1e-2, atol=1e-3), name
        np.savez_compressed(
            os.path.join(HERE, f"run_kernel_{name}.npz"),
            out=out.numpy(), out_f32=out32.numpy().astype(np.float32),
            digest=np.array(cases.digest(x, gate, up, down, routed, gs, go, gpo, gidx)),
        )
        print("run_kernel", name, tuple(out.shape), "max|out|", float(out.float().abs().max()))

    # --- fused (token-major) golden outputs: reference operator on the stacked layout + combine
    for name in cases.FUSED_CASES:
        x, w13, w2, ids, w = cases.fused_inputs(name)
        T, H = x.shape
        E, I = w13.shape[0], w13.shape[1] // 2
        k = ids.shape[1]
        flat = ids.reshape(-1)
        gs = torch.bincount(flat, minlength=E).to(torch.int32)
        go, gpo, gidx = ref_meta(gs, E)
        order = torch.argsort(flat, stable=True)
        P = int(gpo[-1])
        stacked = torch.zeros((P, H), dtype=torch.float16)
        rank = torch.arange(order.numel()) - go.long()[flat[order]]
        slot = gpo.long()[flat[order]] + rank
        stacked[slot] = x[order // k]
        routed = w.reshape(-1)[order].float()
        y = torch.empty((P, H), dtype=torch.float16)
        ref_run_kernel(stacked, w13[:, :I].contiguous(), w13[:, I:].contiguous(), w2, routed, gs, go, gpo, gidx, y)
        y32 = rs["reference"]((stacked, w13[:, :I], w13[:, I:], w2, routed, gs, go, gpo, gidx),
                              dict(hidden=H, experts=E), P, "cpu")
        out32 = torch.zeros((T, H), dtype=torch.float32).index_add_(0, order // k, y32[slot])
        np.savez_compressed(
            os.path.join(HERE, f"fused_{name}.npz"),
            out_f32=out32.numpy(), digest=np.array(cases.digest(x, w13, w2, ids, w)),
        )
        print("fused", name, tuple(out32.shape), "max|out|", float(out32.abs().max()))

    # --- routing metadata golden outputs
    for name, c in cases.ALIGN_CASES.items():
        ids = cases.align_inputs(name)
        flat = ids.reshape(-1)
        gs = torch.bincount(flat, minlength=c["experts"]).to(torch.int32)
        go, gpo, gidx = ref_meta(gs, c["experts"])
        order = torch.argsort(flat, stable=True)
        P = int(gpo[-1])
        R = flat.numel()
        sorted_ids = torch.full((P,), R, dtype=torch.int32)
        rank = torch.arange(R) - go.long()[flat[order]]
        sorted_ids[gpo.long()[flat[order]] + rank] = order.to(torch.int32)
        np.savez_compressed(
            os.path.join(HERE, f"align_{name}.npz"),
            group_sizes=gs.numpy(), group_offsets=go.numpy(), group_padded_offsets=gpo.numpy(),
            group_idx_for_bx=gidx.numpy(), sorted_route_ids=sorted_ids.numpy(),
            digest=np.array(cases.digest(ids)),
        )
        print("align", name, "P", P)


if __name__ == "__main__":
    main()
