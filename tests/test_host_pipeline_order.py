"""CPU: HostPipeline's stream/event ordering, run against a fake CUDA stream model.

The fake records, per stream, the ordered list of operations (copies, the compute call, event
records and event waits). Their happens-before graph has an edge from each op to the next op of
its stream and from each event record to every wait on that event. The test checks that the
pipeline's invariants are implied by that graph (they hold in every execution a GPU may choose),
for several depths: an upload into a buffer slot follows the slot's previous compute; a compute
follows its upload and the slot's previous download; a download follows its compute; and a
schedule that honours the waits runs every op (no wait on an event that is never recorded).
"""
import contextlib
import types

import pytest

from muxi_race_b200 import host_pipeline


class FakeEvent:
    def __init__(self):
        self.stream = None
        self.index = None

    def record(self, stream):
        stream.ops.append(("record", self))


class FakeStream:
    def __init__(self, name):
        self.name = name
        self.ops = []

    def wait_event(self, ev):
        self.ops.append(("wait", ev))

    def synchronize(self):
        pass


class FakeCuda:
    def __init__(self):
        self.compute = FakeStream("compute")
        self.current = self.compute
        self.n = 0

    def Stream(self, dev):  # noqa: N802 - mirrors torch.cuda.Stream
        self.n += 1
        return FakeStream(f"copy{self.n}")

    def Event(self):  # noqa: N802
        return FakeEvent()

    def current_stream(self, dev=None):
        return self.current

    @contextlib.contextmanager
    def stream(self, s):
        prev, self.current = self.current, s
        try:
            yield
        finally:
            self.current = prev


class FakeTensor:
    def __init__(self, cuda, name, device_type="cuda"):
        self.cuda = cuda
        self.name = name
        self.device = types.SimpleNamespace(type=device_type)

    def copy_(self, src, non_blocking=False):
        self.cuda.current.ops.append(("copy", src.name, self.name))
        return self

    def record_stream(self, s):
        pass


def run_streams(streams):
    """Execute the ops in a GPU-like order; return the global execution order of (stream, op)."""
    pos = {s.name: 0 for s in streams}
    done_records = set()
    order = []
    progress = True
    while progress:
        progress = False
        for s in streams:
            while pos[s.name] < len(s.ops):
                kind, arg = s.ops[pos[s.name]][0], s.ops[pos[s.name]][1:]
                if kind == "wait" and id(arg[0]) not in done_records:
                    break
                if kind == "record":
                    done_records.add(id(arg[0]))
                order.append((s.name, s.ops[pos[s.name]]))
                pos[s.name] += 1
                progress = True
    stuck = [s.name for s in streams if pos[s.name] < len(s.ops)]
    assert not stuck, f"streams never finish: {stuck}"
    return order


@pytest.mark.parametrize("depth", [1, 2, 3])
def test_pipeline_ordering(monkeypatch, depth):
    cuda = FakeCuda()
    made = []

    def empty_like(t, device=None):
        made.append(FakeTensor(cuda, f"dev[{t.name}]#{len(made)}"))
        return made[-1]

    fake_torch = types.SimpleNamespace(cuda=cuda, empty_like=empty_like)
    monkeypatch.setattr(host_pipeline, "torch", fake_torch)
    calls = 7
    buffers = []

    def fn(*args):
        d_out = args[-1]
        cuda.current.ops.append(("compute", tuple(a.name for a in args[:-1]), d_out.name))

    x_like = FakeTensor(cuda, "x")
    out_like = FakeTensor(cuda, "out")
    pipe = host_pipeline.HostPipeline(fn, [x_like], out_like, depth=depth)
    for i in range(calls):
        pipe.submit([FakeTensor(cuda, f"hx{i}", "cpu")], FakeTensor(cuda, f"ho{i}", "cpu"))
        buffers.append((pipe.ins[i % depth][0].name, pipe.outs[i % depth].name))
    pipe.synchronize()
    streams = [cuda.compute, pipe.up, pipe.down]
    run_streams(streams)  # every wait is satisfiable
    # happens-before graph over (stream, index) nodes
    succ = {}
    waits = {}
    for st in streams:
        for j, op in enumerate(st.ops):
            succ.setdefault((st.name, j), set())
            if j + 1 < len(st.ops):
                succ[(st.name, j)].add((st.name, j + 1))
            if op[0] == "wait":
                waits.setdefault(id(op[1]), []).append((st.name, j))
    for st in streams:
        for j, op in enumerate(st.ops):
            if op[0] == "record":
                succ[(st.name, j)].update(waits.get(id(op[1]), []))

    def before(a, b):
        seen, todo = set(), [a]
        while todo:
            n = todo.pop()
            if n == b:
                return True
            if n not in seen:
                seen.add(n)
                todo.extend(succ[n])
        return False

    node = {}
    n_compute = 0
    for st in streams:
        for j, op in enumerate(st.ops):
            if op[0] == "copy" and op[1].startswith("hx"):
                node[("up", int(op[1][2:]))] = (st.name, j)
            elif op[0] == "compute":
                node[("compute", n_compute)] = (st.name, j)
                n_compute += 1
            elif op[0] == "copy" and op[2].startswith("ho"):
                node[("down", int(op[2][2:]))] = (st.name, j)
    for i in range(calls):
        assert ("up", i) in node and ("compute", i) in node and ("down", i) in node, f"call {i} incomplete"
        assert before(node[("up", i)], node[("compute", i)])
        assert before(node[("compute", i)], node[("down", i)])
        if i >= depth:
            assert before(node[("compute", i - depth)], node[("up", i)]), "upload may overwrite inputs in use"
            assert before(node[("down", i - depth)], node[("compute", i)]), "compute may overwrite a result"
    # calls i and i+1 use different slots when depth > 1, so their transfers can overlap compute
    if depth > 1:
        assert buffers[0] != buffers[1]
