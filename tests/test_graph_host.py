"""graph.call dispatch (shape.cast / optimizer.fusion nodes) on the CPU, with stand-in tensors."""
import pytest

from manifesto_b200 import graph
from manifesto_b200.dtype import DType
from manifesto_b200.errors import DTypeMismatch, InvalidArgument
from manifesto_b200.fusion import Target


class FakeTensor:
    def __init__(self, shape, dtype):
        self._shape, self._dtype, self.closed = tuple(shape), DType(dtype), False

    def shape(self):
        return self._shape

    def dtype(self):
        return self._dtype

    def __len__(self):
        n = 1
        for d in self._shape:
            n *= d
        return n

    def dispatch_pointer(self):
        return 0x1000

    def close(self):
        self.closed = True


class FakeBackend:
    """Records conversions instead of launching them."""

    def __init__(self):
        self.calls = []

    def convert(self, src, dst_dtype, compat=0, stream=None):
        self.calls.append((src.dtype(), DType(dst_dtype), compat))
        return FakeTensor(src.shape(), dst_dtype)

    def empty(self, shape, dtype):
        return FakeTensor(shape, dtype)


def node(attrs, op=graph.SHAPE_CAST, inputs=("x",), nid="c"):
    return graph.GraphNode(nid, op, list(inputs), dict(attrs))


@pytest.mark.parametrize("attr,want", [
    (DType.FLOAT32, DType.FLOAT32), (int(DType.FLOAT8_E4M3), DType.FLOAT8_E4M3), ("F8_E4M3", DType.FLOAT8_E4M3),
    ("bf16", DType.BFLOAT16), (None, DType.FLOAT16), ("", DType.FLOAT16), (DType.INVALID, DType.FLOAT16)])
def test_cast_target_follows_derive_cast_output(attr, want):
    attrs = {} if attr is None else {"dtype": attr}
    assert graph.cast_target(node(attrs), DType.FLOAT16) == want


def test_cast_target_rejects_unknown_names():
    with pytest.raises(InvalidArgument, match="unknown dtype name"):
        graph.cast_target(node({"dtype": "F7"}), DType.FLOAT32)


def run(g, inputs, compat=0):
    be = FakeBackend()
    res = graph.GraphBackend(be, compat=compat).call_graph(graph.GraphCallRequest("g", g, inputs))
    return be, res


def test_cast_chain_and_identity_pass_through():
    x = FakeTensor((4, 8), DType.BFLOAT16)
    g = graph.Graph(nodes=[
        graph.GraphNode("adaptor_cast_a_0", graph.SHAPE_CAST, ["x"],
                        {"dtype": DType.FLOAT32, "from_dtype": DType.BFLOAT16}),
        graph.GraphNode("same", graph.SHAPE_CAST, ["adaptor_cast_a_0"], {"dtype": "F32"}),
        graph.GraphNode("q", graph.SHAPE_CAST, ["same"], {"dtype": "F8_E5M2"}),
    ], inputs=["x"], outputs={"f": "same", "q": "q"})
    be, res = run(g, {"x": x}, compat=1)
    assert be.calls == [(DType.BFLOAT16, DType.FLOAT32, 1), (DType.FLOAT32, DType.FLOAT8_E5M2, 1)]
    assert res.outputs["f"].dtype() == DType.FLOAT32 and res.outputs["q"].dtype() == DType.FLOAT8_E5M2
    assert res.outputs["q"].shape() == (4, 8) and not x.closed and not res.outputs["f"].closed


def test_intermediates_are_freed_outputs_kept():
    x = FakeTensor((16,), DType.FLOAT32)
    g = graph.Graph(nodes=[graph.GraphNode("a", graph.SHAPE_CAST, ["x"], {"dtype": "BF16"}),
                           graph.GraphNode("b", graph.SHAPE_CAST, ["a"], {"dtype": "F16"})],
                    inputs=["x"], outputs={"out": "b"})
    be = FakeBackend()
    made = []
    orig = be.convert
    be.convert = lambda *a, **k: made.append(orig(*a, **k)) or made[-1]
    res = graph.GraphBackend(be).call_graph(graph.GraphCallRequest("g", g, {"x": x}))
    assert made[0].closed and not made[1].closed and res.outputs["out"] is made[1]


def test_errors():
    x = FakeTensor((4,), DType.FLOAT16)
    bad_from = graph.Graph([node({"dtype": "F32", "from_dtype": "BF16"})], ["x"], {"o": "c"})
    with pytest.raises(DTypeMismatch, match="from_dtype BF16 but the input is F16"):
        run(bad_from, {"x": x})
    with pytest.raises(InvalidArgument, match="missing input 'x'"):
        run(bad_from, {})
    two = graph.Graph([node({"dtype": "F32"}, inputs=("x", "x"))], ["x"], {"o": "c"})
    with pytest.raises(InvalidArgument, match="shape.cast needs one input"):
        run(two, {"x": x})
    other = graph.Graph([node({}, op="nn.matmul")], ["x"], {"o": "c"})
    with pytest.raises(InvalidArgument, match="'nn.matmul' .* not supported"):
        run(other, {"x": x})
    dangling = graph.Graph([node({"dtype": "F32"}, inputs=("nope",))], ["x"], {"o": "c"})
    with pytest.raises(InvalidArgument, match="unknown value 'nope'"):
        run(dangling, {"x": x})
    no_kernel = graph.Graph([node({}, op=graph.FUSE_OP)], ["x"], {"o": "c"})
    with pytest.raises(InvalidArgument, match="has no CUDA kernel"):
        run(no_kernel, {"x": x})
    bad_out = graph.Graph([node({"dtype": "F32"})], ["x"], {"o": "zz"})
    with pytest.raises(InvalidArgument, match="unknown node 'zz'"):
        run(bad_out, {"x": x})


def test_kernel_set():
    class K:
        def target(self):
            return Target.CUDA
    k = K()
    ks = graph.KernelSet([k])
    assert ks.for_target(Target.CUDA) is k and ks.for_target(Target.CPU) is None and ks.targets() == [Target.CUDA]


def g_of(*nodes, outputs=None):
    return graph.Graph([graph.GraphNode(i, graph.SHAPE_CAST, list(ins), {}) for i, ins in nodes], ["x", "y"],
                       outputs or {})


def sched(g, cap=0):
    s = graph.schedule_streams(g, cap)
    return {k: (v.stream_id, [(b.event_id, b.stream_id, b.wait) for b in v.barriers]) for k, v in s.items()}


def test_schedule_chain_stays_on_one_stream():
    assert sched(g_of(("a", "x"), ("b", "a"), ("c", "b"))) == {"a": (0, []), "b": (0, []), "c": (0, [])}


def test_schedule_fork_and_merge():
    # two roots open streams 0 and 1; the merge takes the lowest and waits on the other
    got = sched(g_of(("a", "x"), ("b", "y"), ("c", ("a", "b"))))
    assert got == {"a": (0, []), "b": (1, [(1, 1, False)]), "c": (0, [(1, 1, True)])}


def test_schedule_diamond():
    # b continues a's chain; c (also fed by a) finds the chain taken and opens stream 1;
    # d merges onto stream 0 and waits on c's signal
    got = sched(g_of(("a", "x"), ("b", "a"), ("c", "a"), ("d", ("b", "c"))))
    assert got == {"a": (0, [(1, 0, False)]), "b": (0, []), "c": (1, [(1, 0, True), (2, 1, False)]),
                   "d": (0, [(2, 1, True)])}


def test_schedule_stream_cap():
    got = sched(g_of(("a", "x"), ("b", "a"), ("c", "a"), ("d", ("b", "c"))), cap=1)
    assert all(v == (0, []) for v in got.values())
    got = sched(g_of(("a", "x"), ("b", "y"), ("c", "x")), cap=2)
    assert got == {"a": (0, []), "b": (1, []), "c": (0, [])}
