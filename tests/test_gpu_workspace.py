"""Graphs running inside an attached workspace (runtime.WorkspaceAttacher): one device
allocation planned by workspace.plan_graph, inputs copied to their slots, every node writing
its own slot; results bit-identical to the allocating path and to the oracle."""
import numpy as np
import pytest

from manifesto_b200 import fusion, graph, synthetic
from manifesto_b200 import workspace as wsp
from manifesto_b200.dtype import DType
from manifesto_b200.errors import DTypeMismatch, InvalidArgument, ShapeMismatch
from oracle.ref import BF16, E4M3, F16, F32

pytestmark = pytest.mark.gpu

T = wsp.port_type


def cast_chain():
    """x BF16 -> a F16 -> b BF16 -> c F16, all [N]: c's slot is a's (a graph output)."""
    bf, hf = T(DType.BFLOAT16, "N"), T(DType.FLOAT16, "N")
    return graph.Graph(nodes=[
        graph.GraphNode("a", graph.SHAPE_CAST, ["x"], {"dtype": "F16"}, input_types=[bf], output_type=hf),
        graph.GraphNode("b", graph.SHAPE_CAST, ["a"], {"dtype": "BF16"}, input_types=[hf], output_type=bf),
        graph.GraphNode("c", graph.SHAPE_CAST, ["b"], {"dtype": "F16"}, input_types=[bf], output_type=hf),
    ], inputs=["x"], outputs={"a": "a", "c": "c"}, bindings={"N": 1 << 20})


def host(backend, t, np_dtype):
    return np.frombuffer(backend.download(t)[1], np_dtype)


def test_cast_chain_in_workspace(backend, ref):
    g = cast_chain()
    gb = graph.GraphBackend(backend)
    topo = gb.attach_workspace("chain", g)
    ws = gb.workspace("chain")
    assert ws.snapshot == {0} and topo.workspace.size == 2 * 2 * (1 << 20)
    for n in (1 << 20, 1000):
        x = synthetic.normal_bf16(601 + n, n, 0.0, 50.0)
        xt = backend.upload([n], DType.BFLOAT16, x)
        out = gb.call_graph(graph.GraphCallRequest("chain", g, {"x": xt}, launch_bindings={"N": n})).outputs
        a = ref.convert(x, BF16, F16).view(np.uint16)
        c = ref.convert(ref.convert(a, F16, BF16).view(np.uint16), BF16, F16).view(np.uint16)
        assert np.array_equal(host(backend, out["a"], np.uint16), a)
        assert np.array_equal(host(backend, out["c"], np.uint16), c)
        assert out["c"].shape() == (n,) and ws.contains(out["c"].dispatch_pointer())
        assert not ws.contains(out["a"].dispatch_pointer())      # saved before c overwrote its slot
        plain = graph.GraphBackend(backend).call_graph(graph.GraphCallRequest("chain", g, {"x": xt})).outputs
        for k in ("a", "c"):
            assert backend.download(plain[k])[1] == backend.download(out[k])[1]
            plain[k].close()
        out["a"].close()
        xt.close()
    xt = backend.upload([(1 << 20) + 8], DType.BFLOAT16, synthetic.normal_bf16(1, (1 << 20) + 8))
    with pytest.raises(ShapeMismatch):      # a launch binding above the planned bound
        gb.call_graph(graph.GraphCallRequest("chain", g, {"x": xt}, launch_bindings={"N": (1 << 20) + 8}))
    xt.close()
    xt = backend.upload([1 << 20], DType.FLOAT16, synthetic.normal_bf16(2, 1 << 20))
    with pytest.raises(DTypeMismatch):
        gb.call_graph(graph.GraphCallRequest("chain", g, {"x": xt}))
    xt.close()
    other = cast_chain()
    other.nodes[2].inputs = ["a"]
    xt = backend.upload([1 << 20], DType.BFLOAT16, synthetic.normal_bf16(3, 1 << 20))
    with pytest.raises(InvalidArgument):    # planned for another graph
        gb.call_graph(graph.GraphCallRequest("chain", other, {"x": xt}))
    gb.detach_workspace("chain")
    out = gb.call_graph(graph.GraphCallRequest("chain", g, {"x": xt})).outputs   # allocating path again
    assert out["c"].dtype() == DType.FLOAT16
    for t in (xt, *out.values()):
        t.close()
    gb.close()


def diamond(n: int):
    f32, f16, bf, q = T(DType.FLOAT32, n), T(DType.FLOAT16, n), T(DType.BFLOAT16, n), T(DType.FLOAT8_E4M3, n)
    add = fusion.FusionAST(fusion.binary(fusion.NodeType.ADD, fusion.input_node(0), fusion.input_node(1)),
                           ["b", "c"], "d", dtype=DType.FLOAT32)
    k = fusion.emit_cuda(add, in_dtypes=[DType.FLOAT16, DType.BFLOAT16], out_dtype=DType.FLOAT32)
    g = graph.Graph(nodes=[
        graph.GraphNode("a", graph.SHAPE_CAST, ["x"], {"dtype": "F32"}, input_types=[bf], output_type=f32),
        graph.GraphNode("b", graph.SHAPE_CAST, ["a"], {"dtype": "F16"}, input_types=[f32], output_type=f16),
        graph.GraphNode("c", graph.SHAPE_CAST, ["a"], {"dtype": "BF16"}, input_types=[f32], output_type=bf),
        graph.GraphNode("d", graph.FUSE_OP, ["b", "c"], {graph.KERNEL_ATTRIBUTE: graph.KernelSet([k])},
                        input_types=[f16, bf], output_type=f32),
        graph.GraphNode("e", graph.SHAPE_CAST, ["y"], {"dtype": "F8_E4M3"}, input_types=[bf], output_type=q),
    ], inputs=["x", "y"], outputs={"d": "d", "e": "e"})
    return g, k


@pytest.mark.parametrize("align", [64, 1024])
def test_scheduled_diamond_in_workspace(backend, ref, align):
    """e (stream 2, reading only y) is given the bytes of a and d: it must wait for the nodes
    on streams 0 and 1 that use them, and d (a graph output) is saved before e runs."""
    n = 1 << 22
    g, k = diamond(n)
    topo = wsp.plan_graph(g, align=align)
    deps, snap = graph.plan_hazards(g, topo)
    assert deps[4] == (0, 1, 2, 3) and snap == {3}
    sched = graph.schedule_streams(g)
    assert [sched[i].stream_id for i in "abcde"] == [0, 0, 1, 0, 2]
    gb = graph.GraphBackend(backend)
    gb.attach_workspace("diamond", g, topo)
    assert gb.workspace("diamond").base % align == 0
    x = synthetic.normal_bf16(701, n)
    y = synthetic.normal_bf16(702, n, 0.0, 30.0)
    ins = {"x": backend.upload([n], DType.BFLOAT16, x), "y": backend.upload([n], DType.BFLOAT16, y)}
    serial = graph.GraphBackend(backend).call_graph(graph.GraphCallRequest("diamond", g, ins)).outputs
    a = ref.convert(x, BF16, F32).view(np.uint32)
    want_e = ref.convert(y, BF16, E4M3)
    for rep in range(3):
        out = gb.call_graph(graph.GraphCallRequest("diamond", g, ins), schedule=sched).outputs
        for name in ("d", "e"):
            assert backend.download(out[name])[1] == backend.download(serial[name])[1], (rep, name)
        assert np.array_equal(host(backend, out["e"], np.uint8), want_e)
        out["d"].close()
    d = host(backend, serial["d"], np.float32)
    b = ref.convert(a, F32, F16).view(np.uint16)
    c = ref.convert(a, F32, BF16).view(np.uint16)
    want_d = ref.fused_eval(fusion.node_table(fusion.FusionAST(
        fusion.binary(fusion.NodeType.ADD, fusion.input_node(0), fusion.input_node(1)), ["b", "c"], "d",
        dtype=DType.FLOAT32).root), [b, c], [F16, BF16], [0, 0], F32, n).view(np.float32)
    assert np.array_equal(d.view(np.uint32), want_d.view(np.uint32))
    for t in list(ins.values()) + list(serial.values()):
        t.close()
    gb.close()
    k.close()


def test_pass_through_cast_copies_into_its_slot(backend):
    bf = T(DType.BFLOAT16, 4096)
    g = graph.Graph(nodes=[graph.GraphNode("same", graph.SHAPE_CAST, ["x"], {}, input_types=[bf], output_type=bf)],
                    inputs=["x"], outputs={"same": "same"})
    gb = graph.GraphBackend(backend)
    gb.attach_workspace("id", g)
    x = synthetic.normal_bf16(801, 4096)
    xt = backend.upload([4096], DType.BFLOAT16, x)
    out = gb.call_graph(graph.GraphCallRequest("id", g, {"x": xt})).outputs["same"]
    assert out.dispatch_pointer() != xt.dispatch_pointer() and gb.workspace("id").contains(out.dispatch_pointer())
    assert backend.download(out)[1] == x.tobytes()
    xt.close()
    gb.close()


def test_inputs_that_live_in_the_arena(backend, ref):
    """An output fed back as the next call's input: one that is exactly the input's slot
    needs no copy; one that straddles the slot is copied out before the slot is written."""
    from manifesto_b200._abi import call
    from manifesto_b200.backend import DeviceTensor, DeviceView
    n = 4096
    bf, hf = T(DType.BFLOAT16, n), T(DType.FLOAT16, n)
    g = graph.Graph(nodes=[
        graph.GraphNode("a", graph.SHAPE_CAST, ["x"], {"dtype": "F16"}, input_types=[bf], output_type=hf),
        graph.GraphNode("b", graph.SHAPE_CAST, ["a"], {"dtype": "BF16"}, input_types=[hf], output_type=bf),
    ], inputs=["x"], outputs={"b": "b"})
    gb = graph.GraphBackend(backend)
    topo = gb.attach_workspace("loop", g)
    ws = gb.workspace("loop")
    # a@0, x@2n, b reuses x's slot once x is dead; the arena is 4n bytes
    assert topo.input_ports == {"x": 2 * n} and topo.output_ports == {"b": 2 * n} and topo.workspace.size == 4 * n

    def round_trip(v):
        return ref.convert(ref.convert(v, BF16, F16).view(np.uint16), F16, BF16).view(np.uint16)

    x = synthetic.normal_bf16(901, n, 0.0, 50.0)
    xt = backend.upload([n], DType.BFLOAT16, x)
    out = gb.call_graph(graph.GraphCallRequest("loop", g, {"x": xt})).outputs["b"]
    assert out.dispatch_pointer() == ws.input_slots["x"].ptr
    want = round_trip(x)
    assert np.array_equal(host(backend, out, np.uint16), want)
    out = gb.call_graph(graph.GraphCallRequest("loop", g, {"x": out})).outputs["b"]   # its own slot
    want = round_trip(want)
    assert np.array_equal(host(backend, out, np.uint16), want)
    # the same values placed across a's slot and x's slot
    straddle = ws.base + 2 * n - 256
    call("mf_memcpy_d2d_async", straddle, xt.dispatch_pointer(), 2 * n, None)
    call("mf_stream_sync", None)
    view = DeviceTensor(backend, (n,), DType.BFLOAT16, DeviceView(straddle, 2 * n))
    out = gb.call_graph(graph.GraphCallRequest("loop", g, {"x": view})).outputs["b"]
    assert np.array_equal(host(backend, out, np.uint16), round_trip(x))
    xt.close()
    gb.close()
