"""graph.call on the GPU: typer-inserted shape.cast adaptors around a fused SwiGLU node."""
import numpy as np
import pytest

from manifesto_b200 import fusion, graph, synthetic
from manifesto_b200.dtype import DType
from oracle.ref import BF16, E4M3, F16, F32

from .conftest import host_threads
from .test_gpu_fused_quant import ulp_diff_16

pytestmark = pytest.mark.gpu


def test_graph_call_casts_and_fusion(backend, ref):
    rows, hidden = 32, 4096
    n = rows * hidden
    x = synthetic.normal_bf16(301, n)
    gam = synthetic.normal_bf16(302, hidden, 1.0, 0.1)
    bet = synthetic.normal_bf16(303, hidden, 0.0, 0.1)
    y16 = synthetic.normal_f32(304, n).astype(np.float16).view(np.uint16)  # producer emits F16

    f = fusion.swiglu_chain()
    k = fusion.emit_cuda(f, in_dtypes=[DType.BFLOAT16] * 4, in_bcast=[0, hidden, hidden, 0], out_dtype=DType.BFLOAT16)
    g = graph.Graph(nodes=[
        # what typer.buildAdaptorNode inserts for the F16 -> BF16 edge into the fused node's slot 3
        graph.GraphNode("adaptor_cast_h_3", graph.SHAPE_CAST, ["y"],
                        {"dtype": DType.BFLOAT16, "from_dtype": DType.FLOAT16},
                        {"synthesized_for_edge": "dtype F16 != BF16"}),
        graph.GraphNode("h", graph.FUSE_OP, ["x", "gamma", "beta", "adaptor_cast_h_3"],
                        {graph.FUSE_ATTRIBUTE_AST: f, graph.KERNEL_ATTRIBUTE: graph.KernelSet([k])}),
        graph.GraphNode("h_f32", graph.SHAPE_CAST, ["h"], {"dtype": "F32"}),
        graph.GraphNode("h_q", graph.SHAPE_CAST, ["h"], {"dtype": "F8_E4M3", "from_dtype": "BF16"}),
    ], inputs=["x", "gamma", "beta", "y"], outputs={"h": "h", "h_f32": "h_f32", "h_q": "h_q"},
        execution_dtype=DType.BFLOAT16)
    ins = {"x": backend.upload([rows, hidden], DType.BFLOAT16, x), "gamma": backend.upload([hidden], DType.BFLOAT16, gam),
           "beta": backend.upload([hidden], DType.BFLOAT16, bet), "y": backend.upload([rows, hidden], DType.FLOAT16, y16)}
    res = graph.GraphBackend(backend).call_graph(graph.GraphCallRequest("block", g, ins))
    out = res.outputs
    assert out["h"].shape() == (rows, hidden) and out["h"].dtype() == DType.BFLOAT16
    assert out["h_f32"].dtype() == DType.FLOAT32 and out["h_q"].dtype() == DType.FLOAT8_E4M3

    y_bf16 = ref.convert(y16, F16, BF16).view(np.uint16)
    want_h = ref.fused_eval(fusion.node_table(f.root), [x, gam, bet, y_bf16], [BF16] * 4, [0, hidden, hidden, 0],
                            BF16, n, threads=host_threads())
    got_h = np.frombuffer(backend.download(out["h"])[1], np.uint16)
    assert ulp_diff_16(got_h, want_h).max() <= 1
    # the casts of the device's own fused output are bit-exact
    got_f32 = np.frombuffer(backend.download(out["h_f32"])[1], np.uint32)
    assert np.array_equal(got_f32, ref.convert(got_h, BF16, F32).view(np.uint32))
    got_q = np.frombuffer(backend.download(out["h_q"])[1], np.uint8)
    assert np.array_equal(got_q, ref.convert(got_h, BF16, E4M3))
    for t in list(ins.values()) + list(out.values()):
        t.close()
    k.close()


def test_scheduled_streams_match_serial(backend, ref):
    """A diamond plus an independent branch, run on the streams schedule_streams assigns
    (events between them), gives the same bytes as the serial run and as the oracle."""
    n = 1 << 20
    x = synthetic.normal_bf16(401, n)
    y = synthetic.normal_bf16(402, n, 0.0, 30.0)
    add = fusion.FusionAST(fusion.binary(fusion.NodeType.ADD, fusion.input_node(0), fusion.input_node(1)),
                           ["b", "c"], "d", dtype=DType.FLOAT32)
    k = fusion.emit_cuda(add, in_dtypes=[DType.FLOAT16, DType.BFLOAT16], out_dtype=DType.FLOAT32)
    g = graph.Graph(nodes=[
        graph.GraphNode("a", graph.SHAPE_CAST, ["x"], {"dtype": "F32"}),
        graph.GraphNode("b", graph.SHAPE_CAST, ["a"], {"dtype": "F16"}),
        graph.GraphNode("c", graph.SHAPE_CAST, ["a"], {"dtype": "BF16"}),
        graph.GraphNode("d", graph.FUSE_OP, ["b", "c"], {graph.KERNEL_ATTRIBUTE: graph.KernelSet([k])}),
        graph.GraphNode("e", graph.SHAPE_CAST, ["y"], {"dtype": "F8_E4M3"}),
    ], inputs=["x", "y"], outputs={"d": "d", "e": "e"})
    sched = graph.schedule_streams(g)
    assert [sched[i].stream_id for i in "abcde"] == [0, 0, 1, 0, 2]
    ins = {"x": backend.upload([n], DType.BFLOAT16, x), "y": backend.upload([n], DType.BFLOAT16, y)}
    gb = graph.GraphBackend(backend)
    par = gb.call_graph(graph.GraphCallRequest("diamond", g, ins), schedule=sched).outputs
    ser = gb.call_graph(graph.GraphCallRequest("diamond", g, ins)).outputs
    for name in ("d", "e"):
        assert backend.download(par[name])[1] == backend.download(ser[name])[1]
    a = ref.convert(x, BF16, F32)
    b = ref.convert(a, F32, F16).view(np.uint16)
    c = ref.convert(a, F32, BF16).view(np.uint16)
    want_d = ref.fused_eval(fusion.node_table(add.root), [b, c], [F16, BF16], [0, 0], F32, n, threads=host_threads())
    assert backend.download(par["d"])[1] == want_d.tobytes()
    assert backend.download(par["e"])[1] == ref.convert(y, BF16, E4M3).tobytes()
    for t in list(ins.values()) + list(par.values()) + list(ser.values()):
        t.close()
    k.close()
