"""The workspace planner restatement (ir/planner.go, ir/workspace.go, compiler/plan.go) against
the reference's own planner tests (ir/planner_test.go, ir/workspace_test.go,
compiler/plan_test.go), plus exact offsets for the cases the device path relies on."""
import pytest

from manifesto_b200 import workspace as wsp
from manifesto_b200.dtype import DType
from manifesto_b200.graph import Graph, GraphNode, plan_hazards

F32 = DType.FLOAT32


def linear_topology(ports: int):
    """makeLinearTopology (ir/planner_test.go:22-40): ports F32 [64, 64]; node i reads port i
    and writes port i+1."""
    ps = [wsp.Port(wsp.port_type(F32, 64, 64)) for _ in range(ports)]
    topo = wsp.Topology([wsp.TopologyNode("step", "", [ps[i]], [ps[i + 1]]) for i in range(ports - 1)])
    return topo, ps


def interval(ivs, pid):
    return next((iv for iv in ivs if iv.port_id == pid), None)


# ---- ir/planner_test.go ----------------------------------------------------

def test_assign_port_ids_unique_and_idempotent():
    topo, ps = linear_topology(4)
    wsp.assign_port_ids(topo)
    ids = [p.id for p in ps]
    assert 0 not in ids and len(set(ids)) == 4
    wsp.assign_port_ids(topo)
    assert [p.id for p in ps] == ids


def test_assign_port_ids_keeps_existing_and_continues_after_them():
    topo, ps = linear_topology(3)
    ps[1].id = 7
    wsp.assign_port_ids(topo)
    # node 0: output ps[1] (7), then input ps[0]; node 1: output ps[2]
    assert (ps[1].id, ps[0].id, ps[2].id) == (7, 8, 9)


def test_liveness_linear_chain():
    topo, ps = linear_topology(4)
    wsp.assign_port_ids(topo)
    ivs = wsp.analyze_liveness(topo.nodes, {})
    assert len(ivs) == 4
    p0, p1 = interval(ivs, ps[0].id), interval(ivs, ps[1].id)
    assert (p0.start, p0.end) == (0, 0)       # unproduced input
    assert (p1.start, p1.end) == (0, 1)
    assert all(iv.size == 64 * 64 * 4 for iv in ivs)


def test_liveness_multi_consumer():
    t = wsp.port_type(F32, 32, 32)
    inp, shared, o1, o2 = (wsp.Port(t) for _ in range(4))
    topo = wsp.Topology([wsp.TopologyNode("produce", "", [inp], [shared]),
                         wsp.TopologyNode("consume1", "", [shared], [o1]),
                         wsp.TopologyNode("consume2", "", [shared], [o2])])
    wsp.assign_port_ids(topo)
    iv = interval(wsp.analyze_liveness(topo.nodes, {}), shared.id)
    assert (iv.start, iv.end) == (0, 2)


def test_liveness_rejects_unbound_symbol():
    p = wsp.Port(wsp.port_type(F32, "B", 768))
    topo = wsp.Topology([wsp.TopologyNode("use", "", [p], [])])
    wsp.assign_port_ids(topo)
    with pytest.raises(wsp.PlanError) as e:
        wsp.analyze_liveness(topo.nodes, {})
    assert "unbound" in str(e.value) and "B" in str(e.value)
    assert str(e.value) == ('port id=1 (unproduced input): dim[0] symbol "B" is unbound '
                            '(run unifier first to populate bindings)')


def test_liveness_resolves_bound_symbols():
    p = wsp.Port(wsp.port_type(F32, "B", 768))
    topo = wsp.Topology([wsp.TopologyNode("use", "", [p], [])])
    wsp.assign_port_ids(topo)
    ivs = wsp.analyze_liveness(topo.nodes, {"B": 4})
    assert len(ivs) == 1 and ivs[0].size == 4 * 768 * 4


def test_allocate_disjoint_intervals_share_offset():
    total, out = wsp.allocate_offsets([wsp.Interval(1, 0, 2, size=128), wsp.Interval(2, 3, 5, size=128)], 64)
    assert out[0].offset == out[1].offset and total == 128


def test_allocate_overlapping_intervals_get_distinct_offsets():
    total, out = wsp.allocate_offsets([wsp.Interval(1, 0, 5, size=128), wsp.Interval(2, 3, 7, size=128)], 64)
    by = {iv.port_id: iv for iv in out}
    assert by[1].offset != by[2].offset and total == 256


def test_allocate_rounds_to_alignment():
    total, out = wsp.allocate_offsets([wsp.Interval(1, 0, 5, size=17), wsp.Interval(2, 3, 7, size=17)], 64)
    assert all(iv.size == 64 and iv.offset % 64 == 0 for iv in out) and total == 128


def test_plan_workspace_linear_topology():
    topo, ps = linear_topology(4)
    wsp.plan_workspace(topo, {}, 64)
    assert topo.workspace.size > 0 and topo.workspace.align == 64 and len(topo.workspace.allocations) == 4
    for p in ps:
        assert p.allocation is not None and p.allocation.port_id == p.id and p.allocation.base_offset % 64 == 0


def test_plan_workspace_alignment_default_and_power_of_two():
    topo, _ = linear_topology(2)
    wsp.plan_workspace(topo)
    assert topo.workspace.align == 64
    topo, _ = linear_topology(2)
    with pytest.raises(wsp.PlanError, match="power of two"):
        wsp.plan_workspace(topo, align=48)


def test_port_byte_size():
    assert wsp.port_byte_size(wsp.Port(wsp.PortType(F32)), {}) == 4          # 0-d: one element
    assert wsp.port_byte_size(wsp.Port(wsp.port_type(DType.INT4, 3, 5)), {}) == 8   # BytesFor packs Int4
    assert wsp.port_byte_size(wsp.Port(wsp.port_type(DType.BOOL, 9)), {}) == 2
    with pytest.raises(wsp.PlanError, match="rejected scalar size"):
        wsp.port_byte_size(wsp.Port(wsp.PortType()), {})                       # DType Invalid
    with pytest.raises(wsp.PlanError, match="port is nil"):
        wsp.port_byte_size(None, {})


# ---- ir/workspace_test.go --------------------------------------------------

def test_interval_overlaps_symmetric():
    cases = [((0, 3), (4, 7), False), ((0, 3), (3, 7), True), ((0, 10), (2, 5), True), ((0, 5), (3, 7), True)]
    for (a0, a1), (b0, b1), want in cases:
        a, b = wsp.Interval(0, a0, a1), wsp.Interval(0, b0, b1)
        assert a.overlaps(b) == want and b.overlaps(a) == want


# ---- compiler/plan_test.go -------------------------------------------------

def chain(n: int, t: wsp.PortType, op: str = "noop") -> Graph:
    nodes, prev = [], "x"
    for i in range(1, n + 1):
        nodes.append(GraphNode(f"n{i}", op, [prev], input_types=[t], output_type=t))
        prev = f"n{i}"
    return Graph(nodes, ["x"])


def test_bridge_shares_producer_consumer_ports():
    t = wsp.port_type(F32, 4, 4)
    topo = wsp.build_planning_topology(chain(3, t)).topology
    assert len(topo.nodes) == 3
    assert topo.nodes[1].inputs[0] is topo.nodes[0].outputs[0]
    assert topo.nodes[2].inputs[0] is topo.nodes[1].outputs[0]
    boundary = topo.nodes[0].inputs[0]
    assert boundary.type.dtype == F32 and boundary.type.dims == (wsp.Dimension(static=4), wsp.Dimension(static=4))
    assert all(n.outputs[0].type.dtype == F32 for n in topo.nodes)


@pytest.mark.parametrize("op", wsp.ALIAS_OPS)
def test_bridge_aliases_reshape_ports(op):
    flat, heads = wsp.port_type(F32, 4, 8), wsp.port_type(F32, 4, 2, 4)
    src, dst = (flat, heads) if op == "shape.view_as_heads" else (heads, flat)
    g = Graph([GraphNode("produce", "linear", ["x"], input_types=[src], output_type=src),
               GraphNode("reshape", op, ["produce"], input_types=[src], output_type=dst),
               GraphNode("consume", "rope", ["reshape"], input_types=[dst], output_type=dst)], ["x"])
    topo = wsp.build_planning_topology(g).topology
    prod = topo.nodes[0].outputs[0]
    assert topo.nodes[1].inputs[0] is prod and topo.nodes[1].outputs[0] is prod and topo.nodes[2].inputs[0] is prod
    wsp.assign_port_ids(topo)
    iv = interval(wsp.analyze_liveness(topo.nodes, {}), prod.id)
    assert (iv.start, iv.end) == (0, 2)


def test_plan_graph_non_overlapping_offsets():
    g = chain(2, wsp.port_type(F32, 4, 4))
    topo = wsp.plan_graph(g)
    assert topo.workspace.size >= 64 and topo.workspace.size % 64 == 0
    assert all(n.outputs[0].allocation.base_offset % 64 == 0 for n in topo.nodes)
    assert all(iv.size >= 64 for iv in topo.workspace.allocations)


def test_plan_graph_reuses_offsets_when_lifetimes_do_not_overlap():
    topo = wsp.plan_graph(chain(3, wsp.port_type(F32, 8, 8)))
    assert topo.workspace.size <= 512
    assert len({iv.offset for iv in topo.workspace.allocations}) <= 2


def test_plan_graph_symbol_bindings():
    t = wsp.port_type(F32, "B", 16)
    g = chain(1, t)
    g.bindings = {"B": 4}
    assert wsp.plan_graph(g).workspace.size >= 256
    g.bindings = {}
    with pytest.raises(wsp.PlanError) as e:
        wsp.plan_graph(g)
    assert "unbound" in str(e.value) and "B" in str(e.value)


def test_plan_graph_unknown_producer_and_unplanned_output():
    t = wsp.port_type(F32, 4)
    with pytest.raises(wsp.PlanError, match="is not defined before consumer"):
        wsp.plan_graph(Graph([GraphNode("n1", "noop", ["y"], input_types=[t], output_type=t)], ["x"]))
    g = chain(1, t)
    g.outputs = {"out": "nope"}
    with pytest.raises(wsp.PlanError, match="has no workspace allocation"):
        wsp.plan_graph(g)


# ---- exact offsets and the hazards the device path handles ------------------

def test_exact_offsets_of_an_equal_size_chain_and_its_hazards():
    """x -> a -> b -> c, every tensor 64 bytes.  IDs: a.out 1, x 2, b.out 3, c.out 4.
    a@0, x@64 (live with a), b@64 (x dead after step 0), c@0 (a dead after step 1):
    c overwrites a graph output, so a must be snapshotted; b waits for x's reader
    (node 0), c for a's writer and reader (nodes 0, 1)."""
    t = wsp.port_type(F32, 4, 4)
    g = chain(3, t)
    g.outputs = {"a_out": "n1", "c_out": "n3"}
    topo = wsp.plan_graph(g)
    offs = [n.outputs[0].allocation.base_offset for n in topo.nodes]
    assert offs == [0, 64, 0] and topo.input_ports == {"x": 64} and topo.workspace.size == 128
    assert topo.output_ports == {"a_out": 0, "c_out": 0}
    deps, snap = plan_hazards(g, topo)
    assert deps == [(), (0,), (0, 1)] and snap == {0}
    g.outputs = {"c_out": "n3"}
    assert plan_hazards(g, topo)[1] == set()


def test_lowest_gap_is_reused():
    """A[0,5] 128 B @0, B[0,1] 64 B @128, C[0,5] 64 B @192; D[2,3] 64 B fits B's gap @128;
    E[2,3] 128 B fits no gap and goes on top @256."""
    ivs = [wsp.Interval(1, 0, 5, size=128), wsp.Interval(2, 0, 1, size=64), wsp.Interval(3, 0, 5, size=64),
           wsp.Interval(4, 2, 3, size=64), wsp.Interval(5, 2, 3, size=100)]
    total, out = wsp.allocate_offsets(ivs, 64)
    assert [iv.offset for iv in out] == [0, 128, 192, 128, 256] and total == 384
    assert [iv.size for iv in out] == [128, 64, 64, 64, 128]


def test_diamond_hazards_under_a_stream_schedule():
    """a = f(x); b, c = g(a), h(a); d = k(b, c); e = m(y) with N-element F32/F16/BF16/E4M3 ports.
    e's output is given a's bytes (and d's): e runs on its own stream, so it must wait for
    every node that touched them; d is a graph output that e overwrites."""
    from manifesto_b200.graph import schedule_streams
    n = 1024
    f32, f16, bf, q = (wsp.port_type(d, n) for d in (F32, DType.FLOAT16, DType.BFLOAT16, DType.FLOAT8_E4M3))
    g = Graph([GraphNode("a", "shape.cast", ["x"], input_types=[bf], output_type=f32),
               GraphNode("b", "shape.cast", ["a"], input_types=[f32], output_type=f16),
               GraphNode("c", "shape.cast", ["a"], input_types=[f32], output_type=bf),
               GraphNode("d", "optimizer.fusion", ["b", "c"], input_types=[f16, bf], output_type=f32),
               GraphNode("e", "shape.cast", ["y"], input_types=[bf], output_type=q)],
              ["x", "y"], {"d": "d", "e": "e"})
    topo = wsp.plan_graph(g)
    offs = [nd.outputs[0].allocation.base_offset for nd in topo.nodes]
    # a@0 (4N), x@4N, y@6N, b@4N (x dead), c@8N, d@0 (a dead), e@0 (b, c, d dead)
    assert offs == [0, 4 * n, 8 * n, 0, 0] and topo.input_ports == {"x": 4 * n, "y": 6 * n}
    deps, snap = plan_hazards(g, topo)
    assert deps == [(), (0,), (), (0, 1, 2), (0, 1, 2, 3)] and snap == {3}
    assert [schedule_streams(g)[i].stream_id for i in "abcde"] == [0, 0, 1, 0, 2]
