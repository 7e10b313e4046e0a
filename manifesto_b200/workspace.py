"""The static workspace plan a graph runs in: one device allocation, one offset per port.

manifesto's compiler plans every lowered graph before the first dispatch
(compiler/plan.go:242-289 PlanGraph): it bridges the typed ast.Graph to an ir.Topology
whose producer and consumer share one Port per tensor (buildPlanningTopology,
compiler/plan.go:29-90), runs liveness analysis and an interval-colouring allocator
over the nodes in execution order (ir.PlanWorkspace, ir/planner.go:43-96), and records
each graph input's and output's byte offset (attachGraphIOPorts, compiler/plan.go:
179-228).  A backend that advertises runtime.WorkspaceAttacher
(runtime/executor.go:28-48) then allocates WorkspaceLayout.Size bytes once and
resolves every port to base + offset (runtime/orchestrator.go:180-217).

This module restates that planner so the plan can be made without the Go compiler, or
checked against it; GraphBackend.attach_workspace (graph.py) consumes it on the device.
The allocator's rules are kept exactly, because two implementations that disagree
about offsets cannot share a workspace: intervals sorted by (Start, PortID), sizes and
offsets rounded up to Align, a block evicted only once its End is strictly below the
new Start (touching lifetimes overlap), the lowest aligned gap that fits.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Iterable, Sequence

from .dtype import DType

DEFAULT_ALIGN = 64
# ops whose output is a view of their first input (compiler/plan.go:166-173)
ALIAS_OPS = ("shape.view_as_heads", "shape.merge_heads")


class PlanError(ValueError):
    """A planning failure (the Go planner's `error` returns)."""


@dataclass(frozen=True)
class Dimension:
    """ir.Dimension (ir/port_type.go:51-94): a named symbol, or a static size when symbol is ''."""
    symbol: str = ""
    static: int = 0

    def is_symbolic(self) -> bool:
        return self.symbol != ""


@dataclass(frozen=True)
class PortType:
    """ir.PortType (ir/port_type.go:21-27): the fields the planner reads (dtype, shape schema)."""
    dtype: DType = DType.INVALID
    dims: tuple[Dimension, ...] = ()


def port_type(dtype: DType, *dims: int | str) -> PortType:
    """A PortType from plain dims: an int is a static size, a str a symbol."""
    return PortType(DType(dtype), tuple(Dimension(symbol=d) if isinstance(d, str) else Dimension(static=int(d))
                                        for d in dims))


@dataclass
class PortAllocation:
    """ir.PortAllocation (ir/port_allocation.go:12-36) without stride formulas."""
    port_id: int
    base_offset: int
    port_type: PortType


class Port:
    """ir.Port (ir/port.go:20-38).  Compared by identity, like the Go pointer: a producer's
    output and its consumers' inputs are the same object."""
    __slots__ = ("id", "type", "allocation")

    def __init__(self, type: PortType | None = None, id: int = 0):
        self.id = id
        self.type = type if type is not None else PortType()
        self.allocation: PortAllocation | None = None

    def __repr__(self) -> str:
        return f"Port(id={self.id}, dtype={self.type.dtype.name})"


@dataclass
class Interval:
    """ir.Interval (ir/workspace.go:41-57): a port's lifetime [start, end] in execution steps,
    inclusive, and its place in the workspace."""
    port_id: int
    start: int
    end: int
    offset: int = 0
    size: int = 0

    def overlaps(self, other: "Interval") -> bool:
        """Interval.Overlaps (ir/workspace.go:63-73): inclusive ranges, touching ones overlap."""
        return not (self.end < other.start or other.end < self.start)


@dataclass
class WorkspaceLayout:
    """ir.WorkspaceLayout (ir/workspace.go:12-35)."""
    size: int = 0
    align: int = 0
    allocations: list[Interval] = field(default_factory=list)
    bindings: dict[str, int] = field(default_factory=dict)


@dataclass
class TopologyNode:
    """ir.Node: the fields the planner reads."""
    name: str
    op: str = ""
    inputs: list[Port | None] = field(default_factory=list)
    outputs: list[Port | None] = field(default_factory=list)


@dataclass
class Topology:
    """ir.Topology (ir/topology.go:17-40): nodes in execution order plus the planner output.
    input_ports / output_ports map graph input and output names to byte offsets."""
    nodes: list[TopologyNode] = field(default_factory=list)
    workspace: WorkspaceLayout = field(default_factory=WorkspaceLayout)
    input_ports: dict[str, int] = field(default_factory=dict)
    output_ports: dict[str, int] = field(default_factory=dict)


def is_power_of_two(value: int) -> bool:
    return value > 0 and value & (value - 1) == 0


def align_up(value: int, align: int) -> int:
    """alignUp (ir/planner.go:417-427)."""
    if align <= 1:
        return value
    if not is_power_of_two(align):
        raise PlanError(f"planner: alignUp requires power-of-two align, got {align}")
    return (value + align - 1) & ~(align - 1)


def _ports(node: TopologyNode) -> Iterable[Port]:
    for p in node.outputs:
        if p is not None:
            yield p
    for p in node.inputs:
        if p is not None:
            yield p


def assign_port_ids(topology: Topology) -> None:
    """AssignPortIDs (ir/planner.go:107-168): outputs then inputs of each node in order; a port
    that has an ID keeps it, the others take sequential IDs after the largest one seen."""
    next_id = 1
    seen: set[int] = set()
    for node in topology.nodes:
        for p in _ports(node):
            if id(p) in seen:
                continue
            seen.add(id(p))
            if p.id >= next_id:
                next_id = p.id + 1
    seen.clear()
    for node in topology.nodes:
        for p in _ports(node):
            if id(p) in seen:
                continue
            seen.add(id(p))
            if p.id == 0:
                p.id = next_id
                next_id += 1


def resolve_dims(dims: Sequence[Dimension], bindings: dict[str, int]) -> list[int]:
    """The concrete shape of a dims schema under `bindings` (the sizing loop of PortByteSize)."""
    out = []
    for i, d in enumerate(dims):
        if not d.is_symbolic():
            out.append(int(d.static))
            continue
        if d.symbol not in bindings:
            raise PlanError(f"dim[{i}] symbol \"{d.symbol}\" is unbound (run unifier first to populate bindings)")
        out.append(int(bindings[d.symbol]))
    return out


def port_byte_size(port: Port | None, bindings: dict[str, int]) -> int:
    """PortByteSize (ir/planner.go:437-480): a 0-d port holds one element; symbols resolve
    through `bindings`; the dtype's BytesFor packs Int4 and Bool."""
    if port is None:
        raise PlanError("port is nil")
    dt = port.type.dtype
    if not port.type.dims:
        try:
            return dt.bytes_for(1)
        except ValueError as e:
            raise PlanError(f"dtype {dt.name} rejected scalar size: {e}") from None
    count = 1
    for n in resolve_dims(port.type.dims, bindings):
        count *= n
    try:
        return dt.bytes_for(count)
    except ValueError as e:
        raise PlanError(f"dtype {dt.name} rejected {count} elements: {e}") from None


def analyze_liveness(nodes: Sequence[TopologyNode], bindings: dict[str, int]) -> list[Interval]:
    """AnalyzeLiveness (ir/planner.go:186-283): one interval per distinct port, from the step of
    its producer (or 0 for a port nothing produces: graph inputs, weights) to the step of
    its last consumer, sorted by (start, port ID)."""
    intervals: dict[int, Interval] = {}

    def size_of(p: Port, what: str) -> int:
        try:
            return port_byte_size(p, bindings)
        except PlanError as e:
            raise PlanError(f"port id={p.id}{what}: {e}") from None

    for step, node in enumerate(nodes):
        if node is None:
            continue
        for p in node.outputs:
            if p is None or p.id == 0 or p.id in intervals:
                continue
            intervals[p.id] = Interval(p.id, step, step, size=size_of(p, ""))
        for p in node.inputs:
            if p is None or p.id == 0:
                continue
            iv = intervals.get(p.id)
            if iv is None:
                intervals[p.id] = Interval(p.id, 0, step, size=size_of(p, " (unproduced input)"))
            elif step > iv.end:
                iv.end = step
    return sorted(intervals.values(), key=lambda iv: (iv.start, iv.port_id))


def _lowest_offset(size: int, live: list[tuple[int, int, int]], align: int) -> int:
    """chooseLowestNonConflictingOffset (ir/planner.go:376-411): scan the live blocks by offset;
    on an overlap move past that block (aligned) and rescan from the first."""
    blocks = sorted(live, key=lambda b: b[0])
    candidate = 0
    while True:
        for off, sz, _ in blocks:
            if candidate >= off + sz or candidate + size <= off:
                continue
            candidate = align_up(off + sz, align)
            break
        else:
            return candidate


def allocate_offsets(intervals: Sequence[Interval], align: int) -> tuple[int, list[Interval]]:
    """AllocateOffsets (ir/planner.go:296-350): interval colouring.  Returns the aligned high
    water mark and copies of the intervals (sorted) with offset and rounded size set."""
    if align <= 0:
        align = DEFAULT_ALIGN
    if not intervals:
        return 0, []
    work = sorted((Interval(iv.port_id, iv.start, iv.end, iv.offset, iv.size) for iv in intervals),
                  key=lambda iv: (iv.start, iv.port_id))
    live: list[tuple[int, int, int]] = []   # (offset, size, end)
    high = 0
    for iv in work:
        iv.size = align_up(iv.size, align)
        live = [b for b in live if b[2] >= iv.start]
        iv.offset = _lowest_offset(iv.size, live, align)
        live.append((iv.offset, iv.size, iv.end))
        high = max(high, iv.offset + iv.size)
    return align_up(high, align), work


def plan_workspace(topology: Topology, bindings: dict[str, int] | None = None, align: int = 0) -> None:
    """PlanWorkspace (ir/planner.go:43-96): IDs, liveness, offsets; fills topology.workspace and
    every port's allocation in place.  align <= 0 means 64; it must be a power of two."""
    if topology is None:
        raise PlanError("planner: topology is required")
    if align <= 0:
        align = DEFAULT_ALIGN
    if not is_power_of_two(align):
        raise PlanError(f"planner: Align={align} must be a power of two")
    bindings = dict(bindings or {})
    assign_port_ids(topology)
    total, allocated = allocate_offsets(analyze_liveness(topology.nodes, bindings), align)
    topology.workspace = WorkspaceLayout(total, align, allocated, dict(bindings))
    by_id = {iv.port_id: iv for iv in allocated}
    seen: set[int] = set()
    for node in topology.nodes:     # attachAllocationsToPorts (ir/planner.go:482-513)
        for p in _ports(node):
            if id(p) in seen:
                continue
            seen.add(id(p))
            iv = by_id.get(p.id)
            if iv is not None:
                p.allocation = PortAllocation(p.id, iv.offset, p.type)


# ------------------------------------------------------------ graph bridge

@dataclass
class PlanningBridge:
    """planningBridge (compiler/plan.go:18-22)."""
    topology: Topology
    boundary_ports: dict[str, Port]
    producer_ports: dict[str, Port]


def build_planning_topology(graph) -> PlanningBridge:
    """buildPlanningTopology (compiler/plan.go:29-90) over graph.Graph: one node per graph
    node with a single output port; an input slot takes its producer's output port, or
    the graph input's boundary port, which takes the first consumer's input type; alias
    ops (shape.view_as_heads, shape.merge_heads) output their input port."""
    topo = Topology()
    producers: dict[str, Port] = {}
    boundary = {name: Port() for name in graph.inputs if name}
    for node in graph.nodes:
        if node is None:
            continue
        tn = TopologyNode(node.id, node.op, [None] * len(node.inputs))
        for slot, ref in enumerate(node.inputs):
            p = producers.get(ref)
            if p is None:
                p = boundary.get(ref)
                if p is None:
                    raise PlanError(f"compiler: node \"{node.id}\" input \"{ref}\": producer \"{ref}\" is not defined "
                                    f"before consumer (run NormalizeGraph)")
                if p.type.dtype == DType.INVALID and slot < len(node.input_types):
                    p.type = node.input_types[slot]
            tn.inputs[slot] = p
        if node.op in ALIAS_OPS and tn.inputs and tn.inputs[0] is not None:
            out = tn.inputs[0]
        else:
            out = Port(node.output_type if node.output_type is not None else PortType())
        tn.outputs = [out]
        producers[node.id] = out
        topo.nodes.append(tn)
    return PlanningBridge(topo, boundary, producers)


def plan_graph(graph, bindings: dict[str, int] | None = None, align: int = 0) -> Topology:
    """PlanGraph (compiler/plan.go:242-289) without NormalizeGraph and stream scheduling: the
    graph's nodes must already be in execution order (graph.schedule_streams assigns
    streams).  Bindings default to the graph's own (the typer's SymbolMap)."""
    if graph is None:
        raise PlanError("compiler: graph is required")
    bridge = build_planning_topology(graph)
    if bindings is None:
        bindings = getattr(graph, "bindings", None) or {}
    try:
        plan_workspace(bridge.topology, bindings, align if align > 0 else DEFAULT_ALIGN)
    except PlanError as e:
        raise PlanError(f"compiler: plan workspace: {e}") from None
    topo = bridge.topology
    for name in graph.inputs:       # attachGraphIOPorts (compiler/plan.go:179-228)
        if not name:
            continue
        p = bridge.boundary_ports.get(name)
        if p is None or p.allocation is None:
            raise PlanError(f"compiler: plan graph: compiler: graph input \"{name}\" has no workspace allocation")
        topo.input_ports[name] = p.allocation.base_offset
    for name, producer in graph.outputs.items():
        if not name:
            continue
        p = bridge.producer_ports.get(producer)
        if p is None or p.allocation is None:
            raise PlanError(f"compiler: plan graph: compiler: graph output \"{name}\" producer \"{producer}\" has no "
                            f"workspace allocation")
        topo.output_ports[name] = p.allocation.base_offset
    return topo
