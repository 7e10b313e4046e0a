"""graph.call on the GPU for the nodes of the conversion path.

manifesto's runtime hands every graph.call to its Backend (runtime.Backend.CallGraph,
runtime/executor.go:22-27,53-72); the backend walks the lowered graph (ast.Graph /
ast.GraphNode, ast/graph.go:17-44) and runs each node.  GraphBackend.call_graph does
that on the device for the two node kinds this path owns:

* ``shape.cast`` -- the adaptor the typer inserts on a dtype mismatch
  (typer/adaptor.go:111-130; contract asset/template/operation/shape/cast.yml):
  one input, the same shape, storage dtype ``Attributes["dtype"]``.  The target is a
  dtype value (what the typer writes) or a dtype name (what a hand-written node's
  config holds, parsed like dtype.Parse); with none, the node passes its input
  through (typer/deriver_adaptor.go:13-29).  ``Attributes["from_dtype"]``, when
  present, must name the input's dtype.  Runs mf_convert (reference rounding).
* ``optimizer.fusion`` -- a FuseOp node (optimizer/fuse.go:16-22,113-127) whose
  ``compiled_kernel`` attribute (codegen/codegen.go:28) is a KernelSet with a CUDA
  kernel; runs it over the inputs in the node's input order.

Every other op is refused with MFError (MF_ERR_INVALID_ARGUMENT).  Values are device
tensors keyed by graph input name or node ID; ``Graph.outputs`` maps output names to
node IDs.  Nodes run in list order (the lowered graph is topologically sorted);
intermediate tensors no output refers to are freed when the call returns.

Multi-stream execution: given a stream schedule (ir.ScheduleStreams output,
ir/stream_scheduler.go:56-141 -- each node's StreamID and SyncBarriers), every
StreamID maps to a CUDA stream and every EventID to a CUDA event, both resolved into
flat tables before the first dispatch; a node waits (cudaStreamWaitEvent) on its Wait
barriers, runs on its stream, then records (cudaEventRecord) its signal barriers.
schedule_streams restates the scheduler over this module's Graph (edges are input
names produced by earlier nodes) so a schedule can be made without the Go compiler.

Workspace: GraphBackend.attach_workspace is runtime.WorkspaceAttacher.AttachWorkspace
(runtime/executor.go:28-48, called once per graph by runtime/orchestrator.go:193-217).
It takes the planner's ir.Topology (workspace.plan_graph restates the planner, from the
nodes' input_types / output_type and the graph's bindings), makes one device allocation
of WorkspaceLayout.Size bytes and resolves every port to base + offset.  A call of that
graph then copies its inputs into their slots and has every node write its own slot: no
allocation per node or per call.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Sequence

from . import workspace as wsp
from ._abi import call
from .backend import CUDABackend, DeviceBuffer, DeviceTensor, DeviceView, convert_raw, stream_handle
from .dtype import DECODE_SOURCES, DType, parse
from .errors import DTypeMismatch, DTypeUnsupported, InvalidArgument, ShapeMismatch
from .fusion import CUDAKernel, Target

SHAPE_CAST = "shape.cast"
FUSE_OP = "optimizer.fusion"            # optimizer.FuseOp
FUSE_ATTRIBUTE_AST = "fusion_ast"       # optimizer.FuseAttributeAST
KERNEL_ATTRIBUTE = "compiled_kernel"    # codegen.KernelAttribute


@dataclass
class GraphNode:
    """ast.GraphNode: the fields a backend reads."""
    id: str
    op: str
    inputs: list[str] = field(default_factory=list)
    attributes: dict[str, Any] = field(default_factory=dict)
    metadata: dict[str, Any] = field(default_factory=dict)
    input_types: list[wsp.PortType] = field(default_factory=list)   # set by the typer; read by the planner
    output_type: wsp.PortType | None = None


@dataclass
class Graph:
    """ast.Graph: nodes in topological order, input names, output name -> node ID."""
    nodes: list[GraphNode]
    inputs: list[str] = field(default_factory=list)
    outputs: dict[str, str] = field(default_factory=dict)
    execution_dtype: DType = DType.FLOAT32
    bindings: dict[str, int] = field(default_factory=dict)   # the typer's SymbolMap


@dataclass
class GraphCallRequest:
    """runtime.GraphCallRequest: the fields this backend uses."""
    graph_name: str
    graph: Graph
    inputs: dict[str, DeviceTensor]
    launch_bindings: dict[str, int] = field(default_factory=dict)


@dataclass
class GraphCallResult:
    outputs: dict[str, DeviceTensor]


@dataclass(frozen=True)
class SyncEvent:
    """ir.SyncEvent (ir/sync_event.go:14-26): wait before / signal after a node's dispatch."""
    event_id: int
    stream_id: int
    wait: bool


@dataclass
class NodeSchedule:
    """The scheduler's per-node output: ir.Node.StreamID and SyncBarriers (ir/node.go:43-51)."""
    stream_id: int = 0
    barriers: list[SyncEvent] = field(default_factory=list)


def schedule_streams(g: "Graph", max_streams: int = 0) -> dict[str, NodeSchedule]:
    """ir.ScheduleStreams (ir/stream_scheduler.go:56-141) and its pickStream rule (:229-287)
    over a Graph: a node continues its single predecessor stream when it is the next node
    of that stream's chain, a merge takes the lowest predecessor stream, anything else
    opens a new stream while fewer than max_streams exist (<= 0: one per node).  A
    predecessor on another stream gives the node a Wait barrier and the predecessor a
    signal with the same event ID."""
    cap = max_streams if max_streams >= 1 else len(g.nodes)
    producer = {}
    for i, n in enumerate(g.nodes):
        producer.setdefault(n.id, i)
    ids = {n.id: i + 1 for i, n in enumerate(g.nodes)}   # node.ID = index + 1
    out = {n.id: NodeSchedule() for n in g.nodes}
    last_on_stream: dict[int, int] = {}
    next_stream, next_event = 0, 1
    for i, n in enumerate(g.nodes):
        preds: dict[int, int] = {}   # stream -> most recent producer node ID
        for ref in n.inputs:
            j = producer.get(ref)
            if j is None or j >= i:
                continue
            p = g.nodes[j]
            st = out[p.id].stream_id
            if st not in preds or ids[p.id] > preds[st]:
                preds[st] = ids[p.id]
        if not preds:
            if next_stream < cap:
                assigned, next_stream = next_stream, next_stream + 1
            else:
                assigned = 0
        elif len(preds) == 1:
            (only, pred_id), = preds.items()
            if last_on_stream.get(only) == pred_id:
                assigned = only
            elif next_stream < cap:
                assigned, next_stream = next_stream, next_stream + 1
            else:
                assigned = only
        else:
            assigned = min(preds)
        out[n.id].stream_id = assigned
        last_on_stream[assigned] = ids[n.id]
        for st, pred_id in preds.items():
            if st == assigned:
                continue
            out[n.id].barriers.append(SyncEvent(next_event, st, True))
            out[g.nodes[pred_id - 1].id].barriers.append(SyncEvent(next_event, st, False))
            next_event += 1
    return out


class KernelSet:
    """codegen.KernelSet (codegen/attach.go:14-60): emitted kernels keyed by target."""

    def __init__(self, kernels: Sequence[Any] = ()):
        self._kernels = {k.target(): k for k in kernels}

    def for_target(self, target: Target):
        return self._kernels.get(target)

    def targets(self) -> list[Target]:
        return list(self._kernels)


def cast_target(node: GraphNode, input_dtype: DType) -> DType:
    """The output dtype of a shape.cast node (deriveCastOutput, typer/deriver_adaptor.go:13-29)."""
    raw = node.attributes.get("dtype")
    if raw is None or raw == "":
        return DType(input_dtype)
    if isinstance(raw, str):
        try:
            target = parse(raw)
        except ValueError as e:
            raise InvalidArgument(f"shape.cast {node.id!r}: {e}") from None
    else:
        target = DType(int(raw))
    return DType(input_dtype) if target == DType.INVALID else target


def _dtype_attr(node: GraphNode, key: str) -> DType | None:
    raw = node.attributes.get(key)
    if raw is None or raw == "":
        return None
    return parse(raw) if isinstance(raw, str) else DType(int(raw))


# ---------------------------------------------------------------- workspace

@dataclass
class _Slot:
    """A port's place in an attached workspace."""
    ptr: int
    dtype: DType
    dims: tuple
    capacity: int       # bytes the plan reserved: the port's size at the plan's bindings

    def resolve(self, bindings: dict[str, int], what: str) -> tuple[tuple[int, ...], int]:
        try:
            shape = tuple(wsp.resolve_dims(self.dims, bindings))
        except wsp.PlanError as e:
            raise InvalidArgument(f"{what}: {e}") from None
        count = 1
        for d in shape:
            count *= d
        nbytes = self.dtype.bytes_for(count)
        if nbytes > self.capacity:
            raise ShapeMismatch(f"{what}: {list(shape)} x {self.dtype.wire_name()} needs {nbytes} bytes; the "
                                f"workspace plan reserved {self.capacity}")
        return shape, nbytes


def _signature(g: Graph) -> list[tuple]:
    return [(n.id, n.op, tuple(n.inputs)) for n in g.nodes]


def plan_hazards(graph: Graph, topology: wsp.Topology) -> tuple[list[tuple[int, ...]], set[int]]:
    """What running `graph` inside `topology`'s workspace must order or save, from the plan:

    * reuse_deps[k]: the earlier nodes (indices) that read or wrote a port whose bytes
      node k's output overwrites (a port dead before node k runs; the allocator never
      lets ports that are live together overlap).  On one stream execution order covers
      them; across streams node k must wait for them.
    * snapshot: the nodes whose output is a graph output that a later port's bytes
      overwrite -- the planner's liveness ends a port at its last consumer and does not
      count graph outputs as consumers (ir/planner.go:186-283), so such an output must be
      copied out right after its producer runs."""
    ivs = {iv.port_id: iv for iv in topology.workspace.allocations}
    touched: dict[int, set[int]] = {}
    for k, tn in enumerate(topology.nodes):
        for p in list(tn.inputs) + list(tn.outputs):
            if p is not None and p.id in ivs:
                touched.setdefault(p.id, set()).add(k)

    def overlapping(pid: int):
        lo, hi = ivs[pid].offset, ivs[pid].offset + ivs[pid].size
        for q, iv in ivs.items():
            if q != pid and iv.offset < hi and lo < iv.offset + iv.size:
                yield iv

    reuse_deps: list[tuple[int, ...]] = []
    for k, tn in enumerate(topology.nodes):
        p = tn.outputs[0] if tn.outputs else None
        deps: set[int] = set()
        if p is not None and p.id in ivs:
            for iv in overlapping(p.id):
                if iv.end < ivs[p.id].start:
                    deps |= {j for j in touched.get(iv.port_id, ()) if j < k}
        reuse_deps.append(tuple(sorted(deps)))
    index = {n.id: k for k, n in enumerate(graph.nodes)}
    snapshot: set[int] = set()
    for producer in graph.outputs.values():
        k = index.get(producer)
        if k is None or not topology.nodes[k].outputs:
            continue
        pid = topology.nodes[k].outputs[0].id
        if pid in ivs and any(iv.start > ivs[pid].end for iv in overlapping(pid)):
            snapshot.add(k)
    return reuse_deps, snapshot


class AttachedWorkspace:
    """One graph's device arena with every port resolved to base + offset, made once by
    GraphBackend.attach_workspace (runtime.WorkspaceAttacher.AttachWorkspace,
    runtime/executor.go:28-48).

    Two properties of the plan are handled here rather than trusted:
    * the planner's liveness ends a port at its last consumer and knows nothing of graph
      outputs, so a later node can be given a graph output's bytes: such an output
      (`snapshot`) is copied out right after its producer runs; the others are returned
      as views into the arena, valid until the next call of the graph;
    * offset reuse follows execution order, not streams: under a multi-stream schedule a
      node whose output overwrites a dead port's bytes first waits for every node that
      read or wrote that port on another stream (`reuse_deps`)."""

    def __init__(self, graph: Graph, topology: wsp.Topology):
        if [t.name for t in topology.nodes] != [n.id for n in graph.nodes]:
            raise InvalidArgument("workspace: the topology's nodes are not the graph's nodes in order")
        layout = topology.workspace
        self.signature = _signature(graph)
        self.size = layout.size
        self.bindings = dict(layout.bindings)
        ivs = {iv.port_id: iv for iv in layout.allocations}
        nodes: list[tuple[int, DType, tuple, int]] = []      # (offset, dtype, dims, capacity)
        for tn in topology.nodes:
            p = tn.outputs[0] if tn.outputs else None
            if p is None or p.allocation is None or p.id not in ivs:
                raise InvalidArgument(f"workspace: node {tn.name!r} has no output allocation")
            nodes.append((p.allocation.base_offset, p.type.dtype, p.type.dims, wsp.port_byte_size(p, self.bindings)))
        inputs: dict[str, tuple[int, DType, tuple, int]] = {}
        for name in graph.inputs:
            if not name:
                continue
            off = topology.input_ports.get(name)
            port = next((tn.inputs[i] for gn, tn in zip(graph.nodes, topology.nodes)
                         for i, ref in enumerate(gn.inputs) if ref == name), None)
            if off is None or port is None:
                raise InvalidArgument(f"workspace: graph input {name!r} has no workspace offset")
            inputs[name] = (off, port.type.dtype, port.type.dims, wsp.port_byte_size(port, self.bindings))
        self.reuse_deps, self.snapshot = plan_hazards(graph, topology)
        align = max(layout.align, 1)
        pad = align - 256 if align > 256 else 0          # mf_alloc returns 256-byte aligned memory
        self.buffer = DeviceBuffer(max(layout.size, 1) + pad)
        self.base = wsp.align_up(self.buffer.ptr, align) if align > 1 else self.buffer.ptr
        self.node_slots = [_Slot(self.base + off, dt, dims, cap) for off, dt, dims, cap in nodes]
        self.input_slots = {name: _Slot(self.base + off, dt, dims, cap) for name, (off, dt, dims, cap) in inputs.items()}

    def contains(self, ptr: int) -> bool:
        return self.base <= ptr < self.base + max(self.size, 1)

    def close(self) -> None:
        self.buffer.free()


class GraphBackend:
    """runtime.Backend for the device path: CallGraph over shape.cast and FuseOp nodes, and
    runtime.WorkspaceAttacher: a graph with an attached workspace runs inside it."""

    def __init__(self, backend: CUDABackend, compat: int = 0):
        self.backend = backend
        self.compat = compat
        self._workspaces: dict[str, AttachedWorkspace] = {}

    # -- workspace ------------------------------------------------------------
    def attach_workspace(self, graph_name: str, graph: Graph, topology: wsp.Topology | None = None) -> wsp.Topology:
        """AttachWorkspace(graphName, graph, topology): allocate topology.workspace.size bytes
        once and resolve every port to base + offset.  With no topology the plan is made
        here (workspace.plan_graph, the graph's bindings).  Replaces an earlier attachment
        of the same name."""
        if topology is None:
            topology = wsp.plan_graph(graph)
        ws = AttachedWorkspace(graph, topology)
        self.detach_workspace(graph_name)
        self._workspaces[graph_name] = ws
        return topology

    def workspace(self, graph_name: str) -> AttachedWorkspace | None:
        return self._workspaces.get(graph_name)

    def detach_workspace(self, graph_name: str) -> None:
        ws = self._workspaces.pop(graph_name, None)
        if ws is not None:
            call("mf_device_sync")      # a call may still run on a stream of the caller's
            ws.close()

    def close(self) -> None:
        for name in list(self._workspaces):
            self.detach_workspace(name)

    # -- graph.call -----------------------------------------------------------
    def call_graph(self, request: GraphCallRequest, stream=None,
                   schedule: dict[str, NodeSchedule] | None = None) -> GraphCallResult:
        """Run the graph on `stream`, or on the streams of `schedule` (see the module text).
        With a schedule the call returns after every stream has finished.  A graph with an
        attached workspace runs inside it: inputs are copied to their slots, every node
        writes its slot, launch_bindings override the plan's bindings (each size at most
        the planned one)."""
        ws = self._workspaces.get(request.graph_name)
        if ws is not None and ws.signature != _signature(request.graph):
            raise InvalidArgument(f"graph.call {request.graph_name!r}: the attached workspace was planned for "
                                  f"another graph")
        bindings = {**ws.bindings, **request.launch_bindings} if ws is not None else {}
        staged = self._stage_inputs(request, ws, bindings, stream)
        if schedule is None:
            return self._call(request, staged, lambda k, node: stream, None, ws=ws, bindings=bindings)
        from .backend import Event, Stream
        nodes = request.graph.nodes
        for n in nodes:
            if n.id not in schedule:
                raise InvalidArgument(f"graph.call {request.graph_name!r}: node {n.id!r} has no stream assignment")
        # flat handle tables, resolved before the first dispatch
        stream_ids = sorted({schedule[n.id].stream_id for n in nodes} |
                            {b.stream_id for n in nodes for b in schedule[n.id].barriers})
        streams = {sid: Stream() for sid in stream_ids}
        events = {b.event_id: Event() for n in nodes for b in schedule[n.id].barriers}
        sid_of = [schedule[n.id].stream_id for n in nodes]
        reuse_wait = [[j for j in ws.reuse_deps[k] if sid_of[j] != sid_of[k]] if ws is not None else []
                      for k in range(len(nodes))]
        reuse_events = {j: Event() for deps in reuse_wait for j in deps}
        start = Event()
        try:
            # work already queued for the inputs on the caller's stream (the legacy
            # default stream when none is given), the input copies included, comes first
            start.record(stream)
            for st in streams.values():
                st.wait(start)

            def on_stream(k: int, node: GraphNode):
                sched = schedule[node.id]
                for b in sched.barriers:
                    if b.wait:
                        streams[sched.stream_id].wait(events[b.event_id])
                for j in reuse_wait[k]:
                    streams[sched.stream_id].wait(reuse_events[j])
                return streams[sched.stream_id]

            def after(k: int, node: GraphNode) -> None:
                for b in schedule[node.id].barriers:
                    if not b.wait:
                        events[b.event_id].record(streams[b.stream_id])
                if k in reuse_events:
                    reuse_events[k].record(streams[sid_of[k]])

            return self._call(request, staged, on_stream, after, sync=list(streams.values()), ws=ws,
                              bindings=bindings)
        finally:
            for st in streams.values():
                st.sync()
            for ev in list(events.values()) + list(reuse_events.values()):
                ev.close()
            for st in streams.values():
                st.close()
            start.close()

    def _stage_inputs(self, request: GraphCallRequest, ws: AttachedWorkspace | None, bindings: dict[str, int],
                      stream) -> dict[str, DeviceTensor]:
        """Copy each input into its workspace slot.  An input that already lies in the arena
        (an output of an earlier call fed back) and is not exactly its own slot is first
        copied out, before any slot is written: its bytes may overlap its own slot or
        another input's."""
        g = request.graph
        values: dict[str, DeviceTensor] = {}
        plan: list[tuple[str, DeviceTensor, _Slot, tuple[int, ...], int]] = []
        for name in g.inputs:
            if name not in request.inputs:
                raise InvalidArgument(f"graph.call {request.graph_name!r}: missing input {name!r}")
            t = request.inputs[name]
            if ws is None or name not in ws.input_slots:
                values[name] = t
                continue
            slot = ws.input_slots[name]
            shape, nbytes = slot.resolve(bindings, f"graph.call {request.graph_name!r} input {name!r}")
            if t.dtype() != slot.dtype:
                raise DTypeMismatch(f"graph.call {request.graph_name!r}: input {name!r} is "
                                    f"{t.dtype().wire_name()}, the plan says {slot.dtype.wire_name()}")
            if t.nbytes() != nbytes:
                raise ShapeMismatch(f"graph.call {request.graph_name!r}: input {name!r} holds {t.nbytes()} bytes, "
                                    f"the plan's {list(shape)} x {slot.dtype.wire_name()} is {nbytes}")
            plan.append((name, t, slot, shape, nbytes))
        h = stream_handle(stream)
        temps: list[DeviceBuffer] = []
        try:
            sources = {}
            for name, t, slot, _, nbytes in plan:
                src = t.dispatch_pointer()
                if nbytes and src != slot.ptr and ws.contains(src):
                    tmp = DeviceBuffer(nbytes)
                    temps.append(tmp)
                    call("mf_memcpy_d2d_async", tmp.ptr, src, nbytes, h)
                    src = tmp.ptr
                sources[name] = src
            for name, t, slot, shape, nbytes in plan:
                if sources[name] != slot.ptr and nbytes:
                    call("mf_memcpy_d2d_async", slot.ptr, sources[name], nbytes, h)
                values[name] = DeviceTensor(self.backend, shape, slot.dtype, DeviceView(slot.ptr, nbytes))
        finally:
            if temps:
                call("mf_stream_sync", h)
                for tmp in temps:
                    tmp.free()
        return values

    def _call(self, request: GraphCallRequest, values: dict[str, DeviceTensor], stream_for, after, sync=(),
              ws: AttachedWorkspace | None = None, bindings: dict[str, int] | None = None) -> GraphCallResult:
        g = request.graph
        produced: list[DeviceTensor] = []       # tensors this call allocated
        snapshots: dict[str, DeviceTensor] = {}
        try:
            for k, node in enumerate(g.nodes):
                args = []
                for ref in node.inputs:
                    if ref not in values:
                        raise InvalidArgument(f"graph.call {request.graph_name!r}: node {node.id!r} reads "
                                              f"unknown value {ref!r}")
                    args.append(values[ref])
                st = stream_for(k, node)
                out = None
                if ws is not None:
                    slot = ws.node_slots[k]
                    shape, nbytes = slot.resolve(bindings, f"graph.call {request.graph_name!r} node {node.id!r}")
                    out = DeviceTensor(self.backend, shape, slot.dtype, DeviceView(slot.ptr, nbytes))
                res = self._run_node(node, args, st, out)
                if ws is not None and k in ws.snapshot:
                    copy = self.backend.empty(res.shape(), res.dtype())
                    produced.append(copy)
                    if res.nbytes():
                        call("mf_memcpy_d2d_async", copy.dispatch_pointer(), res.dispatch_pointer(), res.nbytes(),
                             stream_handle(st))
                    snapshots[node.id] = copy
                if after is not None:
                    after(k, node)
                if ws is None and res is not None and all(res is not a for a in args):
                    produced.append(res)
                values[node.id] = res
            outputs = {}
            for name, ref in g.outputs.items():
                if ref not in values:
                    raise InvalidArgument(f"graph.call {request.graph_name!r}: output {name!r} refers to "
                                          f"unknown node {ref!r}")
                outputs[name] = snapshots.get(ref, values[ref])
        except BaseException:
            for st in sync:
                st.sync()
            for t in produced:
                t.close()
            raise
        for st in sync:
            st.sync()  # intermediates may still be in use on another stream
        keep = {id(t) for t in outputs.values()}
        for t in produced:
            if id(t) not in keep:
                t.close()
        return GraphCallResult(outputs)

    # -- nodes ----------------------------------------------------------------
    def _run_node(self, node: GraphNode, args: list[DeviceTensor], stream, out: DeviceTensor | None) -> DeviceTensor:
        if node.op == SHAPE_CAST:
            return self._cast(node, args, stream, out)
        if node.op == FUSE_OP:
            return self._fusion(node, args, stream, out)
        raise InvalidArgument(f"graph.call: op {node.op!r} (node {node.id!r}) is not supported by the CUDA backend")

    @staticmethod
    def _check_out(node: GraphNode, out: DeviceTensor, dtype: DType, n: int) -> None:
        if out.dtype() != dtype:
            raise DTypeMismatch(f"graph.call: node {node.id!r} produces {dtype.wire_name()}, its workspace slot is "
                                f"{out.dtype().wire_name()}")
        if len(out) != n:
            raise ShapeMismatch(f"graph.call: node {node.id!r} produces {n} elements, its workspace slot holds "
                                f"{len(out)}")

    def _cast(self, node: GraphNode, args: list[DeviceTensor], stream, out: DeviceTensor | None) -> DeviceTensor:
        if len(args) != 1:
            raise InvalidArgument(f"typer: shape.cast needs one input (node {node.id!r} has {len(args)})")
        x = args[0]
        src = _dtype_attr(node, "from_dtype")
        if src is not None and src != x.dtype():
            raise DTypeMismatch(f"shape.cast {node.id!r}: from_dtype {src.wire_name()} but the input is "
                                f"{x.dtype().wire_name()}")
        target = cast_target(node, x.dtype())
        if out is None:
            if target == x.dtype():
                return x
            return self.backend.convert(x, target, compat=self.compat, stream=stream)
        self._check_out(node, out, target, len(x))
        if target == x.dtype():
            if out.dispatch_pointer() != x.dispatch_pointer() and x.nbytes():
                call("mf_memcpy_d2d_async", out.dispatch_pointer(), x.dispatch_pointer(), x.nbytes(),
                     stream_handle(stream))
            return out
        if x.dtype() not in DECODE_SOURCES:
            raise DTypeUnsupported(f"convert: unsupported source dtype {x.dtype().name}")
        convert_raw(x.dtype(), target, x.dispatch_pointer(), out.dispatch_pointer(), len(x), self.compat, stream)
        return out

    def _fusion(self, node: GraphNode, args: list[DeviceTensor], stream, out: DeviceTensor | None) -> DeviceTensor:
        ks = node.attributes.get(KERNEL_ATTRIBUTE)
        kernel = ks.for_target(Target.CUDA) if isinstance(ks, KernelSet) else None
        if not isinstance(kernel, CUDAKernel):
            raise InvalidArgument(f"graph.call: fusion node {node.id!r} has no CUDA kernel "
                                  f"(attribute {KERNEL_ATTRIBUTE!r})")
        if len(args) != len(kernel.in_dtypes):
            raise InvalidArgument(f"codegen cuda: kernel {kernel.identifier()!r} expects {len(kernel.in_dtypes)} "
                                  f"inputs, got {len(args)}")
        n = 0
        shape: tuple[int, ...] = ()
        for a, dt, bc in zip(args, kernel.in_dtypes, kernel.in_bcast):
            if a.dtype() != dt:
                raise DTypeMismatch(f"fusion {node.id!r}: input dtype {a.dtype().wire_name()}, kernel expects "
                                    f"{dt.wire_name()}")
            if bc:
                if len(a) != bc:
                    raise InvalidArgument(f"fusion {node.id!r}: broadcast input of {len(a)} elements, kernel "
                                          f"expects {bc}")
            elif len(a) > n:
                n, shape = len(a), a.shape()
        for a, bc in zip(args, kernel.in_bcast):
            if not bc and len(a) != n:
                raise InvalidArgument(f"fusion {node.id!r}: inputs of {len(a)} and {n} elements")
        if out is None:
            out = self.backend.empty(shape, kernel.out_dtype)
        else:
            self._check_out(node, out, kernel.out_dtype, n)
        kernel.run([a.dispatch_pointer() for a in args], out.dispatch_pointer(), n, stream=stream)
        return out
