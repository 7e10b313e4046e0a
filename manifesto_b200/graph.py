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
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Sequence

from .backend import CUDABackend, DeviceTensor
from .dtype import DType, parse
from .errors import DTypeMismatch, InvalidArgument
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


@dataclass
class Graph:
    """ast.Graph: nodes in topological order, input names, output name -> node ID."""
    nodes: list[GraphNode]
    inputs: list[str] = field(default_factory=list)
    outputs: dict[str, str] = field(default_factory=dict)
    execution_dtype: DType = DType.FLOAT32


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


class GraphBackend:
    """runtime.Backend for the device path: CallGraph over shape.cast and FuseOp nodes."""

    def __init__(self, backend: CUDABackend, compat: int = 0):
        self.backend = backend
        self.compat = compat

    def call_graph(self, request: GraphCallRequest, stream=None,
                   schedule: dict[str, NodeSchedule] | None = None) -> GraphCallResult:
        """Run the graph on `stream`, or on the streams of `schedule` (see the module text).
        With a schedule the call returns after every stream has finished."""
        if schedule is None:
            return self._call(request, lambda node: stream, None)
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
        start = Event()
        try:
            # work already queued for the inputs on the caller's stream (the legacy
            # default stream when none is given) comes first
            start.record(stream)
            for st in streams.values():
                st.wait(start)

            def on_stream(node: GraphNode):
                sched = schedule[node.id]
                for b in sched.barriers:
                    if b.wait:
                        streams[sched.stream_id].wait(events[b.event_id])
                return streams[sched.stream_id]

            def after(node: GraphNode) -> None:
                for b in schedule[node.id].barriers:
                    if not b.wait:
                        events[b.event_id].record(streams[b.stream_id])

            return self._call(request, on_stream, after, sync=list(streams.values()))
        finally:
            for st in streams.values():
                st.sync()
            for ev in events.values():
                ev.close()
            for st in streams.values():
                st.close()
            start.close()

    def _call(self, request: GraphCallRequest, stream_for, after, sync=()) -> GraphCallResult:
        g = request.graph
        values: dict[str, DeviceTensor] = {}
        for name in g.inputs:
            if name not in request.inputs:
                raise InvalidArgument(f"graph.call {request.graph_name!r}: missing input {name!r}")
            values[name] = request.inputs[name]
        produced: list[DeviceTensor] = []
        try:
            for node in g.nodes:
                args = []
                for ref in node.inputs:
                    if ref not in values:
                        raise InvalidArgument(f"graph.call {request.graph_name!r}: node {node.id!r} reads "
                                              f"unknown value {ref!r}")
                    args.append(values[ref])
                out = self._run_node(node, args, stream_for(node))
                if after is not None:
                    after(node)
                if out is not None and all(out is not a for a in args):
                    produced.append(out)
                values[node.id] = out
            outputs = {}
            for name, ref in g.outputs.items():
                if ref not in values:
                    raise InvalidArgument(f"graph.call {request.graph_name!r}: output {name!r} refers to "
                                          f"unknown node {ref!r}")
                outputs[name] = values[ref]
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
    def _run_node(self, node: GraphNode, args: list[DeviceTensor], stream) -> DeviceTensor:
        if node.op == SHAPE_CAST:
            return self._cast(node, args, stream)
        if node.op == FUSE_OP:
            return self._fusion(node, args, stream)
        raise InvalidArgument(f"graph.call: op {node.op!r} (node {node.id!r}) is not supported by the CUDA backend")

    def _cast(self, node: GraphNode, args: list[DeviceTensor], stream) -> DeviceTensor:
        if len(args) != 1:
            raise InvalidArgument(f"typer: shape.cast needs one input (node {node.id!r} has {len(args)})")
        x = args[0]
        src = _dtype_attr(node, "from_dtype")
        if src is not None and src != x.dtype():
            raise DTypeMismatch(f"shape.cast {node.id!r}: from_dtype {src.wire_name()} but the input is "
                                f"{x.dtype().wire_name()}")
        target = cast_target(node, x.dtype())
        if target == x.dtype():
            return x
        return self.backend.convert(x, target, compat=self.compat, stream=stream)

    def _fusion(self, node: GraphNode, args: list[DeviceTensor], stream) -> DeviceTensor:
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
        out = self.backend.empty(shape, kernel.out_dtype)
        kernel.run([a.dispatch_pointer() for a in args], out.dispatch_pointer(), n, stream=stream)
        return out
