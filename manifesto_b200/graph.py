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
node IDs.  Nodes run in list order (the lowered graph is topologically sorted) on one
stream; intermediate tensors no output refers to are freed when the call returns.
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

    def call_graph(self, request: GraphCallRequest, stream=None) -> GraphCallResult:
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
                out = self._run_node(node, args, stream)
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
            for t in produced:
                t.close()
            raise
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
