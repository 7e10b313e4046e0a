"""FusionAST mirror and the CUDA codegen target.

Mirrors manifesto's optimizer.FusionAST / ASTNode / NodeType
(optimizer/fusion_ast.go:30-180) and adds the CUDA target beside codegen's
CPU and Metal targets (codegen/codegen.go:34-42, codegen/metal.go:79-149):
``emit_cuda`` lowers a FusionAST to a postfix program and compiles it with
``mf_fused_compile``; ``CUDAKernel.run`` is the device counterpart of
``CPUKernel.Run`` (codegen/cpu.go:59-92), with the same argument checks and
error wording.
"""
from __future__ import annotations

import ctypes
import enum
from dataclasses import dataclass, field
from typing import Sequence

import numpy as np

from . import _abi
from ._abi import call
from .backend import stream_handle
from .dtype import DType
from .errors import InvalidArgument


class NodeType(enum.IntEnum):
    """optimizer.NodeType (optimizer/fusion_ast.go:32-65)."""

    INVALID = 0
    INPUT = 1
    CONSTANT = 2
    ADD = 3
    SUB = 4
    MUL = 5
    DIV = 6
    MAX = 7
    MIN = 8
    NEG = 9
    ABS = 10
    SQRT = 11
    EXP = 12
    LOG = 13
    RELU = 14
    SIGMOID = 15
    TANH = 16
    SILU = 17
    GELU = 18
    LEAKY_RELU = 19

    def arity(self) -> int:
        """NodeType.Arity (optimizer/fusion_ast.go:168-180)."""
        if self in (NodeType.INPUT, NodeType.CONSTANT):
            return 0
        if NodeType.NEG <= self <= NodeType.LEAKY_RELU:
            return 1
        if NodeType.ADD <= self <= NodeType.MIN:
            return 2
        return -1


# optimizer.elementwiseTable (optimizer/elementwise.go:15-37); sin/cos disabled
ELEMENTWISE_OPS = {
    "math.add": NodeType.ADD, "math.sub": NodeType.SUB, "math.mul": NodeType.MUL, "math.div": NodeType.DIV,
    "math.max": NodeType.MAX, "math.min": NodeType.MIN, "math.neg": NodeType.NEG, "math.abs": NodeType.ABS,
    "math.sqrt": NodeType.SQRT, "math.exp": NodeType.EXP, "math.log": NodeType.LOG, "math.sign": NodeType.NEG,
    "activation.relu": NodeType.RELU, "activation.sigmoid": NodeType.SIGMOID, "activation.tanh": NodeType.TANH,
    "activation.swish": NodeType.SILU, "activation.gelu": NodeType.GELU,
    "activation.leaky_relu": NodeType.LEAKY_RELU,
}


@dataclass
class ASTNode:
    """optimizer.ASTNode (optimizer/fusion_ast.go:70-76)."""

    type: NodeType
    value: float = 0.0
    input_index: int = 0
    children: list["ASTNode"] = field(default_factory=list)
    dtype: DType = DType.INVALID


def input_node(index: int, dtype: DType = DType.INVALID) -> ASTNode:
    return ASTNode(NodeType.INPUT, input_index=index, dtype=dtype)


def constant_node(value: float, dtype: DType = DType.INVALID) -> ASTNode:
    return ASTNode(NodeType.CONSTANT, value=value, dtype=dtype)


def unary(t: NodeType, child: ASTNode) -> ASTNode:
    return ASTNode(t, children=[child], dtype=child.dtype)


def binary(t: NodeType, left: ASTNode, right: ASTNode) -> ASTNode:
    return ASTNode(t, children=[left, right], dtype=left.dtype if left.dtype != DType.INVALID else right.dtype)


@dataclass
class FusionAST:
    """optimizer.FusionAST (optimizer/fusion_ast.go:86-113)."""

    root: ASTNode
    input_ports: list[str]
    output_port: str = ""
    count_expr: str = ""
    dtype: DType = DType.FLOAT32
    contained_node_ids: list[str] = field(default_factory=list)


class Target(enum.IntEnum):
    """codegen.Target (codegen/codegen.go:34-42) with the new CUDA target."""

    CPU = 0
    METAL = 1
    CUDA = 2


def postfix(root: ASTNode) -> tuple[list[int], list[int], list[float]]:
    """Flatten the tree: (op, arg, consts) in evaluation order."""
    ops: list[int] = []
    args: list[int] = []
    consts: list[float] = []

    def walk(node: ASTNode) -> None:
        t = NodeType(node.type)
        if t.arity() < 0:
            raise InvalidArgument(f"codegen cuda: invalid node type {int(node.type)}")
        if len(node.children) != t.arity():
            raise InvalidArgument(f"codegen cuda: {t.name} expects {t.arity()} children, got {len(node.children)}")
        for c in node.children:
            walk(c)
        ops.append(int(t))
        if t == NodeType.INPUT:
            args.append(int(node.input_index))
        elif t == NodeType.CONSTANT:
            args.append(len(consts))
            consts.append(float(node.value))
        else:
            args.append(0)

    walk(root)
    return ops, args, consts


def node_table(root: ASTNode) -> dict:
    """The tree as parallel arrays (type, value, input, child0, child1, root)."""
    types, values, inputs, c0, c1 = [], [], [], [], []

    def walk(node: ASTNode) -> int:
        kids = [walk(c) for c in node.children]
        idx = len(types)
        types.append(int(node.type))
        values.append(float(node.value))
        inputs.append(int(node.input_index))
        c0.append(kids[0] if len(kids) > 0 else -1)
        c1.append(kids[1] if len(kids) > 1 else -1)
        return idx

    r = walk(root)
    return {"type": np.array(types, np.int32), "value": np.array(values, np.float64),
            "input": np.array(inputs, np.int32), "child0": np.array(c0, np.int32),
            "child1": np.array(c1, np.int32), "root": r}


class CUDAKernel:
    """One FusionAST compiled for the CUDA target."""

    def __init__(self, fusion: FusionAST, in_dtypes: Sequence[DType], in_bcast: Sequence[int], out_dtype: DType):
        ops, args, consts = postfix(fusion.root)
        n_in = len(fusion.input_ports)
        if len(in_dtypes) != n_in or len(in_bcast) != n_in:
            raise InvalidArgument(f"codegen cuda: {n_in} input ports but {len(in_dtypes)} dtypes / {len(in_bcast)} "
                                  "broadcast lengths")
        self._ops = (ctypes.c_int32 * len(ops))(*ops)
        self._args = (ctypes.c_int32 * len(args))(*args)
        self._consts = (ctypes.c_double * max(1, len(consts)))(*consts)
        self._dts = (ctypes.c_int32 * max(1, n_in))(*[int(d) for d in in_dtypes])
        self._bc = (ctypes.c_int64 * max(1, n_in))(*[int(b) for b in in_bcast])
        prog = _abi.FusedProgram(len(ops), self._ops, self._args, len(consts), self._consts, n_in, self._dts,
                                 self._bc, int(out_dtype))
        h = ctypes.c_void_p()
        call("mf_fused_compile", ctypes.byref(prog), ctypes.byref(h))
        self.handle = h.value
        self.fusion = fusion
        self.in_dtypes = [DType(d) for d in in_dtypes]
        self.in_bcast = [int(b) for b in in_bcast]
        self.out_dtype = DType(out_dtype)
        self._identifier = fusion.output_port or "anon_" + "_".join(fusion.input_ports)

    def target(self) -> Target:
        return Target.CUDA

    def identifier(self) -> str:
        return self._identifier

    def inputs(self) -> list[str]:
        return list(self.fusion.input_ports)

    def output(self) -> str:
        return self.fusion.output_port

    def kind(self) -> int:
        """1: the hand-written SwiGLU kernel; 2: the kernel generated for this expression; 0: the interpreter."""
        s = ctypes.c_int()
        call("mf_fused_is_specialised", self.handle, ctypes.byref(s))
        return s.value

    def specialised(self) -> bool:
        """True when the hand-written SwiGLU-chain kernel runs this fusion."""
        return self.kind() == 1

    def generated(self) -> bool:
        """True when the CUDA codegen target compiled a kernel for this expression."""
        return self.kind() == 2

    def run(self, inputs: Sequence[int], output: int, count: int, amax: int | None = None, stream=None) -> None:
        """Evaluate the fusion over `count` elements of device buffers."""
        if len(inputs) != len(self.fusion.input_ports):
            raise InvalidArgument(f"codegen cuda: kernel {self._identifier!r} expects "
                                  f"{len(self.fusion.input_ports)} inputs, got {len(inputs)}")
        ptrs = (ctypes.c_void_p * max(1, len(inputs)))(*[int(p) for p in inputs])
        call("mf_fused_launch", self.handle, ptrs, int(output), int(count), amax, stream_handle(stream))

    def run_fp8(self, inputs: Sequence[int], precast: int, dst: int, count: int, amax: int, scale_inv: int | None,
                fp8_dtype: DType = DType.FLOAT8_E4M3, compat: int = 0, stream=None) -> None:
        """Chain -> pre-cast store -> amax -> per-tensor scaled FP8 cast."""
        if len(inputs) != len(self.fusion.input_ports):
            raise InvalidArgument(f"codegen cuda: kernel {self._identifier!r} expects "
                                  f"{len(self.fusion.input_ports)} inputs, got {len(inputs)}")
        ptrs = (ctypes.c_void_p * max(1, len(inputs)))(*[int(p) for p in inputs])
        call("mf_fused_fp8", self.handle, ptrs, int(precast), int(dst), int(fp8_dtype), int(amax), scale_inv,
             int(count), int(compat), stream_handle(stream))

    def close(self) -> None:
        if self.handle:
            call("mf_fused_destroy", self.handle)
        self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def emit_cuda(fusion: FusionAST, in_dtypes: Sequence[DType] | None = None, in_bcast: Sequence[int] | None = None,
              out_dtype: DType | None = None) -> CUDAKernel:
    """EmitCUDA: the CUDA counterpart of EmitCPU / EmitMetal."""
    if fusion is None:
        raise InvalidArgument("codegen cuda: fusion is required")
    if fusion.root is None:
        raise InvalidArgument("codegen cuda: fusion root is required")
    n = len(fusion.input_ports)
    exec_dtype = fusion.dtype if fusion.dtype in (DType.FLOAT32, DType.FLOAT16, DType.BFLOAT16) else DType.FLOAT32
    in_dtypes = list(in_dtypes) if in_dtypes is not None else [exec_dtype] * n
    in_bcast = list(in_bcast) if in_bcast is not None else [0] * n
    return CUDAKernel(fusion, in_dtypes, in_bcast, out_dtype if out_dtype is not None else exec_dtype)


def swiglu_chain() -> FusionAST:
    """Mul(Silu(Add(Mul(x, gamma), beta)), y): the chain of the fused-FP8 workload."""
    x, g, b, y = (input_node(i, DType.BFLOAT16) for i in range(4))
    root = binary(NodeType.MUL, unary(NodeType.SILU, binary(NodeType.ADD, binary(NodeType.MUL, x, g), b)), y)
    return FusionAST(root=root, input_ports=["x", "gamma", "beta", "y"], output_port="out", dtype=DType.BFLOAT16)


def gelu_affine_chain() -> FusionAST:
    """Gelu(Add(Mul(x, gamma), beta)): an affine-then-GELU chain (no specialised kernel; the
    generic CUDA path runs it)."""
    x, g, b = (input_node(i, DType.BFLOAT16) for i in range(3))
    root = unary(NodeType.GELU, binary(NodeType.ADD, binary(NodeType.MUL, x, g), b))
    return FusionAST(root=root, input_ports=["x", "gamma", "beta"], output_port="out", dtype=DType.BFLOAT16)
