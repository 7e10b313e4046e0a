"""CPU-only checks of the C ABI library and the host-side logic.

No kernel runs here: the library must load without a GPU, export every
symbol include/mfcuda.h declares, and its host-only entry points (program
validation, checkpoint partitioning, error mapping) work on the CPU.
"""
import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols() -> list[str]:
    text = (ROOT / "include" / "mfcuda.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*)\s+(mf_\w+)\s*\(", text, flags=re.M)))


def test_library_exports_every_declared_symbol():
    from manifesto_b200 import _abi
    L = _abi.lib()
    names = declared_symbols()
    assert len(names) >= 40
    for name in names:
        assert hasattr(L, name), name
    # every declared entry point has a ctypes signature (mf_last_error returns a string)
    assert set(names) - {"mf_last_error"} == set(_abi.SIGNATURES)


def test_call_refuses_undeclared_entry_points():
    from manifesto_b200 import _abi
    with pytest.raises(KeyError):
        _abi.call("mf_not_declared")


def test_abi_version_and_no_device_paths():
    from manifesto_b200 import _abi
    L = _abi.lib()
    assert L.mf_abi_version() == 1
    c = ctypes.c_int(-1)
    assert L.mf_device_count(ctypes.byref(c)) == 0 and c.value >= 0


def test_kernels_refuse_before_init():
    """Without mf_init every kernel entry reports ErrBackendClosed (no CPU fallback)."""
    from manifesto_b200 import _abi
    L = _abi.lib()
    c = ctypes.c_int(0)
    L.mf_device_count(ctypes.byref(c))
    if c.value:
        pytest.skip("a GPU is visible; this checks the closed path")
    assert L.mf_convert(5, 2, 1, 1, 16, 0, None) == -6
    assert "not initialised" in _abi.last_error()
    assert L.mf_axpy(1, 1, 16, 1.0, 2, 0, None) == -6
    assert L.mf_init(0) == -8  # ErrNeedsPlatformSetup: no device


def test_error_mapping():
    from manifesto_b200 import errors
    with pytest.raises(errors.DTypeUnsupported):
        errors.raise_for_status(-3, "x")
    with pytest.raises(errors.ShapeInvalid):
        errors.raise_for_status(-7, "x")
    with pytest.raises(errors.AllocatorExhausted):
        errors.raise_for_status(-9, "x")


def test_dtype_rules():
    from manifesto_b200.dtype import DType
    assert DType.INT4.bytes_for(5) == 3 and DType.INT4.logical_elements(3) == 6
    assert DType.BFLOAT16.bytes_for(7) == 14
    with pytest.raises(ValueError):
        DType.FLOAT32.logical_elements(6)
    assert [int(d) for d in (DType.FLOAT8_E4M3, DType.FLOAT8_E5M2, DType.INT4)] == [5, 6, 11]


def test_partition_covers_every_row():
    from manifesto_b200 import checkpoint
    specs = checkpoint.llama3_8b_layout()
    assert len(specs) == 291
    assert sum(s.numel for s in specs) == 8_030_261_248
    for world in (1, 2, 3, 4, 8):
        seen = [[] for _ in specs]
        for r in range(world):
            for t, (first, rows) in enumerate(checkpoint.partition(specs, world, r)):
                seen[t].append((first, rows))
        for t, parts in enumerate(seen):
            assert parts[0][0] == 0
            for (f0, n0), (f1, _) in zip(parts, parts[1:]):
                assert f0 + n0 == f1
            assert sum(n for _, n in parts) == specs[t].rows
            assert max(n for _, n in parts) - min(n for _, n in parts) <= 1


def test_partition_rejects_bad_rank():
    from manifesto_b200 import checkpoint
    from manifesto_b200.errors import InvalidArgument
    with pytest.raises(InvalidArgument):
        checkpoint.partition(checkpoint.llama3_8b_layout(layers=1), 2, 2)


def test_fused_compile_validation_on_host():
    """mf_fused_compile validates postfix programs without touching a device."""
    from manifesto_b200 import fusion
    from manifesto_b200.dtype import DType
    from manifesto_b200.errors import InvalidArgument
    from manifesto_b200.fusion import NodeType as N
    k = fusion.emit_cuda(fusion.swiglu_chain(), in_bcast=[0, 4096, 4096, 0])
    assert k.specialised()
    root = fusion.unary(N.RELU, fusion.binary(N.ADD, fusion.input_node(0), fusion.input_node(1)))
    k = fusion.emit_cuda(fusion.FusionAST(root, ["x", "y"], "result"))
    assert not k.specialised()
    with pytest.raises(InvalidArgument, match="reads input 2"):
        fusion.emit_cuda(fusion.FusionAST(fusion.input_node(2), ["x"], "o"))
    bad = fusion.ASTNode(N.INVALID)
    with pytest.raises(InvalidArgument):
        fusion.emit_cuda(fusion.FusionAST(bad, ["x"], "o"))
    deep = fusion.input_node(0)
    for _ in range(20):
        deep = fusion.binary(N.ADD, fusion.input_node(0), deep)
    # right-leaning chain keeps the stack at depth 21 > 16 slots
    with pytest.raises(InvalidArgument, match="stack slots"):
        fusion.emit_cuda(fusion.FusionAST(deep, ["x"], "o"))


def test_postfix_and_node_table_agree():
    from manifesto_b200 import fusion
    f = fusion.swiglu_chain()
    ops, args, consts = fusion.postfix(f.root)
    assert ops == [1, 1, 5, 1, 3, 17, 1, 5] and args[:2] == [0, 1] and consts == []
    t = fusion.node_table(f.root)
    assert t["root"] == len(t["type"]) - 1 and list(t["type"]) == ops


def test_synthetic_generators_deterministic():
    from manifesto_b200 import synthetic
    a = synthetic.uniform_bytes(1, 1000)
    assert (a == synthetic.uniform_bytes(1, 1000)).all()
    z = synthetic.normal_f32(2, 1 << 16)
    assert abs(float(z.mean())) < 0.02 and abs(float(z.std()) - 1) < 0.02
    assert (synthetic.splitmix64(3, 10, offset=5) == synthetic.splitmix64(3, 15)[5:]).all()
