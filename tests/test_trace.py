"""Tracing and code generation (CPU): parity of parameter lists and
copy-back flags with the reference's own traces, argument-check errors
identical to the reference's, source maps, and NVRTC compiles of every
kernel for sm_100a (NVRTC needs no GPU)."""

import json
import os

import numpy as np
import pytest

import thork_b200 as tk
from thork_b200 import ir
from thork_b200 import runtime as rt

import kernel_zoo

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def ref_traces():
    with open(os.path.join(GOLDEN, "reference_traces.json")) as f:
        return json.load(f)


@pytest.fixture(scope="module")
def zoo():
    return kernel_zoo.build(tk)


def _params(k):
    return [{"name": p.name, "kind": p.kind, "dtype": p.dtype.name, "written": p.written}
            for p in k.params]


@pytest.mark.parametrize("name", sorted(kernel_zoo.build(tk)))
def test_params_and_written_flags_match_reference(name, zoo, ref_traces):
    assert _params(zoo[name]) == ref_traces[name]["params"]


@pytest.mark.parametrize("name", ["copy_tile", "tma_copy"])
def test_tile_kernel_params_match_reference(name, ref_traces):
    tiles = kernel_zoo.build_tiles(tk)
    assert _params(tiles[name]) == ref_traces[name]["params"]


@pytest.mark.parametrize("name", sorted(kernel_zoo.build(tk)))
def test_zoo_kernels_compile_for_sm100a(name, zoo):
    cubin = rt.nvrtc_compile(zoo[name].cuda_source, source_map=zoo[name].source_map)
    assert len(cubin) > 1000


@pytest.mark.parametrize("name", ["regtile_matmul", "tma_matmul", "tcgen05_matmul"])
def test_tile_matmul_kernels_compile_for_sm100a(name):
    """The traced tile matmuls (register tiles + mma.sync, TMA into shared
    tiles, tcgen05 into TMEM) lower through the tile library and compile."""
    import tile_kernels
    k = getattr(tile_kernels, name)(tk)
    cubin = rt.nvrtc_compile(k.cuda_source, source_map=k.source_map)
    assert len(cubin) > 1000


@pytest.mark.parametrize("name", ["copy_tile", "tma_copy"])
def test_tile_copy_kernels_compile_for_sm100a(name):
    k = kernel_zoo.build_tiles(tk)[name]
    cubin = rt.nvrtc_compile(k.cuda_source, source_map=k.source_map)
    assert len(cubin) > 1000


def test_validation_errors_match_reference():
    with open(os.path.join(GOLDEN, "reference_validation.json")) as f:
        ref = json.load(f)
    f32p = ir.Param(name="A", kind="pointer", dtype=tk.dt.float32)
    glp = ir.Param(name="G", kind="kittens_global", dtype=tk.dt.bfloat16)
    cases = {
        "pointer_not_array": (rt._expect_pointer_arg, [1.0, 2.0], f32p),
        "pointer_wrong_dtype": (rt._expect_pointer_arg, np.zeros(4, np.int32), f32p),
        "pointer_unmapped_dtype": (rt._expect_pointer_arg, np.zeros(4, np.float64), f32p),
        "pointer_non_contiguous": (rt._expect_pointer_arg, np.zeros((4, 4), np.float32)[:, 1], f32p),
        "global_not_array": (rt._expect_kittens_arg, "x", glp),
        "global_not_2d": (rt._expect_kittens_arg, np.zeros(8, np.uint16), glp),
        "global_itemsize": (rt._expect_kittens_arg, np.zeros((4, 4), np.float32), glp),
        "global_non_contiguous": (rt._expect_kittens_arg, np.zeros((4, 8), np.uint16)[:, ::2], glp),
    }
    for name, (fn, arg, p) in cases.items():
        with pytest.raises(Exception) as ei:
            fn(arg, p)
        assert type(ei.value).__name__ == ref[name]["type"], name
        assert str(ei.value) == ref[name]["message"], name


def test_bf16_accepts_ml_dtypes_and_uint16_storage():
    ml = pytest.importorskip("ml_dtypes")
    p = ir.Param(name="A", kind="pointer", dtype=tk.dt.bfloat16)
    rt._expect_pointer_arg(np.zeros(4, ml.bfloat16), p)
    rt._expect_pointer_arg(np.zeros(4, np.uint16), p)
    with pytest.raises(TypeError):
        rt._expect_pointer_arg(np.zeros(4, np.int16), p)


def test_source_map_points_at_user_lines():
    this = os.path.abspath(__file__)

    @tk.jit
    def add_two(out: tk.DevicePointer[tk.dt.float32], a: tk.DevicePointer[tk.dt.float32],
                bid: tk.Uint[tk.BlockIdx], tid: tk.Uint[tk.ThreadIdx], bdm: tk.Uint[tk.BlockDim]):
        i = bid * bdm + tid
        x = a[i] + 1.0
        out[i] = x + 1.0  # mapped line

    smap = add_two.source_map
    assert smap and {os.path.abspath(f) for f, _ in smap.values()} == {this}
    src_lines = add_two.cuda_source.splitlines()
    (gen_line, (f, py_line)), = smap.items()
    with open(this) as fh:
        assert "mapped line" in fh.read().splitlines()[py_line - 1]
    assert src_lines[gen_line - 1].strip().startswith("out[")


def test_annotation_and_arity_errors():
    with pytest.raises(TypeError):
        tk.DevicePointer[int]

    @tk.jit
    def bad(x: int):
        pass

    with pytest.raises(TypeError):
        bad.cuda_source

    @tk.jit
    def noann(x):
        pass

    with pytest.raises(TypeError):
        noann.cuda_source
    with pytest.raises(TypeError):
        tk.kittens.Global[tk.dt.bfloat16, (0, 4)]
    with pytest.raises(TypeError):
        tk.Uint[int]


def test_traced_value_in_python_bool_context_raises():
    @tk.jit
    def k(a: tk.DevicePointer[tk.dt.float32], tid: tk.Uint[tk.ThreadIdx]):
        if a[tid] > 0:  # noqa: SIM102 - the error is the point
            a[tid] = 0.0

    with pytest.raises(TypeError, match="boolean context"):
        k.cuda_source


def test_expression_printing_precedence():
    from thork_b200.codegen import format_expr
    a, b, c = ir.Name("a"), ir.Name("b"), ir.Name("c")
    assert format_expr(ir.Bin("-", a, ir.Bin("-", b, c))) == "a - (b - c)"
    assert format_expr(ir.Bin("-", ir.Bin("-", a, b), c)) == "a - b - c"
    assert format_expr(ir.Bin("*", ir.Bin("+", a, b), c)) == "(a + b) * c"
    assert format_expr(ir.Bin("<<", a, ir.Bin("+", b, c))) == "a << b + c"
    assert format_expr(ir.Unary("-", ir.Bin("+", a, b))) == "-(a + b)"
    assert format_expr(ir.Lit(3000000000)) == "3000000000u"
    assert format_expr(ir.Lit(2.0)) == "2.0f"


def test_compile_for_arch_sm100_only():
    @tk.jit
    def k(a: tk.DevicePointer[tk.dt.float32], tid: tk.Uint[tk.ThreadIdx]):
        a[tid] = tk.sqrt(a[tid])

    k.compile_for_arch("100a")
    with pytest.raises(ValueError):
        k.compile_for_arch("90a")
