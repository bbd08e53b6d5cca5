"""Reference entry points outside the hot path that code written for the
reference may still call (CPU): statement formatting, the verification
hooks' registration point, the architecture define, and nvcc compiles
with Python source locations in the errors."""

import pytest

import thork_b200 as tk
from thork_b200 import codegen, ir, tracer
from thork_b200 import runtime as rt


def test_format_stmts_returns_text_and_locations():
    stmts = [ir.StoreStmt(ir.Name("x"), ir.Lit(1)), ir.StoreStmt(ir.Name("y"), ir.Lit(2))]
    stmts[1].loc = ("kernel.py", 7)
    text, locs = codegen.format_stmts(stmts, indent=2)
    assert text.splitlines() == ["  x = 1;", "  y = 2;"]
    assert locs == {1: ("kernel.py", 7)}
    one, _ = codegen.format_stmt(stmts[0])
    assert one == "    x = 1;"


def test_register_stype_hooks_accepts_the_known_keys_only():
    tracer.register_stype_hooks(binop=lambda *a: None)
    assert "binop" in tracer._stype_hooks
    with pytest.raises(TypeError):
        tracer.register_stype_hooks(bogus=lambda: None)


def test_kittens_sm_define_for_cap():
    assert rt.kittens_sm_define_for_cap("100a") == "KITTENS_SM100"
    assert rt.kittens_sm_define_for_cap("120") == "KITTENS_SM120"
    assert rt.kittens_sm_define_for_cap("90a") == "KITTENS_SM90"
    assert rt.kittens_sm_define_for_cap("80") == "KITTENS_SM80"


def test_nvcc_compile_and_error_locations():
    @tk.jit
    def inc(x: tk.DevicePointer[tk.dt.float32], tid: tk.Uint[tk.ThreadIdx]):
        x[tid] = x[tid] + 1.0

    cubin = rt.nvcc_compile(inc.cuda_source, source_map=inc.source_map)
    assert len(cubin) > 1000
    bad = inc.cuda_source.replace("+ 1.0f", "+ undefined_symbol")
    assert bad != inc.cuda_source
    with pytest.raises(RuntimeError, match="nvcc compile failed"):
        rt.nvcc_compile(bad, source_map=inc.source_map)


def test_host_launcher_paths_explain_themselves():
    with pytest.raises(NotImplementedError):
        rt.compile_source_to_shared_lib("")
    with pytest.raises(NotImplementedError):
        rt.dispatch_tk(None, "k", [], [], (1, 1, 1), (1, 1, 1), 0)


@pytest.mark.parametrize("m,chunk", [(8192, 1024), (3000, 512), (1024, 256), (2047, 256),
                                     (5000, 768), (1500, 512), (100000, 12544)])
def test_pipelined_host_path_chunk_schedule(m, chunk):
    """The row chunks of the pipelined host path cover every row once, in
    order; long inputs start and end with short chunks, short ones keep
    equal chunks."""
    from thork_b200.kernels._library import chunk_schedule
    sched = chunk_schedule(m, chunk)
    assert sum(sched) == m and min(sched) > 0 and max(sched) <= chunk
    if m >= 4 * chunk:
        q = chunk // 4
        assert sched[:2] == [q, 2 * q] and sched[-3:] == [3 * q, q, q]
    else:
        assert sched == [min(chunk, m - r0) for r0 in range(0, m, chunk)]
