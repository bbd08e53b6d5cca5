"""Host-side logic of bench.py (no GPU): both arms report the same config,
the post-timing check samples rows from every rank's block, and operands
rotate through enough copies to keep consecutive steps out of L2."""

import importlib.util
import os

import numpy as np
import pytest

from thork_b200 import dist

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(REPO, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_check_rows_cover_every_rank(bench, world):
    m = 8192
    rows = bench.check_row_sample(m, world, dist)
    assert len(rows) <= bench.CHECK_ROWS and len(rows) == len(set(rows.tolist()))
    assert np.all(np.diff(rows) > 0)
    for q in range(world):
        s, e = dist.row_shard(m, world, q)
        mine = rows[(rows >= s) & (rows < e)]
        assert s in mine and e - 1 in mine, f"rank {q}: block edges not sampled"
        assert len(mine) >= 2


def test_check_rows_are_seeded(bench):
    assert np.array_equal(bench.check_row_sample(8192, 4, dist), bench.check_row_sample(8192, 4, dist))


@pytest.mark.parametrize("name", ["bf16_gemm_8192", "bf16_gemm_4096", "e4m3_gemm_8192",
                                  "skinny_m1", "skinny_m16", "skinny_m128", "add_f32"])
@pytest.mark.parametrize("world", [1, 2, 8])
def test_config_keys_complete_and_stable(bench, name, world):
    cfg = bench.config_for(name, world)
    assert cfg == bench.config_for(name, world)
    assert cfg["workload"] == name and "l2_policy" in cfg and "parallelism" in cfg


def test_l2_policy_is_truthful(bench):
    # 4096^3 bf16: A + B + C = 96 MiB fits the 126 MB L2, so operands rotate
    assert bench.gemm_copies(4096, "bf16") >= 2
    assert bench.gemm_copies(4096, "bf16") * 2 * 4096 * 4096 * 2 >= 2 * bench.L2_BYTES
    assert "rotating" in bench.config_for("bf16_gemm_4096", 1)["l2_policy"]
    # 8192^3: 384 MiB (bf16) / 256 MiB (e4m3) already exceed twice the L2
    assert bench.gemm_copies(8192, "bf16") == 1 and bench.gemm_copies(8192, "e4m3") == 1
    for n_loc in (14336, 7168, 1792):
        assert bench.skinny_copies(n_loc) * 4096 * n_loc * 2 >= 3 * bench.L2_BYTES


def test_col_shard_matches_package(bench):
    for world in (1, 2, 4, 8):
        for q in range(world):
            assert bench._col_shard(14336, world, q) == dist.col_shard(14336, world, q)


def test_cpu_rate_uses_whole_product_when_cheap(bench):
    a = np.ones((128, 64), np.float32)
    b = np.ones((64, 32), np.float32)
    tflops, sample, rows = bench.cpu_matmul_rate(a, b, 0.01)
    assert rows == 128 and tflops > 0 and "128x64" in sample


def test_checked_combines_single_rank(bench):
    class One:
        world = 1

        def max(self, x):
            return x

        def min(self, x):
            return x
    ok = bench.checked(One(), {"max_rel_err": 2.5e-3, "tolerance": 1e-2, "bitequal_vs_nccl": None})
    assert ok["pass"] is True
    bad = bench.checked(One(), {"max_rel_err": 2e-2, "tolerance": 1e-2, "bitequal_vs_nccl": None})
    assert bad["pass"] is False
    neq = bench.checked(One(), {"max_rel_err": 0.0, "tolerance": 1e-2, "bitequal_vs_nccl": False})
    assert neq["pass"] is False


def test_auto_gather_config_names_the_resolved_mode(bench):
    assert "multimem" in bench.config_for("bf16_gemm_8192", 8, "auto")["parallelism"]
    assert "P2P" in bench.config_for("bf16_gemm_8192", 2, "auto")["parallelism"]
    assert bench.config_for("bf16_gemm_8192", 1, "auto")["parallelism"] == "1 GPU"
    assert bench.config_for("bf16_gemm_8192", 4, "auto") == bench.config_for("bf16_gemm_8192", 4, "multimem")
