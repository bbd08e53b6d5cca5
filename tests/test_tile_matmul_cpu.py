"""CPU checks of the cluster-pair tile API and tk.kernels.tile_matmul: both
forms trace and compile for sm_100a through NVRTC, a pair kernel refuses a
launch without its cluster before anything is compiled or launched.""" 

import numpy as np
import pytest

import thork_b200 as tk


@pytest.mark.parametrize("ncta", [1, 2])
def test_tile_matmul_compiles_for_sm100a(ncta):
    mm = tk.kernels.tile_matmul(512, 512, 1024, ncta=ncta)
    kern = mm.kernel._kernel
    assert kern.cluster_ctas == ncta
    assert kern.dynamic_smem <= 227 * 1024
    src = mm.cuda_source
    if ncta == 2:
        assert "tmem_acquire2" in src and "mma2_AB" in src and "tma::pair::load_async" in src
    kern.compile_for_arch("100a")


def test_pair_kernel_needs_cluster_launch():
    mm = tk.kernels.tile_matmul(256, 256, 64, ncta=2)
    kern = mm.kernel._kernel
    a = np.zeros((256, 64), np.uint16)
    b = np.zeros((64, 256), np.uint16)
    c = np.zeros((256, 256), np.uint16)
    with pytest.raises(ValueError, match=r"\(2, 1, 1\)"):
        kern[(2, 1, 1), (192, 1, 1)](a, b, c, 64, 256)
    with pytest.raises(ValueError, match="multiple of the cluster"):
        kern[(3, 1, 1), (192, 1, 1), (2, 1, 1)](a, b, c, 64, 256)


def test_tile_matmul_shape_errors():
    with pytest.raises(ValueError):
        tk.kernels.tile_matmul(100, 256, 64)
    with pytest.raises(ValueError):
        tk.kernels.tile_matmul(128, 256, 96)
    with pytest.raises(ValueError):
        tk.kernels.tile_matmul(128, 256, 64, ncta=2)  # pair tiles are 256 rows
    with pytest.raises(ValueError):
        tk.kernels.tile_matmul(256, 256, 64, ncta=3)


def test_pair_mma_needs_pair_allocator():
    kt = tk.kittens
    G = kt.Global
    bf = tk.dt.bfloat16

    @tk.jit
    def bad(A: G[bf, (128, 64)], B: G[bf, (64, 128)]):
        a_s = kt.st_bf(128, 64)
        b_s = kt.st_bf(64, 128)
        sem = kt.semaphore()
        alloc = kt.tensor_allocator()  # one CTA's tensor memory
        acc = kt.tt_fl(128, 256)
        kt.tensor_alloc(acc, alloc, 0)
        kt.warpgroup.mm2_AB(acc, a_s, b_s, sem)

    with pytest.raises(TypeError, match="ncta=2"):
        bad.cuda_source


def test_tensor_to_shared_store_checks_shapes():
    kt = tk.kittens
    G = kt.Global
    bf = tk.dt.bfloat16

    @tk.jit
    def bad(A: G[bf, (128, 64)]):
        d_s = kt.st_bf(64, 64)
        alloc = kt.tensor_allocator()
        acc = kt.tt_fl(128, 128)
        kt.tensor_alloc(acc, alloc, 0)
        kt.warpgroup.store(d_s, acc)

    with pytest.raises(TypeError, match="store\\(shared, tensor\\)"):
        bad.cuda_source


def test_persistent_tile_matmul_compiles_and_checks_shapes():
    mm = tk.kernels.tile_matmul(2048, 4096, 512, persistent=True)
    kern = mm.kernel._kernel
    assert "arrive" in mm.cuda_source and kern.dynamic_smem <= 227 * 1024
    kern.compile_for_arch("100a")
    with pytest.raises(ValueError):
        tk.kernels.tile_matmul(256, 256, 192, persistent=True)  # K/64 not a multiple of 4
    with pytest.raises(ValueError):
        tk.kernels.tile_matmul(256, 256, 256, ncta=2, persistent=True)
