"""Benchmark of the thork hot path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl thork|reference]

For N > 1 launch one process per GPU with torch.distributed.run; torch is
used here only for host-side plumbing (gloo barrier, max-over-ranks, NCCL
unique-id broadcast) — the measured path is thork_b200 + libthork_rt.so.

Workloads (the target configurations; default ``bf16_gemm_8192``):
  bf16_gemm_8192  C = A.B, 8192^3 bf16, A split by contiguous rows over the N
                  GPUs, B replicated, C all-gathered inside the GEMM over NVLink
                  (``--gather nccl``: NCCL all-gather after it); strong scaling
  bf16_gemm_4096  4096^3 bf16 (1 GPU config; rows split the same way at N > 1)
  e4m3_gemm_8192  8192^3 FP8 e4m3 with per-tensor scales, bf16 out, gathered
  skinny_m{1,16,128}  Y = X.W, K=4096, N=14336, bf16; W split by columns
  add_f32         out = A + B over 2^28 fp32 elements (3 GiB of traffic);
                  1024^2 (config 0) is reported under "also"

A step is one pass of the hot path over one batch of synthetic input
already resident in HBM (``value``).  ``e2e`` repeats the step through the
public API (``tk.kernels.*`` / ``thork_b200.dist``) from pinned host buffers,
host<->device copies included.  After the timed regions every rank checks
its result (``check``): a seeded row sample of the gathered C against the
oracle (covering every rank's rows), and at N > 1 the whole gathered C bit
for bit against the NCCL all-gather path; the run exits non-zero when a
check fails.  ``--impl reference`` times the reference's own CPU path (its
NumPy verification arithmetic, restated in oracle/) on a bounded sample of
the same workload, rank 0 only, with every host core.

oracle/ is imported only by the CPU legs (``cpu_baseline``, the reference
arm) and by the post-timing check, never inside a timed GPU region.
"""

import os
import sys


def _impl_from_argv(argv):
    for i, a in enumerate(argv):
        if a == "--impl" and i + 1 < len(argv):
            return argv[i + 1]
        if a.startswith("--impl="):
            return a.split("=", 1)[1]
    return "thork"


# The CPU legs use every host core.  torch.distributed.run exports
# OMP_NUM_THREADS=1, and OpenBLAS fixes its thread pool when NumPy loads, so
# the reference arm (rank 0 alone does the work) sets the counts before the
# import.  The thork arm's cpu_baseline runs at N = 1 only, without torchrun.
if _impl_from_argv(sys.argv) == "reference":
    for _v in ("OPENBLAS_NUM_THREADS", "OMP_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ[_v] = str(os.cpu_count() or 1)

import argparse  # noqa: E402
import json  # noqa: E402
import math  # noqa: E402
import statistics  # noqa: E402
import subprocess  # noqa: E402
import threading  # noqa: E402
import time  # noqa: E402

import numpy as np  # noqa: E402

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "bf16/fp8 GEMM TFLOP/s & % peak at 8192³; elementwise HBM GB/s; 1–8 GPUs"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
L2_BYTES = 126 * (1 << 20)
TOL = 1e-2  # max |C - R| / max |R| for the bf16 / e4m3 GEMMs (north_star)
CHECK_ROWS = 64


def blas_threads():
    """(threads the BLAS pool uses now, library name), via threadpoolctl."""
    try:
        from threadpoolctl import threadpool_info
        for info in threadpool_info():
            if info.get("user_api") == "blas":
                return int(info.get("num_threads", 0)), info.get("internal_api", "blas")
    except Exception:  # pragma: no cover - threadpoolctl missing or failing
        pass
    return None, None


class all_host_threads:
    """Context: let the BLAS pool use every host core (undoes an inherited
    OMP_NUM_THREADS=1), restoring the previous limit on exit."""

    def __enter__(self):
        self._ctl = None
        try:
            from threadpoolctl import threadpool_limits
            self._ctl = threadpool_limits(limits=os.cpu_count() or 1, user_api="blas")
        except Exception:  # pragma: no cover
            self._ctl = None
        return self

    def __exit__(self, *exc):
        if self._ctl is not None:
            self._ctl.restore_original_limits()
        return False


# --------------------------------------------------------------------------
# distributed plumbing
# --------------------------------------------------------------------------
class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        if self.world > 1:
            import datetime
            import torch.distributed as tdist
            tdist.init_process_group("gloo", timeout=datetime.timedelta(seconds=180))
            self.tdist = tdist

    def barrier(self):
        if self.world > 1:
            self.tdist.barrier()

    def _reduce(self, x: float, op) -> float:
        import torch
        t = torch.tensor([x], dtype=torch.float64)
        self.tdist.all_reduce(t, op=op)
        return float(t.item())

    def max(self, x: float) -> float:
        return x if self.world == 1 else self._reduce(x, self.tdist.ReduceOp.MAX)

    def min(self, x: float) -> float:
        return x if self.world == 1 else self._reduce(x, self.tdist.ReduceOp.MIN)

    def bcast_bytes(self, b):
        if self.world == 1:
            return b
        obj = [b]
        self.tdist.broadcast_object_list(obj, src=0)
        return obj[0]

    def close(self):
        if self.world > 1:
            self.tdist.destroy_process_group()


# --------------------------------------------------------------------------
# clocks during the timed region
# --------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, local_rank: int, interval_ms: int = 50):
        cvd = os.environ.get("CUDA_VISIBLE_DEVICES", "")
        ids = [x for x in cvd.split(",") if x.strip()]
        self.index = ids[local_rank] if local_rank < len(ids) else str(local_rank)
        self.interval_ms = interval_ms
        self.samples = []
        self.proc = None
        self.thread = None

    def start(self, wait_first_s: float = 5.0):
        """Start sampling and wait (bounded) for the first sample, so a short
        timed region right after this call is covered."""
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", str(self.interval_ms), "-i", self.index],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()
        t0 = time.perf_counter()
        while not self.samples and time.perf_counter() - t0 < wait_first_s:
            time.sleep(0.02)

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.samples.append((time.perf_counter(), parts))

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=5)

    def summary(self, t0: float, t1: float):
        pad = self.interval_ms / 1000.0
        inside = [p for t, p in self.samples if t0 <= t <= t1 + pad]
        if not inside and self.samples:
            inside = [min(self.samples, key=lambda s: abs(s[0] - (t0 + t1) / 2))[1]]
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}

        def num(v):
            try:
                return float(v)
            except ValueError:
                return None
        sm = [num(p[1]) for p in inside if num(p[1]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for p in inside for n, v in zip(names, p[5:9]) if v.strip() == "Active"})
        pw = [num(p[3]) for p in inside if num(p[3]) is not None]
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": num(inside[0][2]), "reasons": reasons,
                "power_w_max": max(pw) if pw else None, "samples": len(inside),
                "interval_ms": self.interval_ms}


def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return {k: float(p[k]) for k in ("hbm_gbs", "bf16_tflops", "bf16_tflops_sustained")}, "measured"
    except (OSError, KeyError, ValueError):
        return dict(FALLBACK_PEAKS), "fallback"


# --------------------------------------------------------------------------
# configurations (shared by both arms so their `config` keys are identical)
# --------------------------------------------------------------------------
GEMMS = {"bf16_gemm_8192": (8192, "bf16"), "bf16_gemm_4096": (4096, "bf16"),
         "e4m3_gemm_8192": (8192, "e4m3")}
SKINNY_N, SKINNY_K = 14336, 4096


def gemm_copies(size: int, kind: str) -> int:
    """Rotating copies of A and B so that consecutive steps never find their
    operands in L2: one copy when A + B + C already exceed twice the L2."""
    elem = 2 if kind == "bf16" else 1
    ab = 2 * size * size * elem
    if ab + size * size * 2 >= 2 * L2_BYTES:
        return 1
    return int(math.ceil(2 * L2_BYTES / ab))


def skinny_copies(n_loc: int) -> int:
    return max(3, int(math.ceil(3 * L2_BYTES / (SKINNY_K * n_loc * 2))))


def config_for(name: str, world: int, gather: str = "auto") -> dict:
    if gather == "auto":  # as FusedGather(mode="auto") resolves it on multicast-capable GPUs
        gather = "multimem" if world >= 3 else "fused"
    if name in GEMMS:
        size, kind = GEMMS[name]
        copies = gemm_copies(size, kind)
        elem = 2 if kind == "bf16" else 1
        ws = (2 * size * size * elem + size * size * 2) / (1 << 20)
        return {
            "workload": name, "M": size, "N": size, "K": size,
            "dtype_in": kind, "dtype_out": "bf16", "accumulate": "fp32",
            "parallelism": (f"A rows split over {world} GPUs, B replicated, C all-gathered "
                            + {"fused": "inside the GEMM epilogue (P2P stores over NVLink + device "
                                        "flag barrier)",
                               "multimem": "inside the GEMM epilogue (one multimem store per line "
                                           "through an NVLink multicast buffer + device flag "
                                           "barrier)",
                               "nccl": "with NCCL"}[gather]
                            if world > 1 else "1 GPU"),
            "l2_policy": (f"A + B + C = {ws:.0f} MiB > 2x L2 (126 MB): no flush needed"
                          if copies == 1 else
                          f"{copies} rotating copies of A and B "
                          f"({copies * 2 * size * size * elem / (1 << 20):.0f} MiB) > 2x L2"),
        }
    if name.startswith("skinny_m"):
        m = int(name[len("skinny_m"):])
        n_loc0 = SKINNY_N if world == 1 else (lambda r: r[1] - r[0])(
            _col_shard(SKINNY_N, world, 0))
        return {
            "workload": name, "M": m, "N": SKINNY_N, "K": SKINNY_K, "dtype_in": "bf16",
            "dtype_out": "bf16", "accumulate": "fp32",
            "parallelism": (f"W columns split over {world} GPUs, X replicated, Y not gathered"
                            if world > 1 else "1 GPU"),
            "l2_policy": f"{skinny_copies(n_loc0)} rotating copies of W (> 3x L2)",
        }
    if name == "add_f32":
        return {"workload": name, "elements": 1 << 28, "dtype_in": "fp32",
                "parallelism": f"contiguous ranges over {world} GPUs" if world > 1 else "1 GPU",
                "l2_policy": "3 GiB of traffic per step (> L2)"}
    raise SystemExit(f"unknown workload {name}")


def _col_shard(n, world, rank, align=8):
    base, extra = divmod(n // align, world)
    s = rank * base + min(rank, extra)
    return s * align, (s + base + (1 if rank < extra else 0)) * align


# --------------------------------------------------------------------------
# workloads
# --------------------------------------------------------------------------
def bf16_bits(x):
    from thork_b200 import dtypes
    return dtypes.to_bf16_bits(x)


def check_row_sample(m: int, world: int, dist_mod, total: int = CHECK_ROWS, seed: int = 1234):
    """Sorted rows of C to check: the first and last row of every rank's
    block plus seeded random rows inside it, ``total`` in all."""
    rng = np.random.default_rng(seed)
    per = max(2, total // world)
    rows = []
    for q in range(world):
        s, e = dist_mod.row_shard(m, world, q)
        pick = {s, e - 1}
        if e - s > 2:
            pick.update(int(x) for x in rng.choice(np.arange(s + 1, e - 1),
                                                   size=min(per - 2, e - s - 2), replace=False))
        rows.extend(sorted(pick))
    return np.array(sorted(set(rows)), dtype=np.int64)


class GemmWorkload:
    """bf16 / e4m3 GEMM, rows of A split over ranks, C all-gathered (fused
    into the GEMM epilogue over NVLink peer memory, or by NCCL)."""

    def __init__(self, size: int, kind: str, d: Dist, rt, dist_mod, gather: str = "fused",
                 comm=None):
        self.name = f"{kind}_gemm_{size}"
        self.m = self.n = self.k = size
        self.kind = kind
        self.d = d
        self.rt = rt
        self.dist = dist_mod
        self.start, self.stop = dist_mod.row_shard(self.m, d.world, d.rank)
        self.m_loc = self.stop - self.start
        rng = np.random.default_rng(0)
        a = rng.standard_normal((self.m, self.k), dtype=np.float32)
        b = rng.standard_normal((self.k, self.n), dtype=np.float32)
        self.chk_rows = check_row_sample(self.m, d.world, dist_mod)
        if kind == "bf16":
            self.a_host = bf16_bits(a[self.start:self.stop])
            self.b_host = bf16_bits(b)
            self.chk_a = bf16_bits(a[self.chk_rows])
            self.sa = self.sb = 1.0
        else:
            from thork_b200 import dtypes
            # per-tensor scales of the full A and B (every rank draws the same
            # inputs), then this rank's rows
            qa, self.sa = dtypes.quantize_e4m3(a)
            self.a_host = np.ascontiguousarray(qa[self.start:self.stop])
            self.chk_a = np.ascontiguousarray(qa[self.chk_rows])
            self.b_host, self.sb = dtypes.quantize_e4m3(b)
            del qa
        self.scale = float(self.sa) * float(self.sb)
        del a, b
        self.elem = self.a_host.dtype.itemsize
        self.copies = gemm_copies(size, kind)
        self.As = [rt.DeviceArray.from_host(self.a_host) for _ in range(self.copies)]
        self.Bs = [rt.DeviceArray.from_host(self.b_host) for _ in range(self.copies)]
        self.A, self.B = self.As[0], self.Bs[0]
        self.i = 0
        self.gather = gather if d.world > 1 else "none"
        rows_out = self.m if d.world > 1 else self.m_loc
        self.C = rt.empty((rows_out, self.n), np.uint16) if self.gather in ("none", "nccl") else None
        self.comm = comm
        self.own_comm = False
        self.fg = None
        if d.world > 1:
            if self.comm is None:
                uid = None
                if d.rank == 0:
                    import ctypes
                    buf = (ctypes.c_uint8 * 128)()
                    rt.check(rt.lib().thork_nccl_get_unique_id(buf))
                    uid = bytes(buf)
                uid = d.bcast_bytes(uid)
                self.comm = dist_mod.Communicator(d.rank, d.world, unique_id=uid)
                self.own_comm = True
            if self.gather in ("auto", "fused", "multimem"):
                self.fg = dist_mod.FusedGather(
                    self.comm, self.m, self.n,
                    mode={"auto": "auto", "fused": "p2p", "multimem": "multimem"}[self.gather])
                self.gather = "multimem" if self.fg.mode == "multimem" else "fused"
        # our kernels per step: the GEMM, plus the flag barrier when fused
        self.launches_per_step = 2 if self.fg is not None else 1
        self.last = None

    flops_total = property(lambda self: 2.0 * self.m * self.n * self.k)
    flops_local = property(lambda self: 2.0 * self.m_loc * self.n * self.k)
    # bytes of C one GPU sends to its peers per step (the all-gather)
    gather_bytes_per_gpu = property(lambda self: 2.0 * self.m_loc * self.n * (self.d.world - 1))

    def _operands(self):
        a, b = self.As[self.i % self.copies], self.Bs[self.i % self.copies]
        self.i += 1
        return a, b

    def step(self, stream, ev0=None, ev1=None):
        a, b = self._operands()
        if ev0 is not None:
            ev0.record(stream)
        if self.fg is not None:
            self.last = self.fg.matmul(a, b, stream, gemm_done=ev1, dtype=self.kind,
                                       scale_a=self.scale)
            return
        self.dist.sharded_matmul(self.comm, a, b, self.C, self.m, dtype=self.kind,
                                 scale=self.scale, gather=self.d.world > 1, stream=stream,
                                 gemm_done=ev1)
        self.last = self.C

    def device_barrier(self, stream):
        """Line the GPUs up on the device before a timed region: the fused
        gather's flag barrier, or an NCCL all-reduce (stream-ordered)."""
        if self.fg is not None:
            self.fg.barrier(stream)
        elif self.comm is not None:
            if getattr(self, "_bar", None) is None:
                self._bar = self.rt.empty((1,), np.float32)
            self.comm.allreduce_sum(self._bar.ptr, 1, self.dist.DT_F32, stream)

    def local_step(self, stream, ev0=None, ev1=None):
        """This rank's GEMM alone, without the all-gather (scaling reference)."""
        if getattr(self, "C_loc", None) is None:
            self.C_loc = self.rt.empty((self.m_loc, self.n), np.uint16)
        a, b = self._operands()
        if ev0 is not None:
            ev0.record(stream)
        self.dist.sharded_matmul(None, a, b, self.C_loc, self.m_loc, dtype=self.kind,
                                 scale=self.scale, gather=False, stream=stream, gemm_done=ev1)

    def check(self, stream):
        """One more step outside any timing; the sampled rows of the (gathered)
        C against the oracle, and at N > 1 the whole gathered C bit for bit
        against the NCCL all-gather path."""
        from oracle import oracle
        self.step(stream)
        stream.synchronize()
        c = self.last.to_host(stream=stream)
        rows = self.chk_rows if self.d.world > 1 else self.chk_rows[self.chk_rows < self.m_loc]
        got = oracle.bf16_bits_to_f32(c[rows - (0 if self.d.world > 1 else self.start)])
        with all_host_threads():
            if self.kind == "bf16":
                ref = oracle.gemm_bf16_ref(self.chk_a, self.b_host)
            else:
                ref = oracle.gemm_e4m3_ref(self.chk_a, self.sa, self.b_host, self.sb)
        if self.d.world == 1:
            ref = ref[np.isin(self.chk_rows, rows)]
        err = oracle.max_rel_err(got, ref)
        out = {"max_rel_err": err, "rows": int(len(rows)), "tolerance": TOL,
               "rows_from_every_rank": True,
               "oracle": "fp32 NumPy matmul of the rounded (bf16) / dequantised (e4m3) inputs"}
        if self.d.world > 1:
            c_nccl = self.rt.empty((self.m, self.n), np.uint16)
            self.dist.sharded_matmul(self.comm, self.A, self.B, c_nccl, self.m, dtype=self.kind,
                                     scale=self.scale, gather=True, stream=stream)
            stream.synchronize()
            out["bitequal_vs_nccl"] = bool(np.array_equal(c_nccl.to_host(stream=stream), c))
            del c_nccl
        else:
            out["bitequal_vs_nccl"] = None
        return out

    def e2e_setup(self):
        rt = self.rt
        self.pa = rt.pinned_empty(self.a_host.shape, self.a_host.dtype)
        self.pa[...] = self.a_host
        self.pb = rt.pinned_empty(self.b_host.shape, self.b_host.dtype)
        self.pb[...] = self.b_host
        self.pc = rt.pinned_empty((self.m_loc, self.n), np.uint16)
        # at N > 1 each rank copies its 1/N of B's rows; NVLink completes B
        b_share = self.pb.nbytes // self.d.world if self.k % self.d.world == 0 else self.pb.nbytes
        self.h2d = self.pa.nbytes + b_share
        self.d2h = self.pc.nbytes

    def e2e_step(self, tk):
        if self.d.world == 1:
            dtype = tk.dt.bfloat16 if self.kind == "bf16" else tk.dt.float8_e4m3
            mm = tk.kernels.matmul(self.m, self.n, self.k, dtype, variant="gemm_auto") \
                if self.kind == "bf16" else tk.kernels.matmul(self.m, self.n, self.k, dtype)
            if self.kind == "bf16":
                mm(self.pc, self.pa, self.pb)
            else:
                mm(self.pc, self.pa, self.pb, self.scale, 1.0)
            return
        self.dist.sharded_matmul_host(self.comm, self.pa, self.pb, self.pc, self.m,
                                      dtype=self.kind, scale=self.scale, fused=self.fg)

    def cpu_sample(self, seconds: float):
        """The reference's check (NumPy fp32 matmul of the rounded inputs) on a
        row sample of A; returns (TFLOP/s, sample description, rows)."""
        from oracle import oracle
        if self.kind == "bf16":
            a = oracle.bf16_bits_to_f32(self.a_host)
            b = oracle.bf16_bits_to_f32(self.b_host)
        else:
            a = oracle.e4m3_bits_to_f32(self.a_host)
            b = oracle.e4m3_bits_to_f32(self.b_host) * np.float32(self.scale)
        return cpu_matmul_rate(a, b, seconds)

    def close(self):
        if self.fg is not None:
            self.fg.close()
            self.fg = None
        if self.own_comm and self.comm is not None:
            self.comm.close()
            self.comm = None


def cpu_matmul_rate(a, b, seconds, max_step_s=3.0):
    """NumPy fp32 ``a @ b`` on every host core: the full ``a`` when one
    product takes under ``max_step_s``, else a power-of-two row sample.
    Returns (TFLOP/s, sample description, rows)."""
    with all_host_threads():
        rows = a.shape[0]
        t0 = time.perf_counter()
        _ = a[:min(rows, 256)] @ b
        t = time.perf_counter() - t0
        est = t * rows / min(rows, 256)
        while est > max_step_s and rows > 64:
            rows //= 2
            est /= 2
        reps = max(1, int(seconds / max(est, 1e-6)))
        t0 = time.perf_counter()
        for _ in range(reps):
            _ = a[:rows] @ b
        dt_s = time.perf_counter() - t0
    flops = 2.0 * rows * a.shape[1] * b.shape[1] * reps
    return (flops / dt_s / 1e12,
            f"{reps} x ({rows}x{a.shape[1]} @ {a.shape[1]}x{b.shape[1]}) fp32 NumPy", rows)


class SkinnyWorkload:
    """Decode GEMM Y = X.W (K=4096, N=14336); W split by columns over ranks,
    rotating copies of each W shard so no launch reads W from L2."""

    def __init__(self, m: int, d: Dist, rt, dist_mod):
        self.name = f"skinny_m{m}"
        self.m, self.n, self.k = m, SKINNY_N, SKINNY_K
        self.d, self.rt = d, rt
        c0, c1 = dist_mod.col_shard(self.n, d.world, d.rank)
        self.c0, self.n_loc = c0, c1 - c0
        rng = np.random.default_rng(0)
        w = rng.standard_normal((self.k, self.n), dtype=np.float32) * np.float32(0.02)
        x = rng.standard_normal((m, self.k), dtype=np.float32)
        self.x_host = bf16_bits(x)
        self.w_host = np.ascontiguousarray(bf16_bits(w[:, c0:c1]))
        self.X = rt.DeviceArray.from_host(self.x_host)
        self.W = [rt.DeviceArray.from_host(self.w_host) for _ in range(skinny_copies(self.n_loc))]
        self.Y = rt.empty((m, self.n_loc), np.uint16)
        self.i = 0

    bytes_local = property(lambda self: 2.0 * (self.k * self.n_loc + self.m * self.k + self.m * self.n_loc))
    bytes_total = property(lambda self: 2.0 * (self.k * self.n + self.m * self.k * self.d.world + self.m * self.n))

    def step(self, stream, ev0=None, ev1=None):
        w = self.W[self.i % len(self.W)]
        self.i += 1
        if ev0 is not None:
            ev0.record(stream)
        # decode weights: no earlier kernel writes W (THORK_SKINNY_W_STATIC)
        self.rt.check(self.rt.lib().thork_skinny_gemm_bf16_ex(
            self.X.ptr, w.ptr, self.Y.ptr, self.m, self.n_loc, self.k, 1, stream.handle))
        if ev1 is not None:
            ev1.record(stream)

    def check(self, stream):
        from oracle import oracle
        self.Y.zero(stream)
        self.step(stream)
        stream.synchronize()
        got = oracle.bf16_bits_to_f32(self.Y.to_host(stream=stream))
        with all_host_threads():
            ref = oracle.gemm_bf16_ref(self.x_host, self.w_host)
        return {"max_rel_err": oracle.max_rel_err(got, ref), "rows": self.m,
                "columns": f"{self.c0}..{self.c0 + self.n_loc} (this rank's block, all of them)",
                "tolerance": TOL, "bitequal_vs_nccl": None}

    def e2e_setup(self):
        rt = self.rt
        self.px = rt.pinned_empty(self.x_host.shape, np.uint16)
        self.px[...] = self.x_host
        self.pw = rt.pinned_empty(self.w_host.shape, np.uint16)
        self.pw[...] = self.w_host
        self.py = rt.pinned_empty((self.m, self.n_loc), np.uint16)
        self.h2d = self.px.nbytes + self.pw.nbytes
        self.d2h = self.py.nbytes

    def e2e_step(self, tk):
        tk.kernels.matmul(self.m, self.n_loc, self.k, tk.dt.bfloat16, variant="skinny",
                          static_weights=True)(self.py, self.px, self.pw)

    def cpu_sample(self, seconds):
        from oracle import oracle
        x = oracle.bf16_bits_to_f32(self.x_host)
        w = oracle.bf16_bits_to_f32(self.w_host)
        with all_host_threads():
            t0 = time.perf_counter()
            reps = 0
            while time.perf_counter() - t0 < seconds:
                _ = x @ w
                reps += 1
            dt_s = time.perf_counter() - t0
        return (self.bytes_local * reps / dt_s / 1e9,
                f"{reps} x ({self.m}x{self.k} @ {self.k}x{self.n_loc}) fp32 NumPy", None)

    def close(self):
        pass


class AddWorkload:
    """out = A + B over 2^28 fp32 elements, split by contiguous ranges."""

    def __init__(self, n_total: int, d: Dist, rt, dist_mod):
        self.name = "add_f32"
        self.n_total = n_total
        s, e = dist_mod.row_shard(n_total, d.world, d.rank)
        self.n = e - s
        self.d, self.rt = d, rt
        rng = np.random.default_rng(d.rank)
        self.a_host = rng.standard_normal(self.n, dtype=np.float32)
        self.b_host = rng.standard_normal(self.n, dtype=np.float32)
        self.A = rt.DeviceArray.from_host(self.a_host)
        self.B = rt.DeviceArray.from_host(self.b_host)
        self.C = rt.empty((self.n,), np.float32)

    bytes_local = property(lambda self: 12.0 * self.n)
    bytes_total = property(lambda self: 12.0 * self.n_total)

    def step(self, stream, ev0=None, ev1=None):
        if ev0 is not None:
            ev0.record(stream)
        self.rt.check(self.rt.lib().thork_matrix_add_f32(self.C.ptr, self.A.ptr, self.B.ptr,
                                                         self.n, stream.handle))
        if ev1 is not None:
            ev1.record(stream)

    def check(self, stream):
        from oracle import oracle
        self.C.zero(stream)
        self.step(stream)
        stream.synchronize()
        got = self.C.to_host(stream=stream)
        exact = bool(np.array_equal(got, oracle.add_ref(self.a_host, self.b_host)))
        return {"bitexact": exact, "elements": int(self.n), "max_rel_err": 0.0 if exact else 1.0,
                "tolerance": 0.0, "bitequal_vs_nccl": None}

    def e2e_setup(self):
        rt = self.rt
        self.pa = rt.pinned_empty((self.n,), np.float32)
        self.pa[...] = self.a_host
        self.pb = rt.pinned_empty((self.n,), np.float32)
        self.pb[...] = self.b_host
        self.pc = rt.pinned_empty((self.n,), np.float32)
        self.h2d = self.pa.nbytes + self.pb.nbytes
        self.d2h = self.pc.nbytes

    def e2e_step(self, tk):
        tk.kernels.matrix_add((self.n,))(self.pc, self.pa, self.pb)

    def cpu_sample(self, seconds):
        n = min(self.n, 1 << 26)
        a, b = self.a_host[:n], self.b_host[:n]
        t0 = time.perf_counter()
        reps = 0
        while time.perf_counter() - t0 < seconds:
            _ = a + b
            reps += 1
        dt_s = time.perf_counter() - t0
        return 12.0 * n * reps / dt_s / 1e9, f"{reps} x NumPy a+b over {n} fp32", None

    def close(self):
        pass


def make_workload(name, d, rt, dist_mod, gather="auto", comm=None):
    if name in GEMMS:
        size, kind = GEMMS[name]
        return GemmWorkload(size, kind, d, rt, dist_mod, gather, comm=comm)
    if name.startswith("skinny_m"):
        return SkinnyWorkload(int(name[len("skinny_m"):]), d, rt, dist_mod)
    if name == "add_f32":
        return AddWorkload(1 << 28, d, rt, dist_mod)
    raise SystemExit(f"unknown workload {name}")


def unit_of(w):
    if isinstance(w, GemmWorkload):
        return "TFLOP/s", "tensor"
    return "GB/s", "hbm"


def time_steps(w, rt, steps, warmup, d, per_launch_events=True, sample_every=10):
    """Time ``steps`` back-to-back steps with CUDA events around the whole
    run; the dominant kernel's launch duration comes from events around every
    ``sample_every``-th launch inside the same run (an event between two
    launches stops the second from starting early, so not every launch is
    bracketed)."""
    s = rt.Stream()
    for _ in range(warmup):
        w.step(s)
    s.synchronize()
    sampled = list(range(0, steps, sample_every)) if per_launch_events else []
    evs = {i: (rt.Event(), rt.Event()) for i in sampled}
    e0, e1 = rt.Event(), rt.Event()
    rt.synchronize()
    d.barrier()
    t_wall0 = time.perf_counter()
    # ranks leave the host barrier up to a millisecond apart; where steps
    # wait on each other across GPUs, a device barrier queued just before
    # the start event makes every GPU's timed region start together
    barrier = getattr(w, "device_barrier", None)
    if d.world > 1 and barrier is not None:
        barrier(s)
    e0.record(s)
    for i in range(steps):
        if i in evs:
            w.step(s, evs[i][0], evs[i][1])
        else:
            w.step(s)
    e1.record(s)
    e1.synchronize()
    t_wall1 = time.perf_counter()
    total_ms = e0.elapsed_ms(e1)
    kernel_ms = (sum(a.elapsed_ms(b) for a, b in evs.values()) / len(evs)) if evs else total_ms / steps
    rt.synchronize()
    d.barrier()
    return total_ms, kernel_ms, t_wall0, t_wall1


def checked(d, chk):
    """Combine one check over ranks: worst error, and bit-equality on all."""
    chk = dict(chk)
    chk["max_rel_err"] = d.max(float(chk.get("max_rel_err", 0.0)))
    if chk.get("bitequal_vs_nccl") is not None:
        chk["bitequal_vs_nccl"] = d.min(1.0 if chk["bitequal_vs_nccl"] else 0.0) == 1.0
    if "bitexact" in chk:
        chk["bitexact"] = d.min(1.0 if chk["bitexact"] else 0.0) == 1.0
    chk["max_rel_err"] = float(f"{chk['max_rel_err']:.3e}")
    chk["ranks"] = d.world
    chk["pass"] = (chk["max_rel_err"] <= chk.get("tolerance", TOL)
                   and chk.get("bitequal_vs_nccl") is not False
                   and chk.get("bitexact", True) is not False)
    return chk


def run_thork(args, d: Dist):
    import thork_b200 as tk
    from thork_b200 import dist as dist_mod
    rt = tk.runtime
    rt.set_device(d.local_rank)
    peaks, peak_src = load_peaks()
    sampler = ClockSampler(d.local_rank)
    sampler.start()
    w = make_workload(args.workload, d, rt, dist_mod, args.gather)
    cfg = config_for(args.workload, d.world,
                     w.gather if isinstance(w, GemmWorkload) and d.world > 1 else args.gather)
    unit, bound = unit_of(w)

    total_ms, kernel_ms, tw0, tw1 = time_steps(w, rt, args.steps, args.warmup, d)
    clocks = sampler.summary(tw0, tw1)
    ms_step = d.max(total_ms / args.steps)

    if unit == "TFLOP/s":
        value = w.flops_total / (ms_step * 1e-3) / 1e12
        achieved = w.flops_local / (kernel_ms * 1e-3) / 1e12
        # a timed region over ~0.5 s runs under the 1 kW power cap: compare with
        # the sustained cuBLAS figure; shorter regions with the burst figure
        sustained = total_ms > 500.0
        base_peak = peaks["bf16_tflops_sustained" if sustained else "bf16_tflops"]
        kind = "sustained" if sustained else "burst"
        peak = base_peak * (2.0 if w.kind == "e4m3" else 1.0)
        peak_note = (f"{peak_src} bf16 {kind} (cuBLAS)" if w.kind == "bf16"
                     else f"2 x {peak_src} bf16 {kind} (no measured FP8 peak)")
        alg = f"2*M_local*N*K = {w.flops_local:.4g} FLOP per launch"
    else:
        value = w.bytes_total / (ms_step * 1e-3) / 1e9
        achieved = w.bytes_local / (kernel_ms * 1e-3) / 1e9
        peak = peaks["hbm_gbs"]
        peak_note = f"{peak_src} HBM copy"
        alg = f"{w.bytes_local:.4g} algorithmic bytes per launch"

    # end to end through the public API, pinned host buffers, copies included
    w.e2e_setup()
    e2e_steps = max(2, min(args.steps, 10))
    w.e2e_step(tk)
    rt.synchronize()
    d.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        w.e2e_step(tk)
    e2e_s = d.max((time.perf_counter() - t0) / e2e_steps)
    if unit == "TFLOP/s":
        e2e_val = w.flops_total / e2e_s / 1e12
    else:
        e2e_val = w.bytes_total / e2e_s / 1e9

    line = {
        "metric": METRIC, "value": round(value, 2), "unit": unit, "n_gpus": d.world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 5),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": {"bf16_gemm_8192": "bf16", "bf16_gemm_4096": "bf16", "e4m3_gemm_8192": "e4m3"}.get(
            args.workload, "bf16" if args.workload.startswith("skinny") else "f32"),
        "data": "synthetic: seeded N(0,1) inputs (target shapes and distributions), host-rounded",
        "config": cfg,
        "roofline": {"bound": bound, "achieved": round(achieved, 2), "peak": round(peak, 1),
                     "unit": unit, "frac": round(achieved / peak, 4),
                     "traffic": None, "peak_source": peak_note, "algorithmic": alg,
                     "kernel_ms": round(kernel_ms, 5)},
        "e2e": {"value": round(e2e_val, 3), "unit": unit, "h2d_bytes_per_step": int(w.h2d),
                "d2h_bytes_per_step": int(w.d2h), "steps": e2e_steps,
                "api": "tk.kernels.matmul/matrix_add" if d.world == 1 else "thork_b200.dist.sharded_matmul_host"},
        "gpu_launches": args.steps * getattr(w, "launches_per_step", 1),
        "clocks": clocks,
    }
    if isinstance(w, GemmWorkload) and d.world > 1:
        # the same sharded GEMM without gathering C, for scaling with and without the gather
        import types
        loc_ms, _, _, _ = time_steps(types.SimpleNamespace(step=w.local_step), rt, args.steps,
                                     args.warmup, d, per_launch_events=False)
        loc_step = d.max(loc_ms / args.steps)
        gb = w.gather_bytes_per_gpu
        line["without_gather"] = {
            "value": round(w.flops_total / (loc_step * 1e-3) / 1e12, 2), "unit": unit,
            "ms_per_step": round(loc_step, 5),
            "gather_ms_per_step": round(ms_step - loc_step, 5),
            "gather_bytes_per_gpu": int(gb),
            # what each GPU pushes over NVLink per step, over the whole step and
            # over the part of the step the gather adds to the GEMM
            "gather_GBps_per_gpu": round(gb / (ms_step * 1e-3) / 1e9, 1),
            "gather_GBps_per_gpu_exposed": (round(gb / ((ms_step - loc_step) * 1e-3) / 1e9, 1)
                                            if ms_step > loc_step else None),
        }
    line["check"] = checked(d, w.check(rt.Stream()))
    if d.rank == 0 and d.world == 1:
        v, sample, _ = w.cpu_sample(args.cpu_seconds)
        nthreads, blas = blas_threads()
        line["cpu_baseline"] = {"value": round(v, 4), "unit": unit, "cores": os.cpu_count(),
                                "kind": "port", "sample": sample,
                                "threads": os.cpu_count() if unit == "TFLOP/s" else 1,
                                "blas": blas}
    if args.also:
        line["also"] = also_measurements(args, d, rt, dist_mod, peaks, main=w, sampler=sampler,
                                         ms_step=ms_step)
    sampler.stop()
    traffic = traffic_from_profiles(args.workload) if d.world == 1 else None
    if traffic is not None:
        line["roofline"]["traffic"] = traffic
    w.close()
    failed = [k for k, v in [("main", line["check"])] + [
        (k, v.get("check")) for k, v in line.get("also", {}).items() if isinstance(v, dict)]
        if v is not None and not v.get("pass", True)]
    if failed:
        line["check_failed"] = failed
    if d.rank == 0:
        print(json.dumps(line), flush=True)
    return 1 if failed else 0


def _also_entry(w, d, rt, peaks, steps):
    total_ms, kernel_ms, _, _ = time_steps(w, rt, steps, 10, d, per_launch_events=False)
    ms = d.max(kernel_ms)
    if isinstance(w, GemmWorkload):
        v = w.flops_total / (ms * 1e-3) / 1e12
        peak = peaks["bf16_tflops"] * (2.0 if w.kind == "e4m3" else 1.0) * d.world
        out = {"TFLOP/s": round(v, 1), "frac_of_peak": round(v / peak, 3), "ms": round(ms, 4),
               "peak": (f"{d.world} x " if d.world > 1 else "")
               + ("2 x measured bf16 burst (no measured FP8 peak)" if w.kind == "e4m3"
                  else "measured bf16 burst"),
               "l2_policy": config_for(w.name, d.world)["l2_policy"]}
    else:
        v = w.bytes_total / (ms * 1e-3) / 1e9
        per_gpu = w.bytes_local / (kernel_ms * 1e-3) / 1e9
        out = {"GB/s": round(v, 1), "us": round(ms * 1e3, 2),
               "GB/s_per_gpu": round(per_gpu, 1),
               "frac_of_hbm": round(d.min(per_gpu) / peaks["hbm_gbs"], 3)}
    out["check"] = checked(d, w.check(rt.Stream()))
    return out


def also_measurements(args, d, rt, dist_mod, peaks, main=None, sampler=None, ms_step=None):
    """Short device-resident timings of the other target configurations.  At
    N = 1: every config, a sustained run of the headline GEMM, config 0 and
    the traced tile matmul.  At N > 1: the multi-GPU configs (FP8 8192^3 with
    the fused all-gather, decode GEMMs with W split by columns)."""
    out = {}
    if d.world == 1:
        plan = (("e4m3_gemm_8192", 100), ("bf16_gemm_4096", 200), ("skinny_m1", 300),
                ("skinny_m16", 300), ("skinny_m128", 300), ("add_f32", 100))
    else:
        plan = (("e4m3_gemm_8192", 100), ("skinny_m1", 300), ("skinny_m16", 300),
                ("skinny_m128", 300))
    comm = main.comm if isinstance(main, GemmWorkload) else None
    for name, steps in plan:
        w = make_workload(name, d, rt, dist_mod, gather=args.gather, comm=comm)
        out[name] = _also_entry(w, d, rt, peaks, steps)
        w.close()
        del w
    if d.world > 1:
        return out
    if isinstance(main, GemmWorkload) and ms_step:
        out[main.name + "_sustained"] = sustained_run(main, rt, d, peaks, sampler, ms_step)
    # config 0: 1024 x 1024 fp32 add of the config's seeded N(0,1) arrays
    # (12.6 MB, L2-resident; latency-bound)
    from oracle import oracle
    ah, bh = oracle.add_inputs((1024, 1024), seed=0)
    a, b = rt.to_device(ah), rt.to_device(bh)
    c = rt.empty((1024, 1024), np.float32)
    s = rt.Stream()
    e0, e1 = rt.Event(), rt.Event()
    for _ in range(10):
        rt.lib().thork_matrix_add_f32(c.ptr, a.ptr, b.ptr, 1 << 20, s.handle)
    e0.record(s)
    for _ in range(200):
        rt.lib().thork_matrix_add_f32(c.ptr, a.ptr, b.ptr, 1 << 20, s.handle)
    e1.record(s)
    e1.synchronize()
    us = e0.elapsed_ms(e1) / 200 * 1e3
    exact = bool(np.array_equal(c.to_host(stream=s), oracle.add_ref(ah, bh)))
    out["add_f32_1024x1024"] = {"GB/s": round(12 * (1 << 20) / us / 1e3, 1), "us": round(us, 2),
                                "note": "L2-resident, launch-latency bound",
                                "check": {"bitexact": exact, "max_rel_err": 0.0 if exact else 1.0,
                                          "tolerance": 0.0, "pass": exact}}
    # the same config through the drop-in call with NumPy arrays (copy-in, launch, copy-back)
    import thork_b200 as tk
    ch = np.empty_like(ah)
    add = tk.kernels.matrix_add((1024, 1024))
    for _ in range(5):
        add(ch, ah, bh)
    t0 = time.perf_counter()
    for _ in range(50):
        add(ch, ah, bh)
    call_us = (time.perf_counter() - t0) / 50 * 1e6
    out["add_f32_1024x1024_dropin"] = {"us_per_call": round(call_us, 1),
                                       "note": "kernel(out, a, b) on pageable NumPy arrays"}
    out["traced_tile_gemm_4096"] = traced_tile_gemm(tk, rt, peaks)
    for ncta in (1, 2):
        out[f"traced_tile_matmul_4096_{ncta}cta"] = traced_tile_matmul(tk, rt, peaks, ncta)
    out["traced_tile_matmul_4096_persistent"] = traced_tile_matmul(tk, rt, peaks, 1, persistent=True)
    return out


def traced_tile_matmul(tk, rt, peaks, ncta, size=4096, persistent=False):
    """tk.kernels.tile_matmul: the warp-specialised tcgen05 pipeline written
    with tk.kittens (1-CTA 128x256 tiles, or cluster pairs with
    cta_group::2 256x256 tiles), device-resident, CUDA-event timed."""
    m = n = k = size
    rng = np.random.default_rng(0)
    a_h = bf16_bits(rng.standard_normal((m, k), dtype=np.float32))
    b_h = bf16_bits(rng.standard_normal((k, n), dtype=np.float32))
    A, B = rt.to_device(a_h), rt.to_device(b_h)
    D = rt.empty((m, n), np.uint16)
    # the same rotation as the library's bf16_gemm_4096 line: A + B + C fit L2
    copies = gemm_copies(size, "bf16")
    rot = [(D, rt.to_device(a_h), rt.to_device(b_h)) for _ in range(copies - 1)]
    mm = tk.kernels.tile_matmul(m, n, k, ncta=ncta, persistent=persistent)
    mm(D, A, B)  # trace + NVRTC compile
    out = time_traced(mm, (D, A, B), rt, 2.0 * m * n * k, peaks,
                      f"tk.kernels.tile_matmul(ncta={ncta}, persistent={persistent}): traced "
                      "warp-specialised pipeline", rotate=rot)
    out["check"] = check_gemm_rows(D, A, B, rt)
    return out


def sustained_run(w, rt, d, peaks, sampler, ms_step, seconds=2.5):
    """The headline GEMM back to back for ``seconds`` (CUDA events around the
    run, clocks sampled inside it): the number under the 1 kW power cap."""
    steps = max(100, int(seconds * 1e3 / max(ms_step, 1e-3)))
    total_ms, _, t0, t1 = time_steps(w, rt, steps, 10, d, per_launch_events=False)
    clocks = sampler.summary(t0, t1) if sampler is not None else None
    v = w.flops_total / (total_ms / steps * 1e-3) / 1e12
    return {"TFLOP/s": round(v, 1), "steps": steps, "seconds": round(total_ms / 1e3, 3),
            "frac_of_sustained_peak": round(v / peaks["bf16_tflops_sustained"], 3),
            "peak": "measured bf16 sustained (cuBLAS, seconds-long loop)", "clocks": clocks}


def traced_tile_gemm(tk, rt, peaks, size=4096):
    """A user-written @tk.jit tile matmul in the style of the reference's
    level-06 tcgen05 test kernel (one 128x128 output tile per CTA, a
    single-stage TMA -> tcgen05.mma loop, TMEM -> registers -> shared -> TMA
    store), timed device-resident with CUDA events on the launch stream: the
    traced tile path, not the library GEMM."""
    G = tk.kittens.Global
    bf = tk.dt.bfloat16
    TM, TN, TK = 128, 128, 64

    @tk.jit
    def tile_mm(A: G[bf, (TM, TK)], B: G[bf, (TK, TN)], D: G[bf, (TM, TN)], K: tk.Uint,
                N: tk.Uint, bid: tk.Uint[tk.BlockIdx], tid: tk.Uint[tk.ThreadIdx]):
        lane = tk.kittens.warpgroup.laneid()
        bm = bid // (N // TN)
        bn = bid % (N // TN)
        a_s = tk.kittens.st_bf(TM, TK)
        b_s = tk.kittens.st_bf(TK, TN)
        d_s = tk.kittens.st_bf(TM, TN)
        arrived = tk.kittens.semaphore()
        consumed = tk.kittens.semaphore()
        done = tk.kittens.semaphore()
        with tk.if_(tid == 0):
            tk.kittens.init_semaphore(arrived, 0, 1)
            tk.kittens.init_semaphore(consumed, 1, 0)
            tk.kittens.init_semaphore(done, 0, 1)
        tk.syncthreads()
        alloc = tk.kittens.tensor_allocator()
        acc = tk.kittens.tt_fl(TM, TN)
        with tk.if_(lane == 0):
            tk.kittens.tensor_alloc(acc, alloc, 0)
        tk.kittens.warpgroup.sync(1)
        phase = tk.local(tk.dt.int32, 0)
        for it in tk.range(K // TK):
            with tk.if_(tid == 0):
                tk.kittens.wait(consumed, phase ^ 1)
                tk.kittens.tma.expect_bytes(arrived, (TM * TK + TK * TN) * 2)
                tk.kittens.tma.load_async(a_s, A, (bm, it), arrived)
                tk.kittens.tma.load_async(b_s, B, (it, bn), arrived)
            tk.kittens.wait(arrived, phase)
            phase ^= 1
            with tk.if_(lane == 0):
                with tk.if_(it == 0) as first:
                    tk.kittens.warpgroup.mm_AB(acc, a_s, b_s, consumed)
                with first.else_():
                    tk.kittens.warpgroup.mma_AB(acc, a_s, b_s, consumed)
        with tk.if_(lane == 0):
            tk.kittens.tcgen05_commit(done)
        tk.kittens.wait(done, 0)
        d_r = tk.kittens.rt_bf(TM // 4, TN)
        tk.kittens.warpgroup.load_async(d_r, acc)
        tk.kittens.tensor_load_wait()
        tk.kittens.warpgroup.sync(1)
        tk.kittens.warpgroup.store(d_s, d_r)
        tk.kittens.warpgroup.sync(1)
        with tk.if_(lane == 0):
            tk.kittens.tma.store_async(D, d_s, (bm, bn))
            tk.kittens.tma.store_async_read_wait()

    m = n = k = size
    rng = np.random.default_rng(0)
    a_h = bf16_bits(rng.standard_normal((m, k), dtype=np.float32))
    b_h = bf16_bits(rng.standard_normal((k, n), dtype=np.float32))
    A, B = rt.to_device(a_h), rt.to_device(b_h)
    D = rt.empty((m, n), np.uint16)
    copies = gemm_copies(size, "bf16")
    rot = [(rt.to_device(a_h), rt.to_device(b_h), D, k, n) for _ in range(copies - 1)]
    launch = tile_mm[((m // TM) * (n // TN), 1, 1), (128, 1, 1)]
    launch(A, B, D, k, n)  # trace + NVRTC compile
    out = time_traced(launch, (A, B, D, k, n), rt, 2.0 * m * n * k, peaks,
                      "reference level-06 style: single stage, 128x128 tile per CTA", rotate=rot)
    out["check"] = check_gemm_rows(D, A, B, rt)
    return out


def check_gemm_rows(D, A, B, rt, nrows=CHECK_ROWS):
    """Seeded rows of a bf16 C = A.B on the device against the oracle."""
    from oracle import oracle
    m = D.shape[0]
    rows = np.sort(np.random.default_rng(99).choice(m, size=min(nrows, m), replace=False))
    a = A.to_host()[rows]
    with all_host_threads():
        ref = oracle.gemm_bf16_ref(a, B.to_host())
    err = oracle.max_rel_err(oracle.bf16_bits_to_f32(D.to_host()[rows]), ref)
    return {"max_rel_err": float(f"{err:.3e}"), "rows": int(len(rows)), "tolerance": TOL,
            "pass": err <= TOL}


def time_traced(launch, args, rt, flops, peaks, note, reps=50, rotate=()):
    """Device time of a traced kernel: its device-resident arguments packed
    once (``prepare``), ``reps`` launches queued back to back on one stream,
    CUDA events around them.  ``rotate`` holds further argument tuples (copies
    of the inputs) that the launches cycle through, so that consecutive
    launches do not find their operands in L2.  The synchronous drop-in call
    (argument packing, launch, synchronise) is timed beside it on the host."""
    s = rt.Stream()
    prepared = [launch.prepare(*a) for a in (args,) + tuple(rotate)]
    for i in range(5):
        prepared[i % len(prepared)].launch(s)
    s.synchronize()
    e0, e1 = rt.Event(), rt.Event()
    e0.record(s)
    for i in range(reps):
        prepared[i % len(prepared)].launch(s)
    e1.record(s)
    e1.synchronize()
    ms = e0.elapsed_ms(e1) / reps
    t0 = time.perf_counter()
    for _ in range(5):
        launch(*args)
    call_ms = (time.perf_counter() - t0) / 5 * 1e3
    tf = flops / (ms * 1e-3) / 1e12
    return {"TFLOP/s": round(tf, 1), "ms": round(ms, 4),
            "frac_of_peak": round(tf / peaks["bf16_tflops"], 3), "note": note,
            "timing": f"{reps} prepared launches back to back, CUDA events",
            "l2_policy": (f"{len(prepared)} rotating copies of the inputs" if len(prepared) > 1
                          else "one copy of the inputs (L2-warm)"),
            "dropin_call_ms": round(call_ms, 4),
            "status": rt.kernel_status()}


def traffic_from_profiles(workload):
    """Per-launch DRAM bytes recorded from an ncu capture (profiles/*.json)."""
    path = os.path.join(REPO, "profiles", "traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get(workload)
    except (OSError, ValueError):
        return None


def run_reference(args, d: Dist):
    """The reference's CPU path (NumPy verification arithmetic), rank 0 only,
    every host core; the same problem at every N (the CPU does the whole job)."""
    if d.rank != 0:
        return 0
    from oracle import oracle
    name = args.workload
    steps = args.steps + args.warmup
    nthreads, blas = blas_threads()
    if name in GEMMS:
        size, kind = GEMMS[name]
        a, b = oracle.gemm_inputs(size, size, size, seed=0)
        if kind == "e4m3":
            qa, sa = oracle.quantize_e4m3(a)
            qb, sb = oracle.quantize_e4m3(b)
            a = oracle.e4m3_bits_to_f32(qa) * sa
            b = oracle.e4m3_bits_to_f32(qb) * sb
        else:
            a, b = oracle.round_bf16(a), oracle.round_bf16(b)
        # the whole product per step unless one takes over ~90 s / steps
        _, _, rows = cpu_matmul_rate(a, b, 0.0, max_step_s=max(0.05, min(3.0, 90.0 / steps)))
        times = []
        for i in range(steps):
            t0 = time.perf_counter()
            _ = a[:rows] @ b
            times.append(time.perf_counter() - t0)
        t = statistics.median(times[args.warmup:] or times)
        value, unit = 2.0 * rows * size * size / t / 1e12, "TFLOP/s"
        sample = (f"rows 0..{rows} of A ({rows}x{size} @ {size}x{size}) fp32 NumPy per step"
                  + (" (the whole product)" if rows == size else ""))
    elif name.startswith("skinny_m"):
        m = int(name[len("skinny_m"):])
        x, w = oracle.skinny_inputs(m, SKINNY_N, SKINNY_K, seed=0)
        x, w = oracle.round_bf16(x), oracle.round_bf16(w)
        times = []
        for _ in range(steps):
            t0 = time.perf_counter()
            _ = x @ w
            times.append(time.perf_counter() - t0)
        t = statistics.median(times[args.warmup:] or times)
        value, unit = 2.0 * (SKINNY_K * SKINNY_N + m * SKINNY_K + m * SKINNY_N) / t / 1e9, "GB/s"
        sample = f"full ({m}x{SKINNY_K} @ {SKINNY_K}x{SKINNY_N}) fp32 NumPy per step"
    else:
        n = 1 << 26
        a, b = oracle.add_inputs((n,), seed=0)
        times = []
        for _ in range(steps):
            t0 = time.perf_counter()
            _ = oracle.add_ref(a, b)
            times.append(time.perf_counter() - t0)
        t = statistics.median(times[args.warmup:] or times)
        value, unit = 12.0 * n / t / 1e9, "GB/s"
        sample = f"NumPy a+b over {n} fp32 (2^26 of the 2^28 elements) per step"
        nthreads = 1
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": unit,
        "n_gpus": d.world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(t * 1e3, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None,
        "dtype": {"bf16_gemm_8192": "bf16", "bf16_gemm_4096": "bf16", "e4m3_gemm_8192": "e4m3"}.get(
            name, "bf16" if name.startswith("skinny") else "f32"),
        "data": "synthetic: seeded N(0,1) inputs (target shapes and distributions), host-rounded",
        # the same config as the thork arm at this N (the CPU computes the whole job)
        "config": config_for(name, d.world, args.gather),
        "cpu_baseline": {"value": round(value, 4), "unit": unit, "cores": os.cpu_count(),
                         "threads": nthreads, "blas": blas, "kind": "port", "sample": sample,
                         "compute": "fp32 NumPy on the host (the reference's verification path)"},
        "e2e": {"value": round(value, 4), "unit": unit, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1500)
    ap.add_argument("--warmup", type=int, default=30)
    ap.add_argument("--workload", default="bf16_gemm_8192")
    ap.add_argument("--impl", default="thork", choices=["thork", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--gather", default="auto", choices=["auto", "fused", "multimem", "nccl"],
                    help="multi-GPU GEMM: all-gather fused into the epilogue (P2P stores, or "
                         "multimem stores through an NVLink multicast buffer; auto: multimem "
                         "from 3 GPUs where supported), or NCCL after it")
    ap.add_argument("--no-also", dest="also", action="store_false",
                    help="omit the short timings of the other configs")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    d = Dist()
    if d.world != args.gpus:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE={d.world}", file=sys.stderr)
    rc = 0
    try:
        if args.impl == "reference":
            rc = run_reference(args, d)
        else:
            rc = run_thork(args, d)
    finally:
        d.close()
    if rc:
        print("bench: a result check failed (see check_failed in the JSON line)", file=sys.stderr)
    sys.exit(rc)


if __name__ == "__main__":
    main()
