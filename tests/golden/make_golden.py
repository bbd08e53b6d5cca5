"""Generate the golden fixtures under tests/golden/ from the reference.

Run in a container that has the reference checkout (read-only) and
ml_dtypes::

    python tests/golden/make_golden.py /path/to/reference

The reference is Python, so it is imported from its source tree (nothing is
copied into this repository).  Outputs:

* ``bf16_rne.npz``  — float32 inputs and the reference's own
  ``_f32_to_bf16_u16`` (``tests/test_kittens.py:20-28``) applied to them,
  plus the round trip through ``_bf16_u16_to_f32`` (``31-36``).
* ``e4m3_sweep.npz`` — float32 inputs and ml_dtypes ``float8_e4m3fn`` bytes
  (the third-party format the FP8 path follows; the reference has no FP8).
* ``reference_validation.json`` — exception type and message the
  reference's argument checks (``src/thork/runtime.py:431-480``) raise for
  bad NumPy arguments.
* ``reference_traces.json`` — for every kernel of tests/kernel_zoo.py, the
  reference trace's parameter list (name, kind, dtype, written).
"""

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def main(ref_root: str) -> None:
    sys.path.insert(0, os.path.join(ref_root, "src"))
    sys.path.insert(0, os.path.join(ref_root, "tests"))
    sys.path.insert(0, os.path.join(REPO, "tests"))
    import ml_dtypes
    import thork as ref_tk
    from thork import ir as ref_ir
    from thork import runtime as ref_rt
    import test_kittens as ref_tests
    import kernel_zoo

    # ---- bf16 rounding (reference helpers)
    rng = np.random.default_rng(2024)
    parts = [
        rng.standard_normal(4096).astype(np.float32),
        (rng.standard_normal(4096) * 1e-3).astype(np.float32),
        (rng.standard_normal(2048) * 1e30).astype(np.float32),
        rng.integers(0, 2 ** 32, 8192, dtype=np.uint64).astype(np.uint32).view(np.float32),
    ]
    # exact ties, neighbours of ties, subnormals, extremes
    base = rng.integers(0, 2 ** 15, 1024, dtype=np.uint32) << np.uint32(16)
    for delta in (0x8000, 0x7FFF, 0x8001, 0x18000):
        parts.append((base + np.uint32(delta)).view(np.float32))
    parts.append(np.array([0.0, -0.0, 1e-45, -1e-45, 1.17549435e-38, 3.4028235e38,
                           -3.4028235e38, 3.3961776e38, 3.3961778e38, np.inf, -np.inf, 1.0, -1.0,
                           0.1, 65504.0], np.float32))
    x = np.concatenate(parts).astype(np.float32)
    finite = np.isfinite(x)
    x = x[finite | np.isinf(x)]  # NaN payloads are excluded (the helper wraps them)
    bits = ref_tests._f32_to_bf16_u16(x)
    back = ref_tests._bf16_u16_to_f32(bits)
    np.savez_compressed(os.path.join(HERE, "bf16_rne.npz"), x_bits=x.view(np.uint32),
                        bf16_bits=bits, widened_bits=back.view(np.uint32))

    # ---- e4m3 (ml_dtypes)
    vals = [rng.standard_normal(8192).astype(np.float32) * 100,
            rng.uniform(-464, 464, 8192).astype(np.float32),
            (rng.standard_normal(4096) * 2.0 ** -8).astype(np.float32)]
    grid = ml_dtypes.finfo(ml_dtypes.float8_e4m3fn)
    codes = np.arange(256, dtype=np.uint8).view(ml_dtypes.float8_e4m3fn).astype(np.float32)
    codes = codes[np.isfinite(codes)]
    mids = np.sort(np.unique(codes))
    vals += [codes, ((mids[1:] + mids[:-1]) / 2).astype(np.float32)]
    e = np.concatenate(vals).astype(np.float32)
    e = e[np.abs(e) <= 464]
    np.savez_compressed(os.path.join(HERE, "e4m3_sweep.npz"), x=e,
                        e4m3_bits=e.astype(ml_dtypes.float8_e4m3fn).view(np.uint8),
                        max_finite=np.float32(grid.max))

    # ---- argument validation
    f32p = ref_ir.Param(name="A", kind="pointer", dtype=ref_tk.dt.float32)
    glp = ref_ir.Param(name="G", kind="kittens_global", dtype=ref_tk.dt.bfloat16)
    cases = {
        "pointer_not_array": (ref_rt._expect_pointer_arg, [1.0, 2.0], f32p),
        "pointer_wrong_dtype": (ref_rt._expect_pointer_arg, np.zeros(4, np.int32), f32p),
        "pointer_unmapped_dtype": (ref_rt._expect_pointer_arg, np.zeros(4, np.float64), f32p),
        "pointer_non_contiguous": (ref_rt._expect_pointer_arg, np.zeros((4, 4), np.float32)[:, 1], f32p),
        "global_not_array": (ref_rt._expect_kittens_arg, "x", glp),
        "global_not_2d": (ref_rt._expect_kittens_arg, np.zeros(8, np.uint16), glp),
        "global_itemsize": (ref_rt._expect_kittens_arg, np.zeros((4, 4), np.float32), glp),
        "global_non_contiguous": (ref_rt._expect_kittens_arg, np.zeros((4, 8), np.uint16)[:, ::2], glp),
    }
    out = {}
    for name, (fn, arg, p) in cases.items():
        try:
            fn(arg, p)
            out[name] = {"type": None, "message": None}
        except Exception as exc:  # noqa: BLE001 - recording the reference's behaviour
            out[name] = {"type": type(exc).__name__, "message": str(exc)}
    with open(os.path.join(HERE, "reference_validation.json"), "w") as f:
        json.dump(out, f, indent=1, sort_keys=True)

    # ---- traces
    traces = {}
    for group in (kernel_zoo.build(ref_tk), kernel_zoo.build_tiles(ref_tk)):
        for name, k in group.items():
            k.cuda_source  # trace + emit
            params = [{"name": p.name, "kind": p.kind, "dtype": p.dtype.name, "written": p.written}
                      for p in k._builder.params]
            traces[name] = {"params": params}
    with open(os.path.join(HERE, "reference_traces.json"), "w") as f:
        json.dump(traces, f, indent=1, sort_keys=True)
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <reference checkout>")
    main(sys.argv[1])
