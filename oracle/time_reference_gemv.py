"""ORACLE — test infrastructure only. Times the reference's own CPU GEMV beside the
oracle's C port, on the six GEMV sweep shapes, where the reference's checkout is
present (HIVE_REFERENCE, as tests/golden/make_golden.py): `reference.gemv_w4` (numpy:
it unpacks the int4 weights to int32 on every call, then einsum and the pairwise sum)
and `hv_oracle.gemv_w4_c` (the C restatement, OpenMP over the host's cores), with a bit
comparison of their outputs. Prints one line per shape: milliseconds per call and GB/s
of the algorithmic 0.625 B per weight.

    python oracle/time_reference_gemv.py
"""
import os
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path[:0] = [str(HERE.parent / "tests" / "golden"), str(HERE),
                str(HERE.parent / "hive-limited_b200")]

import hv_oracle as O    # noqa: E402
import make_golden       # noqa: E402
import synth             # noqa: E402


def main():
    ref_limited, ref = make_golden.load_reference()
    print(f"host cores: {os.cpu_count()}")
    for j, (n, k) in enumerate(synth.GEMV_SHAPES):
        w, a = synth.gemv_case(j, n, k)
        packed, scale = ref_limited.quantize_w4(w)
        del w
        reps = 3 if n * k < 60e6 else 1
        t = time.perf_counter()
        for _ in range(reps):
            y = ref.gemv_w4(a, packed, scale, k)
        t_ref = (time.perf_counter() - t) / reps
        t = time.perf_counter()
        for _ in range(reps):
            y_c = O.gemv_w4_c(a, packed, scale, k)
        t_c = (time.perf_counter() - t) / reps
        same = np.array_equal(y.view(np.uint32), y_c.view(np.uint32))
        alg = n * k * 5 / 8
        print(f"{n}x{k}: reference.gemv_w4 {t_ref * 1e3:.1f} ms ({alg / t_ref / 1e9:.2f} GB/s); "
              f"C port {t_c * 1e3:.2f} ms ({alg / t_c / 1e9:.1f} GB/s); same bits {same}",
              flush=True)


if __name__ == "__main__":
    main()
