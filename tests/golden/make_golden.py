"""Regenerates the committed golden fixtures of tests/golden/ from the reference's own compiled host
code (oracle/_ref/libref_cpu.so, built by `make -C oracle` from the reference tree):

  ref_q6k_dot_cases.npz   the six hand-built blocks of tests/test_q6k_dot.cu:242-332, their fp16 x
                          and the reference's fp64 expectation (cpu_q6k_dot)
  ref_gemv_64x256.npz     tests/test_gemv_q6k.cu:167-219 inputs (srand(123)) and cpu_gemv_q6k output
  ref_gemv_128x512.npz    tests/test_gemv_q6k.cu:222-269 inputs (srand(456)) and cpu_gemv_q6k output

Run from the repository root:  python tests/golden/make_golden.py
"""
import ctypes
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "tests"))
import oracle as orc  # noqa: E402
from test_oracle_pins import regen_reference_case  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def main():
    ref = orc.ref_cpu()
    if ref is None:
        raise SystemExit("oracle/_ref/libref_cpu.so missing: run `make -C oracle` with the reference tree present")
    cases = {}
    exp = np.zeros(6, np.float64)
    for i in range(6):
        b = np.zeros(210, np.uint8)
        x = np.zeros(256, np.uint16)
        e = ctypes.c_double()
        assert ref.ref_dot_case(i, _p(b), _p(x), ctypes.byref(e)) == 0
        cases[f"blk{i}"], cases[f"x{i}"], exp[i] = b, x, e.value
    np.savez(os.path.join(OUT, "ref_q6k_dot_cases.npz"), expected=exp, **cases)
    for name, seed, M, K, d, mod, lo, span in [("ref_gemv_64x256", 123, 64, 256, 0.05, 21, -1.0, 2.0),
                                               ("ref_gemv_128x512", 456, 128, 512, 0.03, 31, -0.5, 1.0)]:
        W, x = regen_reference_case(orc, seed, M, K, d, mod, lo, span)
        y = np.zeros(M, np.float64)
        ref.ref_cpu_gemv_q6k(_p(W), _p(x), _p(y), M, K)
        np.savez(os.path.join(OUT, name + ".npz"), W=W, x=x, y=y, M=M, K=K)
        print(name, "rms(y) =", float(np.sqrt(np.mean(y ** 2))))


if __name__ == "__main__":
    main()
