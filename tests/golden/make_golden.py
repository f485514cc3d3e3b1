"""Generates tests/golden/spinn_ref_vectors.npz from the reference operators.

Run in the development container, where the reference sources are mounted and
oracle/_ref/libspinn_ref.so was built from them (`make -C oracle ref`):

    python tests/golden/make_golden.py

Every output below comes from the reference's own code (op_conv2d, op_gemm, op_matmul,
winograd_pack_weight + winograd_conv_3x3) linked unmodified, with the O-fix epilogue shim
(oracle/ref_shim.c).  Inputs:

* kat1: SPINN/run_time/test_winograd.c:62-75 -- C=2, 4x4, OC=3, pad 1, X[i]=i+1,
  W[i]=(i%5-2)*0.5, bias {1,2,3}; the reference test passes if Winograd and im2col agree
  within 0.1.
* kat2: SPINN/run_time/test_winograd2.c -- one channel, X = 1..16 (4x4), diagonal 3x3
  kernel, pad 1, bias 0 (Winograd must equal the direct convolution).
* conv_res / conv_s2 / gemm / gemm_alpha / matmul: small seeded cases (default_rng(5)).
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import oracle  # noqa: E402
from spinn_b200 import runtime  # noqa: E402  (parameter-block packers only)


def main():
    R = oracle.RefOracle(fix=True)
    out = {}
    # kat1
    x = (np.arange(32, dtype=np.float32) + 1).reshape(1, 2, 4, 4)
    w = ((np.arange(54) % 5 - 2) * 0.5).astype(np.float32).reshape(3, 2, 3, 3)
    b = np.array([1, 2, 3], np.float32)
    p = runtime.conv_params((3, 3), (1, 1), (1, 1, 1, 1), (1, 1), 1, 0, 0)
    out.update(kat1_x=x, kat1_w=w, kat1_b=b, kat1_conv=R.conv2d(x, w, b, None, p, (1, 3, 4, 4)),
               kat1_wino=R.winograd_f23(x, w, b, 1, 1, 4, 4, 0))
    # kat2
    x = np.arange(1, 17, dtype=np.float32).reshape(1, 1, 4, 4)
    w = np.eye(3, dtype=np.float32).reshape(1, 1, 3, 3)
    b = np.zeros(1, np.float32)
    out.update(kat2_x=x, kat2_w=w, kat2_conv=R.conv2d(x, w, b, None, p, (1, 1, 4, 4)),
               kat2_wino=R.winograd_f23(x, w, b, 1, 1, 4, 4, 0))
    rng = np.random.default_rng(5)
    # conv with residual + ReLU (fused_act 5)
    x = rng.uniform(-1, 1, (2, 8, 10, 10)).astype(np.float32)
    w = rng.normal(0, 0.2, (12, 8, 3, 3)).astype(np.float32)
    b = rng.normal(0, 0.1, 12).astype(np.float32)
    r = rng.uniform(-1, 1, (2, 12, 10, 10)).astype(np.float32)
    p5 = runtime.conv_params((3, 3), (1, 1), (1, 1, 1, 1), (1, 1), 1, 0, 5)
    out.update(conv_res_x=x, conv_res_w=w, conv_res_b=b, conv_res_r=r,
               conv_res_y=R.conv2d(x, w, b, r, p5, (2, 12, 10, 10)))
    # strided conv + ReLU
    x = rng.uniform(-1, 1, (1, 4, 9, 9)).astype(np.float32)
    w = rng.normal(0, 0.3, (8, 4, 3, 3)).astype(np.float32)
    b = rng.normal(0, 0.1, 8).astype(np.float32)
    p1 = runtime.conv_params((3, 3), (2, 2), (1, 1, 1, 1), (1, 1), 1, 0, 1)
    out.update(conv_s2_x=x, conv_s2_w=w, conv_s2_b=b, conv_s2_y=R.conv2d(x, w, b, None, p1, (1, 8, 5, 5)))
    # gemm (transB, vector C) and the alpha != 1 case
    a = rng.uniform(-1, 1, (5, 9)).astype(np.float32)
    bm = rng.uniform(-1, 1, (7, 9)).astype(np.float32)
    c = rng.uniform(-1, 1, 7).astype(np.float32)
    out.update(gemm_a=a, gemm_b=bm, gemm_c=c,
               gemm_y=R.gemm(a, bm, c, runtime.gemm_params(1.0, 1.0, 0, 1), (5, 7)),
               gemm_alpha_y=R.gemm(a, bm, c, runtime.gemm_params(0.5, 2.0, 0, 1), (5, 7)))
    # batched matmul with equal batch counts
    a = rng.uniform(-1, 1, (3, 4, 6)).astype(np.float32)
    bm = rng.uniform(-1, 1, (3, 6, 5)).astype(np.float32)
    out.update(matmul_a=a, matmul_b=bm, matmul_y=R.matmul(a, bm, (3, 4, 5)))
    path = os.path.join(HERE, "spinn_ref_vectors.npz")
    np.savez(path, **out)
    print(f"wrote {path}: {len(out)} arrays, {os.path.getsize(path)} bytes")


if __name__ == "__main__":
    main()
