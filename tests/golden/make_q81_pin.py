"""Generates tests/golden/q81_pin.npz: outputs of an independent build of the
published q8_1 matmul kernels, to pin the oracle's restatement of them.

The reference's GPU matmuls are candle-kernels 0.11.0's q8_1 kernels
(quantize_q8_1, MMVQ mul_mat_vec_q, MMQ mul_mat_q), vendored from llama.cpp's
ggml-cuda. vLLM ships its own port of the same llama.cpp kernels
(torch.ops._C.ggml_mul_mat_vec_a8 = one warp per row MMVQ,
torch.ops._C.ggml_mul_mat_a8 = MMQ). This script runs them on random GGUF
blocks written by this project's converter and on activations that include the
quantizer's edge cases (an all-zero block, exact .5 ratios, a single non-zero,
negative maxima), and stores the weights, the outputs and a checksum of the
activations (which tests regenerate with activations()). It needs a CUDA GPU and vLLM;
the fixture it writes is read on the CPU by tests/test_oracle_pins.py.

    python tests/golden/make_q81_pin.py [out.npz]
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", ".."))

from malaga_b200.convert import quantize, seeded_normal  # noqa: E402

CASES = [  # (ggml type, rows N, row length K)
    (8, 32, 1024),    # Q8_0
    (8, 32, 4096),
    (12, 32, 1024),   # Q4_K
    (12, 32, 4096),
    (14, 32, 1024),   # Q6_K
    (14, 32, 4096),
]
ROWS = [1, 4, 8, 16, 64]


def activations(rows: int, K: int, seed: int) -> np.ndarray:
    x = seeded_normal(rows * K, seed, 11, 1.0).reshape(rows, K).astype(np.float32)
    x[0, :32] = 0.0                                   # amax == 0 block
    x[0, 32:64] = np.float32(0.5) * np.arange(-16, 16, dtype=np.float32)   # x/d hits .5 exactly
    x[0, 64] = np.float32(127.0)                      # d == 1 for that block
    x[0, 65:96] = np.float32(2.5) * np.sign(np.arange(31) - 15.5).astype(np.float32)
    x[0, 96:128] = 0.0
    x[0, 100] = np.float32(-3.0)                      # a single negative value
    if rows > 1:
        x[1, :] *= np.float32(1e-3)
    return x


def main(out: str) -> None:
    import vllm._custom_ops as ops  # noqa: F401  (registers torch.ops._C)

    dev = torch.device("cuda:0")
    rec: dict[str, np.ndarray] = {}
    for ci, (t, N, K) in enumerate(CASES):
        w = seeded_normal(N * K, 100 + ci, 3, 0.02).reshape(N, K).astype(np.float32)
        wq = quantize(w, t).reshape(N, -1)
        rec[f"w{ci}"] = wq
        W = torch.from_numpy(wq).to(dev)
        for rows in ROWS:
            x = activations(rows, K, 1000 * ci + rows)
            X = torch.from_numpy(x).to(dev)
            rec[f"xsum{ci}_{rows}"] = np.array([x.astype(np.float64).sum(), np.abs(x).astype(np.float64).sum()])
            if rows <= 8:
                y = torch.ops._C.ggml_mul_mat_vec_a8(W, X, t, N)
                rec[f"vec{ci}_{rows}"] = y.float().cpu().numpy()
            y = torch.ops._C.ggml_mul_mat_a8(W, X, t, N)
            rec[f"mmq{ci}_{rows}"] = y.float().cpu().numpy()
    rec["cases"] = np.array(CASES, np.int64)
    rec["rows"] = np.array(ROWS, np.int64)
    np.savez_compressed(out, **rec)
    print("wrote", out, sum(v.nbytes for v in rec.values()), "bytes")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.join(os.path.dirname(os.path.abspath(__file__)),
                                                             "q81_pin.npz"))
