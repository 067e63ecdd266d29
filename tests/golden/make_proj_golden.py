"""Generate the projection golden vectors in ``proj_golden.npz``.

sqwen's mixer projections are ``ggml_mul_mat`` on GGUF weights (``src/model/attn.rs:127-129,
285``; ``src/model/gdn.rs:264-276, 577``); a Q4_K_M model stores them as q4_K, q6_K and
q8_0 blocks.  The dequantised weights come from gguf-py 0.19.0 (``gguf/quants.py``,
classes ``Q8_0``, ``Q4_K``, ``Q6_K``), the numpy restatement of ggml's block formats that
is installed in this image; the expected products are float64 sums of those weights
times x.

Cases per type: random raw blocks (every bit pattern of the scales, mins and quants is a
valid block) with finite f16 super-block scales of mixed magnitude, plus q8_0 blocks
quantised from N(0,1) rows by gguf-py's bit-exact quantiser.  3 tokens; n_in = 512
(two K super-blocks per row) for q4_K and q8_0, 2048 for q6_K (its 210-byte super-blocks
make 16-byte aligned rows from 2048 values on); n_out = 24, 8 for q6_K.

Run from the repo root:  python tests/golden/make_proj_golden.py
"""
import os

import numpy as np
from gguf.constants import GGMLQuantizationType as QT
from gguf.quants import dequantize, quantize

HERE = os.path.dirname(os.path.abspath(__file__))
N_TOK = 3
SHAPES = {"q4_k": (512, 24), "q8_0": (512, 24), "q6_k": (2048, 8)}  # (n_in, n_out)


def f16_bytes(rng, n, scale):
    return (rng.standard_normal(n) * scale).astype(np.float16).view(np.uint8).reshape(n, 2)


def q4_k_rows(rng, N_IN, N_OUT):
    nb = N_OUT * N_IN // 256
    d = f16_bytes(rng, nb, 1e-3)
    dmin = f16_bytes(rng, nb, 1e-3)
    rest = rng.integers(0, 256, size=(nb, 140), dtype=np.uint8)  # 12 scale bytes + 128 nibble bytes
    return np.concatenate([d, dmin, rest], axis=1).reshape(N_OUT, -1)


def q6_k_rows(rng, N_IN, N_OUT):
    nb = N_OUT * N_IN // 256
    body = rng.integers(0, 256, size=(nb, 208), dtype=np.uint8)  # ql 128, qh 64, int8 scales 16
    d = f16_bytes(rng, nb, 1e-3)
    return np.concatenate([body, d], axis=1).reshape(N_OUT, -1)


def q8_0_rows(rng, N_IN, N_OUT):
    w = rng.standard_normal((N_OUT, N_IN)).astype(np.float32) * 0.05
    w[0, :32] = 0.0  # an all-zero block (d = 0)
    return quantize(w, QT.Q8_0).reshape(N_OUT, -1)


def main():
    rng = np.random.default_rng(20261202)
    out = {}
    for name, qt, gen in (("q4_k", QT.Q4_K, q4_k_rows), ("q6_k", QT.Q6_K, q6_k_rows), ("q8_0", QT.Q8_0, q8_0_rows)):
        N_IN, N_OUT = SHAPES[name]
        x = rng.standard_normal((N_TOK, N_IN)).astype(np.float32)
        out[f"{name}_x"] = x
        rows = np.ascontiguousarray(gen(rng, N_IN, N_OUT))
        w = dequantize(rows, qt).reshape(N_OUT, N_IN).astype(np.float32)
        assert np.isfinite(w).all(), name
        out[f"{name}_w"] = rows
        out[f"{name}_deq"] = w
        out[f"{name}_y"] = (x.astype(np.float64) @ w.astype(np.float64).T).astype(np.float64)
    np.savez_compressed(os.path.join(HERE, "proj_golden.npz"), **out)
    print("wrote", os.path.join(HERE, "proj_golden.npz"), {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
