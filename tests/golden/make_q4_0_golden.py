"""Generate the q4_0 golden vectors in ``q4_0_golden.npz``.

The bytes come from gguf-py 0.19.0 (``gguf/quants.py``, class ``Q4_0``), a numpy
restatement of ggml's ``quantize_row_q4_0`` that is installed in this image.  The
reference (sqwen) calls the same ggml routine through ``ggml_quantize_chunk``
(``src/backend/ffi.rs:435-443``, used at ``tests/attn_test.rs:210-229``) and through
``ggml_set_rows`` into its q4_0 KV cache (``src/engine/kv.rs:367-396``).

The cases cover what the reference's q4_0 test cares about
(``tests/attn_test.rs:781-833``) plus the edge cases of the rounding rule: all-zero
blocks (d = 0), ties on |x| between a positive and a negative element (first index
wins), values whose scaled form lands exactly on a .5 boundary, single spikes,
fp16 overflow/underflow of d, and N(0,1) rows of the production K/V width (512).

Run from the repo root:  python tests/golden/make_q4_0_golden.py
"""
import os

import numpy as np
from gguf.quants import Q4_0, quantize, dequantize
from gguf.constants import GGMLQuantizationType

HERE = os.path.dirname(os.path.abspath(__file__))


def cases() -> np.ndarray:
    rng = np.random.default_rng(20261201)
    blocks = []
    # 1. production-like rows: 64 tokens x 512 (2 KV heads x 256), N(0,1)
    blocks.append(rng.standard_normal((64 * 16, 32)).astype(np.float32))
    # 2. the reference test's LCG (tests/attn_test.rs:67-75) in [-1, 1)
    s = np.uint32((7 * 2654435761 + 1) & 0xFFFFFFFF)
    vals = []
    for _ in range(8 * 32):
        s = np.uint32((int(s) * 1664525 + 1013904223) & 0xFFFFFFFF)
        vals.append(float(int(s) >> 8) / 8388608.0 - 1.0)
    blocks.append(np.array(vals, dtype=np.float32).reshape(8, 32))
    # 3. all zeros (d == 0 -> id == 0 -> every nibble 8)
    blocks.append(np.zeros((2, 32), dtype=np.float32))
    # 4. ties on |x|: +a first / -a first
    b = rng.standard_normal((4, 32)).astype(np.float32) * 0.1
    b[0, 3], b[0, 20] = 1.5, -1.5
    b[1, 3], b[1, 20] = -1.5, 1.5
    b[2, 0], b[2, 31] = 2.0, -2.0
    b[3, 5], b[3, 6] = -0.75, -0.75
    blocks.append(b)
    # 5. scaled values exactly on .5 boundaries: max = -8 so d = 1, id = 1
    b = np.zeros((2, 32), dtype=np.float32)
    b[0, 0] = -8.0
    b[0, 1:] = np.array([(-7.5 + 0.5 * i) for i in range(31)], dtype=np.float32)
    b[1, 0] = 8.0  # d = -1
    b[1, 1:] = np.array([(7.5 - 0.5 * i) for i in range(31)], dtype=np.float32)
    blocks.append(b)
    # 6. single spike, tiny noise
    b = (rng.standard_normal((2, 32)) * 1e-3).astype(np.float32)
    b[0, 17] = 3.0
    b[1, 9] = -3.0
    blocks.append(b)
    # 7. d overflows fp16 (|max| > 8 * 65504) and d underflows to fp16 subnormal/zero
    b = rng.standard_normal((3, 32)).astype(np.float32)
    b[0] *= 1e6
    b[1] *= 1e-6
    b[2] *= 1e-9
    blocks.append(b)
    # 8. wide dynamic range and constant blocks
    b = np.empty((3, 32), dtype=np.float32)
    b[0] = np.logspace(-4, 2, 32).astype(np.float32) * np.where(np.arange(32) % 2, 1, -1)
    b[1] = 0.3
    b[2] = -0.3
    blocks.append(b)
    # 9. uniform random scale per block (bf16-representable inputs, like config 1/2 activations)
    b = rng.standard_normal((256, 32)).astype(np.float32) * rng.uniform(0.01, 10, (256, 1)).astype(np.float32)
    bits = b.view(np.uint32) & np.uint32(0xFFFF0000)
    blocks.append(bits.view(np.float32))
    return np.concatenate(blocks, axis=0)


def main():
    x = cases()
    q = quantize(x, GGMLQuantizationType.Q4_0)
    assert q.shape == (x.shape[0], 18), q.shape
    deq = dequantize(q, GGMLQuantizationType.Q4_0)
    np.savez_compressed(os.path.join(HERE, "q4_0_golden.npz"), x=x, q=q.astype(np.uint8),
                        deq=deq.astype(np.float32))
    print(f"wrote {x.shape[0]} blocks; Q4_0 block size {Q4_0.block_size}")


if __name__ == "__main__":
    main()
