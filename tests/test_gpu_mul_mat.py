"""GPU parity of the mixer projections (sqmix_mul_mat, ggml_mul_mat of attn.rs:127-129,
285 and gdn.rs:264-276, 577) against the golden vectors (gguf-py's dequantizers) and the
CPU oracle at the model's shapes (n_embd 2048, QG 8192, KV 512, d_inner 4096, conv 8192,
32 value heads).

Bar: max |gpu - ref| <= 1e-5 * max |ref| (f32 sums of dequantised weights against
float64 sums of the same weights).
"""
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 1e-5
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "proj_golden.npz")


def rel_err(got, want):
    return np.abs(np.asarray(got, np.float64) - want).max() / max(np.abs(want).max(), 1e-30)


def random_rows(rng, wtype, n_in, n_out):
    """Valid raw rows: random quant / scale bytes, finite f16 super-block scales."""
    nb = n_out * n_in // 256

    def f16(n, s):
        return (rng.standard_normal(n) * s).astype(np.float16).view(np.uint8).reshape(n, 2)

    if wtype == 12:
        rows = np.concatenate([f16(nb, 1e-3), f16(nb, 1e-3), rng.integers(0, 256, (nb, 140), dtype=np.uint8)], 1)
    elif wtype == 14:
        rows = np.concatenate([rng.integers(0, 256, (nb, 208), dtype=np.uint8), f16(nb, 1e-3)], 1)
    elif wtype == 8:
        nb32 = n_out * n_in // 32
        rows = np.concatenate([f16(nb32, 1e-3), rng.integers(0, 256, (nb32, 32), dtype=np.uint8)], 1)
    else:
        w = rng.standard_normal((n_out, n_in)).astype(np.float32) * 0.05
        if wtype == 0:
            return w.view(np.uint8).reshape(n_out, -1)
        if wtype == 1:
            return w.astype(np.float16).view(np.uint8).reshape(n_out, -1)
        return (w.view(np.uint32) >> 16).astype(np.uint16).view(np.uint8).reshape(n_out, -1)
    return np.ascontiguousarray(rows).reshape(n_out, -1)


@pytest.mark.parametrize("name,wtype", [("q4_k", 12), ("q6_k", 14), ("q8_0", 8)])
def test_mul_mat_golden(name, wtype):
    import sqmix

    d = np.load(GOLDEN)
    x = d[f"{name}_x"]
    w = torch.from_numpy(d[f"{name}_w"]).cuda()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    y = sqmix.mul_mat(w, wtype, x.shape[1], torch.from_numpy(x).cuda(), status=status)
    torch.cuda.synchronize()
    assert rel_err(y.cpu().numpy(), d[f"{name}_y"]) <= TOL
    assert int(status.item()) == 0


# (weight type, n_in, n_out, tokens, x dtype): the model's projections (Q4_K_M assigns
# q4_K to most, q6_K to attn_v; ssm_alpha / ssm_beta have 32 rows), ragged row counts,
# several passes of 4 tokens, half-precision activations
CASES = [
    (12, 2048, 8192, 1, torch.float32),   # QG / qkv
    (14, 2048, 512, 2, torch.float32),    # attn_v, MTP verification
    (12, 4096, 2048, 1, torch.float32),   # W_o / ssm_out
    (8, 4096, 2048, 3, torch.float32),
    (0, 2048, 32, 1, torch.float32),      # ssm_alpha as f32
    (30, 2048, 37, 5, torch.bfloat16),    # ragged tile, two passes
    (1, 1024, 100, 4, torch.float16),
    (12, 256, 9, 9, torch.float32),       # one super-block per row, three passes
]


@pytest.mark.parametrize("wtype,n_in,n_out,T,xdt", CASES)
def test_mul_mat_model_shapes_vs_oracle(oracle, wtype, n_in, n_out, T, xdt):
    import sqmix

    rng = np.random.default_rng(1000 + n_out + wtype)
    rows = random_rows(rng, wtype, n_in, n_out)
    x = torch.randn((T, n_in), generator=torch.Generator().manual_seed(n_in + T)).to(xdt)
    want = oracle.mul_mat(rows, wtype, n_in, x.float().numpy())
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    y = sqmix.mul_mat(torch.from_numpy(rows).cuda(), wtype, n_in, x.cuda(), status=status)
    torch.cuda.synchronize()
    assert rel_err(y.cpu().numpy(), want.astype(np.float64)) <= TOL
    assert int(status.item()) == 0


@pytest.mark.parametrize("x_pad", [64, 3])
def test_mul_mat_strided_tokens_and_output(x_pad):
    """x and y with token strides larger than their rows (views into wider buffers); a
    pad of 3 floats leaves the rows of x 4-byte aligned only."""
    import sqmix
    from sqmix._lib import MulMatArgs, check, lib
    import ctypes

    rng = np.random.default_rng(7)
    n_in, n_out, T = 2048, 64, 3
    rows = random_rows(rng, 12, n_in, n_out)
    xw = torch.randn((T, n_in + x_pad), device="cuda")
    yw = torch.full((T, n_out + 16), 7.0, device="cuda")
    w = torch.from_numpy(rows).cuda()
    a = MulMatArgs(w=w.data_ptr(), w_type=12, w_row_bytes=sqmix.mul_mat_row_bytes(12, n_in), n_in=n_in, n_out=n_out,
                   x=xw.data_ptr(), x_dtype=0, x_stride=n_in + x_pad, n_tokens=T, y=yw.data_ptr(), y_stride=n_out + 16)
    check(lib().sqmix_mul_mat(ctypes.byref(a), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)), "mul_mat")
    torch.cuda.synchronize()
    import oracle as orc

    want = orc.mul_mat(rows, 12, n_in, xw[:, :n_in].cpu().numpy())
    got = yw.cpu().numpy()
    assert rel_err(got[:, :n_out], want.astype(np.float64)) <= TOL
    assert (got[:, n_out:] == 7.0).all()  # nothing written past the rows


@pytest.mark.parametrize("T", [1, 2, 6])
def test_mul_mat_group_matches_single_calls_and_oracle(oracle, T):
    """One sqmix_mul_mat_group over projections of the same x -- a ragged q4_K (tiles
    that end inside the tile list), q6_K, q8_0 and two float-typed matrices (the
    32-row beta / alpha) -- equals one sqmix_mul_mat per entry bit for bit, and the
    oracle within the bar; T = 6 takes two passes."""
    import sqmix

    rng = np.random.default_rng(4242 + T)
    n_in = 2048
    specs = [(12, 1000), (14, 512), (8, 40), (0, 32), (30, 32), (12, 16)]
    rows = [random_rows(rng, wt, n_in, n_out) for wt, n_out in specs]
    ws = [torch.from_numpy(r).cuda() for r in rows]
    x = torch.randn((T, n_in), generator=torch.Generator().manual_seed(T)).cuda()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    got = sqmix.mul_mat_group([(w, wt) for w, (wt, _) in zip(ws, specs)], n_in, x, status=status)
    single = [sqmix.mul_mat(w, wt, n_in, x) for w, (wt, _) in zip(ws, specs)]
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    xh = x.cpu().numpy()
    for (wt, n_out), r, g, s in zip(specs, rows, got, single):
        assert g.shape == (T, n_out)
        assert torch.equal(g, s), (wt, n_out)
        assert rel_err(g.cpu().numpy(), oracle.mul_mat(r, wt, n_in, xh).astype(np.float64)) <= TOL, (wt, n_out)


def test_mul_mat_group_bf16_x_4096_inputs(oracle):
    """A group at n_in = 4096 (two units per warp) with bf16 activations and 3 tokens."""
    import sqmix

    rng = np.random.default_rng(99)
    n_in, T = 4096, 3
    specs = [(12, 2048), (8, 64)]
    rows = [random_rows(rng, wt, n_in, n_out) for wt, n_out in specs]
    x = torch.randn((T, n_in), generator=torch.Generator().manual_seed(5)).to(torch.bfloat16)
    got = sqmix.mul_mat_group([(torch.from_numpy(r).cuda(), wt) for r, (wt, _) in zip(rows, specs)], n_in, x.cuda())
    torch.cuda.synchronize()
    for (wt, n_out), r, g in zip(specs, rows, got):
        want = oracle.mul_mat(r, wt, n_in, x.float().numpy())
        assert rel_err(g.cpu().numpy(), want.astype(np.float64)) <= TOL, (wt, n_out)


# The prefill form (n_tokens >= 128; >= 48 with at least 48 output tiles of 128 x 128,
# >= 16 with at least 96): a tcgen05 GEMM on tf32 operands for f32 x (f16 / bf16 for
# 16-bit x), f32 accumulation.  Bar: max |gpu - ref| <= 3e-3 * max |ref| against the
# float64 sums of the exact dequantised weights.
PREFILL_TOL = 3e-3
PREFILL_CASES = [
    (12, 2048, 300, 130, torch.float32),   # ragged weight tile, ragged second token tile
    (12, 2048, 6144, 48, torch.float32),   # 48 tokens with 48 tiles
    (12, 2048, 12288, 16, torch.float32),  # 16 tokens with 96 tiles
    (14, 2048, 128, 128, torch.bfloat16),  # attn_v's format
    (8, 4096, 200, 256, torch.float32),
    (0, 2048, 32, 137, torch.float32),     # the 32-row f32 beta / alpha
    (30, 2048, 40, 300, torch.float16),
    (1, 1024, 128, 129, torch.float32),
    (12, 4096, 512, 512, torch.float32),   # W_o / ssm_out at a pp512 batch
]


@pytest.mark.parametrize("wtype,n_in,n_out,T,xdt", PREFILL_CASES)
def test_mul_mat_prefill_gemm_vs_oracle(oracle, wtype, n_in, n_out, T, xdt):
    import sqmix

    rng = np.random.default_rng(2000 + n_out + wtype + T)
    rows = random_rows(rng, wtype, n_in, n_out)
    x = torch.randn((T, n_in), generator=torch.Generator().manual_seed(T + n_in)).to(xdt)
    want = oracle.mul_mat(rows, wtype, n_in, x.float().numpy())
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    y = sqmix.mul_mat(torch.from_numpy(rows).cuda(), wtype, n_in, x.cuda(), status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert rel_err(y.cpu().numpy(), want.astype(np.float64)) <= PREFILL_TOL


@pytest.mark.parametrize("x_pad", [8, 3])
def test_mul_mat_prefill_group_and_strides(oracle, x_pad):
    """A prefill group (q4_K, q6_K, f32 rows) of one strided x into strided outputs; a pad
    of 3 floats leaves the rows of x 4-byte aligned only (no tensor-map staging)."""
    import ctypes

    from sqmix._lib import MulMatArgs, check, lib

    rng = np.random.default_rng(31)
    n_in, T = 2048, 130
    specs = [(12, 1000), (14, 512), (0, 32)]
    rows = [random_rows(rng, wt, n_in, n_out) for wt, n_out in specs]
    ws = [torch.from_numpy(r).cuda() for r in rows]
    xw = torch.randn((T, n_in + x_pad), generator=torch.Generator().manual_seed(3)).cuda()
    ys = [torch.full((T, n_out + 5), 7.0, device="cuda") for _, n_out in specs]
    import sqmix

    arr = (MulMatArgs * len(specs))()
    for i, ((wt, n_out), w, y) in enumerate(zip(specs, ws, ys)):
        arr[i] = MulMatArgs(w=w.data_ptr(), w_type=wt, w_row_bytes=sqmix.mul_mat_row_bytes(wt, n_in), n_in=n_in,
                            n_out=n_out, x=xw.data_ptr(), x_dtype=0, x_stride=n_in + x_pad, n_tokens=T, y=y.data_ptr(),
                            y_stride=n_out + 5)
    check(lib().sqmix_mul_mat_group(arr, len(specs), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)),
          "mul_mat_group")
    torch.cuda.synchronize()
    xh = xw[:, :n_in].cpu().numpy()
    for (wt, n_out), r, y in zip(specs, rows, ys):
        got = y.cpu().numpy()
        assert rel_err(got[:, :n_out], oracle.mul_mat(r, wt, n_in, xh).astype(np.float64)) <= PREFILL_TOL, wt
        assert (got[:, n_out:] == 7.0).all()
