"""The ggml custom-op bridge (row f3): graph nodes built as ggml tensors (the struct that
sqwen's FFI mirrors at src/backend/ffi.rs:22-39), translated by sqmix_ggml_fa_args /
sqmix_ggml_gdn_args into the C-ABI argument structs, and run through the
ggml_custom_op_t callbacks.

CPU: the struct layout, the translation of strides / types / pointers, the rejection of
malformed nodes, and that threads other than 0 do nothing.  GPU: the callbacks on real
device tensors equal the direct entry points (the attention node without a workspace
takes the static scratch of sqmix_fa_decode_noalloc).
"""
import ctypes

import numpy as np
import pytest
import torch

F32, F16, Q4_0, I32, I64, BF16 = 0, 1, 2, 26, 27, 30
ESIZE = {F32: 4, F16: 2, BF16: 2, I32: 4, I64: 8}


def _lib():
    import sqmix

    return sqmix.lib()


def tensor(typ, ne, data=0, nb=None, srcs=()):
    """A ggml tensor: ne (up to 4 dims, padded with 1), nb in bytes (contiguous if None)."""
    from sqmix._lib import GgmlTensor

    t = GgmlTensor()
    t.type = typ
    ne = list(ne) + [1] * (4 - len(ne))
    for d in range(4):
        t.ne[d] = ne[d]
    if nb is None:
        if typ == Q4_0:
            nb = [18, 18 * ne[0] // 32]
        else:
            nb = [ESIZE[typ]]
        while len(nb) < 4:
            nb.append(nb[-1] * ne[len(nb) - 1])
    for d in range(4):
        t.nb[d] = nb[d]
    t.data = data
    t._keep = list(srcs)
    for i, s in enumerate(srcs):
        if s is not None:
            t.src[i] = ctypes.pointer(s)
    return t


def fa_node(T=1, q_type=F32, gate=True, new=1, cap=4096, q_strides=None, base=0x10000):
    q = tensor(q_type, [256, T, 16], base + 0x1000, nb=q_strides)
    k = tensor(Q4_0, [512, cap], base + 0x2000)
    v = tensor(Q4_0, [512, cap], base + 0x3000)
    step = tensor(I64, [2], base + 0x4000)
    g = tensor(F32, [256, 16, T], base + 0x5000) if gate else None
    kn = tensor(F32, [256, 2, new], base + 0x6000) if new else None
    vn = tensor(F32, [256, 2, new], base + 0x7000) if new else None
    return tensor(F32, [256, 16, T], base + 0x8000, srcs=(q, k, v, step, g, kn, vn))


def test_ggml_tensor_mirror_layout():
    from sqmix._lib import GgmlTensor

    assert ctypes.sizeof(GgmlTensor) == 336 == _lib().sqmix_ggml_tensor_bytes()
    assert GgmlTensor.data.offset == 248 and GgmlTensor.src.offset == 152 and GgmlTensor.nb.offset == 48


def test_fa_node_translation():
    from sqmix._lib import FaArgs, GgmlFaOp

    base = 0x10000
    # Q as the permuted view of attn.rs:229-237: [256, T, 16] over a [256, 16, T] buffer
    node = fa_node(T=2, q_type=BF16, q_strides=[2, 2 * 256 * 16, 2 * 256, 2 * 256 * 16 * 2], base=base)
    op = GgmlFaOp(scale=1 / 16, rope_n_rot=64, rope_freq_base=1e7, rope_pos_offset=77, config=3, flags=1,
                  norm_eps=1e-6)
    a = FaArgs()
    assert _lib().sqmix_ggml_fa_args(ctypes.byref(node), ctypes.byref(op), ctypes.byref(a)) == 0
    assert (a.q, a.q_dtype, a.q_stride_tok, a.q_stride_head) == (base + 0x1000, BF16, 4096, 256)
    assert (a.k_cache, a.v_cache, a.capacity) == (base + 0x2000, base + 0x3000, 4096)
    assert (a.n_kv, a.q_pos0) == (base + 0x4000, base + 0x4008)
    assert (a.gate, a.gate_stride_head, a.gate_stride_tok) == (base + 0x5000, 256, 4096)
    assert (a.k_new, a.v_new, a.n_new, a.k_new_stride_tok) == (base + 0x6000, base + 0x7000, 1, 512)
    assert (a.out, a.n_q, a.rope_n_rot, a.rope_pos_offset, a.config, a.flags) == (base + 0x8000, 2, 64, 77, 3, 1)
    assert a.workspace is None and abs(a.scale - 1 / 16) < 1e-9


@pytest.mark.parametrize("bad,msg", [
    (dict(T=3), b"T=3"),
    (dict(cap=1000), b"capacity"),
    (dict(q_type=I32), b"Q must be"),
])
def test_fa_node_rejections(bad, msg):
    from sqmix._lib import FaArgs, GgmlFaOp

    node = fa_node(**bad)
    a = FaArgs()
    op = GgmlFaOp(scale=1 / 16)
    assert _lib().sqmix_ggml_fa_args(ctypes.byref(node), ctypes.byref(op), ctypes.byref(a)) == -1
    assert msg in _lib().sqmix_last_error()


def test_fa_node_missing_sources_and_idle_threads():
    from sqmix._lib import GgmlFaOp

    node = fa_node()
    node.src[3] = ctypes.POINTER(type(node))()  # no step scalars
    op = GgmlFaOp(scale=1 / 16, status=12345)
    _lib().sqmix_ggml_fa_decode_op(ctypes.byref(node), 1, 4, ctypes.byref(op))  # thread 1: nothing
    assert op.status == 12345
    _lib().sqmix_ggml_fa_decode_op(ctypes.byref(node), 0, 4, ctypes.byref(op))  # thread 0: translation fails
    assert op.status == -1 and b"src[0..3]" in _lib().sqmix_last_error()


def gdn_node(T=2, n_seqs=1, n_planes=2, typ=F32, sel=True, base=0x20000):
    q = tensor(typ, [128, 16, T, n_seqs], base + 0x100)
    k = tensor(typ, [128, 16, T, n_seqs], base + 0x200)
    v = tensor(typ, [128, 32, T, n_seqs], base + 0x300)
    g = tensor(F32, [1, 32, T, n_seqs], base + 0x400)
    b = tensor(F32, [1, 32, T, n_seqs], base + 0x500)
    st = tensor(F32, [128 * 128 * 32, n_planes, n_seqs], base + 0x600)
    s = tensor(I32, [n_seqs], base + 0x700) if sel else None
    return tensor(F32, [128, 32, T, n_seqs], base + 0x800, srcs=(q, k, v, g, b, st, s))


def test_gdn_node_translation():
    from sqmix._lib import GdnArgs, GgmlGdnOp

    base = 0x20000
    node = gdn_node(T=2, n_seqs=3, n_planes=3, typ=BF16, base=base)
    op = GgmlGdnOp(n_snap=2, l2_eps=1e-6, flags=1, h_v_offset=0)
    a = GdnArgs()
    assert _lib().sqmix_ggml_gdn_args(ctypes.byref(node), ctypes.byref(op), ctypes.byref(a)) == 0
    assert (a.q, a.k, a.v, a.dtype) == (base + 0x100, base + 0x200, base + 0x300, BF16)
    assert (a.qk_stride_tok, a.qk_stride_seq, a.v_stride_tok, a.v_stride_seq) == (2048, 4096, 4096, 8192)
    assert (a.g, a.beta, a.state, a.sel, a.out) == (base + 0x400, base + 0x500, base + 0x600, base + 0x700,
                                                     base + 0x800)
    assert (a.n_planes, a.n_seqs, a.n_tokens, a.h_k, a.h_v, a.n_snap, a.flags) == (3, 3, 2, 16, 32, 2, 1)


def test_gdn_node_rejects_strided_gates():
    from sqmix._lib import GdnArgs, GgmlGdnOp

    node = gdn_node()
    node.src[3].contents.nb[1] = 8  # g not contiguous
    a = GdnArgs()
    assert _lib().sqmix_ggml_gdn_args(ctypes.byref(node), ctypes.byref(GgmlGdnOp(n_snap=1)), ctypes.byref(a)) == -1
    assert b"g and beta" in _lib().sqmix_last_error()


# ------------------------------------------------------------------ GPU ---

@pytest.mark.gpu
@pytest.mark.parametrize("workspace", [False, True])
def test_fa_callback_equals_decode(workspace):
    import sqmix
    from sqmix._lib import GgmlFaOp

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    g = torch.Generator(device="cuda")
    g.manual_seed(31)
    n_kv, cap = 3000, 3072
    kc, vc = sqmix.new_kv_cache(cap), sqmix.new_kv_cache(cap)
    sqmix.set_rows_q4_0(torch.randn((n_kv - 1, 2, 256), generator=g, device="cuda"),
                        torch.randn((n_kv - 1, 2, 256), generator=g, device="cuda"),
                        torch.arange(n_kv - 1, device="cuda"), kc, vc, cap, rope_n_rot=64, rope_freq_base=1e7)
    q = torch.randn((16, 1, 256), generator=g, device="cuda")  # a [256, 16, T] buffer
    gate = torch.randn((1, 16, 256), generator=g, device="cuda")
    kn = torch.randn((1, 2, 256), generator=g, device="cuda")
    vn = torch.randn((1, 2, 256), generator=g, device="cuda")
    step = torch.tensor([n_kv, n_kv - 1], dtype=torch.int64, device="cuda")
    out = torch.full((1, 16, 256), float("nan"), device="cuda")
    # Q as ggml's permuted view [256, T, 16] of the [256, 16, T] tensor: nb1 = token, nb2 = head
    qt = tensor(F32, [256, 1, 16], q.data_ptr(), nb=[4, 4 * 256 * 16, 4 * 256, 4 * 256 * 16])
    node = tensor(F32, [256, 16, 1], out.data_ptr(), srcs=(
        qt, tensor(Q4_0, [512, cap], kc.data_ptr()), tensor(Q4_0, [512, cap], vc.data_ptr()),
        tensor(I64, [2], step.data_ptr()), tensor(F32, [256, 16, 1], gate.data_ptr()),
        tensor(F32, [256, 2, 1], kn.data_ptr()), tensor(F32, [256, 2, 1], vn.data_ptr())))
    ws = sqmix.new_fa_workspace(1) if workspace else None
    op = GgmlFaOp(scale=1 / 16, rope_n_rot=64, rope_freq_base=1e7, n_splits=64,
                  workspace=ws.data_ptr() if ws is not None else None, workspace_bytes=ws.numel() if ws is not None else 0,
                  stream=torch.cuda.current_stream().cuda_stream, status=99)
    _lib().sqmix_ggml_fa_decode_op(ctypes.byref(node), 0, 1, ctypes.byref(op))
    torch.cuda.synchronize()
    assert op.status == 0, _lib().sqmix_last_error()
    want = sqmix.flash_attn_ext(q.view(1, 16, 256), kc, vc, cap, step[0:1], step[1:2], gate=gate, rope_n_rot=64,
                                rope_freq_base=1e7, n_splits=64, k_new=kn, v_new=vn)
    torch.cuda.synchronize()
    assert torch.allclose(out, want, rtol=1e-6, atol=1e-7)


@pytest.mark.gpu
def test_gdn_callback_equals_decode():
    import sqmix
    from sqmix._lib import GgmlGdnOp

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    g = torch.Generator(device="cuda")
    g.manual_seed(32)
    T, n_planes = 2, 2
    q = torch.randn((1, T, 16, 128), generator=g, device="cuda").to(torch.bfloat16)
    k = torch.randn((1, T, 16, 128), generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn((1, T, 32, 128), generator=g, device="cuda").to(torch.bfloat16)
    gl = -torch.rand((1, T, 32), generator=g, device="cuda")
    b = torch.rand((1, T, 32), generator=g, device="cuda")
    S0 = torch.randn((1, n_planes, 32, 128, 128), generator=g, device="cuda") * 0.02
    sel = torch.tensor([1], dtype=torch.int32, device="cuda")
    S1, S2 = S0.clone(), S0.clone()
    out = torch.empty((1, T, 32, 128), device="cuda")
    node = tensor(F32, [128, 32, T, 1], out.data_ptr(), srcs=(
        tensor(BF16, [128, 16, T, 1], q.data_ptr()), tensor(BF16, [128, 16, T, 1], k.data_ptr()),
        tensor(BF16, [128, 32, T, 1], v.data_ptr()), tensor(F32, [1, 32, T, 1], gl.data_ptr()),
        tensor(F32, [1, 32, T, 1], b.data_ptr()), tensor(F32, [128 * 128 * 32, n_planes, 1], S1.data_ptr()),
        tensor(I32, [1], sel.data_ptr())))
    op = GgmlGdnOp(n_snap=2, l2_eps=1e-6, stream=torch.cuda.current_stream().cuda_stream, status=99)
    _lib().sqmix_ggml_gdn_decode_op(ctypes.byref(node), 0, 1, ctypes.byref(op))
    want = sqmix.gated_delta_net(q, k, v, gl, b, S2, n_planes=n_planes, sel=sel, n_snap=2, l2_eps=1e-6)
    torch.cuda.synchronize()
    assert op.status == 0, _lib().sqmix_last_error()
    assert torch.equal(out, want)
    assert torch.equal(S1, S2)
