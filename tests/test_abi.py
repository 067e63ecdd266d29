"""C-ABI checks that need no GPU: exports, argument validation, host bookkeeping."""
import ctypes
import os
import re
import struct

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "sqmix.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(sqmix_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol(sqmix_lib):
    L = sqmix_lib.lib()
    names = declared_functions()
    assert len(names) >= 30
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, f"not exported: {missing}"


def test_python_mirror_binds_every_declared_symbol(sqmix_lib):
    assert sorted(sqmix_lib.exported_symbols()) == declared_functions()


def test_version(sqmix_lib):
    assert b"sm_100a" in sqmix_lib.lib().sqmix_version()


def test_argument_validation_without_gpu(sqmix_lib):
    from sqmix._lib import FaArgs, KvAppendArgs

    L = sqmix_lib.lib()
    a = FaArgs(n_q=3)
    assert L.sqmix_fa_decode(ctypes.byref(a), None) == sqmix_lib.SQMIX_EINVAL
    assert b"null" in L.sqmix_last_error() or b"n_q" in L.sqmix_last_error()
    # all pointers set (fake), bad n_q
    fake = ctypes.c_void_p(256)
    a = FaArgs(q=fake, k_cache=fake, v_cache=fake, n_kv=fake, q_pos0=fake, out=fake, workspace=fake,
               n_q=3, capacity=256, scale=0.0625)
    assert L.sqmix_fa_decode(ctypes.byref(a), None) == sqmix_lib.SQMIX_EINVAL
    assert b"n_q=3" in L.sqmix_last_error()
    # workspace too small -> ENOSPC (checked before any launch)
    a = FaArgs(q=fake, k_cache=fake, v_cache=fake, n_kv=fake, q_pos0=fake, out=fake, workspace=fake,
               n_q=1, capacity=256, scale=0.0625, workspace_bytes=16, n_splits=4)
    assert L.sqmix_fa_decode(ctypes.byref(a), None) == sqmix_lib.SQMIX_ENOSPC
    b = KvAppendArgs(k=fake, v=fake, rows=fake, k_cache=fake, v_cache=fake, dtype=0, n_tokens=1,
                     k_stride_tok=512, v_stride_tok=512, capacity=100)
    assert L.sqmix_kv_append_q4_0(ctypes.byref(b), None) == sqmix_lib.SQMIX_EINVAL
    assert b"capacity" in L.sqmix_last_error()
    assert L.sqmix_kv_convert_rows(fake, fake, 256, 200, 100, 0, 1, None) == sqmix_lib.SQMIX_EINVAL


def test_front_end_argument_validation_without_gpu(sqmix_lib):
    from sqmix._lib import GdnConvArgs, HeadNormArgs

    L = sqmix_lib.lib()
    fake = ctypes.c_void_p(256)
    ok = dict(x=fake, x_dtype=0, x_stride_tok=8192, x_stride_seq=8192, weight=fake, conv_state=fake, n_planes=2,
              n_snap=1, n_seqs=1, n_tokens=1, channels=8192, kernel=4, head_dim=128, n_qk_channels=4096,
              l2_eps=1e-6, out=fake)
    for bad, what in ((dict(kernel=9), b"kernel=9"), (dict(head_dim=100), b"head_dim=100"),
                      (dict(channels=8000), b"channels=8000"), (dict(n_snap=3), b"n_snap=3"),
                      (dict(n_qk_channels=100), b"n_qk_channels=100"), (dict(out=None), b"null"),
                      (dict(x_stride_tok=100), b"x strides")):
        a = GdnConvArgs(**{**ok, **bad})
        assert L.sqmix_gdn_conv(ctypes.byref(a), None) == sqmix_lib.SQMIX_EINVAL, bad
        assert what in L.sqmix_last_error(), (bad, L.sqmix_last_error())
    h = HeadNormArgs(x=fake, x_dtype=7, out=fake, n_tokens=1, n_heads=1, head_dim=128)
    assert L.sqmix_head_norm(ctypes.byref(h), None) == sqmix_lib.SQMIX_EINVAL
    assert b"dtype 7" in L.sqmix_last_error()
    h = HeadNormArgs(x=fake, x_dtype=0, out=fake, n_tokens=1, n_heads=1, head_dim=128, eps=-1.0)
    assert L.sqmix_head_norm(ctypes.byref(h), None) == sqmix_lib.SQMIX_EINVAL


def test_gdn_decode_argument_validation_without_gpu(sqmix_lib):
    from sqmix._lib import GdnArgs

    L = sqmix_lib.lib()
    fake = 1 << 20  # never dereferenced: validation fails before any launch
    ok = dict(q=fake, k=fake, v=fake, dtype=sqmix_lib.SQMIX_F32, qk_stride_tok=16 * 128, v_stride_tok=32 * 128,
              qk_stride_seq=16 * 128, v_stride_seq=32 * 128, g=fake, beta=fake, state=fake, n_planes=1, sel=None,
              n_seqs=1, n_tokens=1, h_k=16, h_v=32, n_snap=1, l2_eps=0.0, out=fake, flags=0)
    for bad in (dict(flags=2), dict(flags=-1), dict(n_snap=2), dict(h_v=0), dict(h_v_offset=-1)):
        a = GdnArgs(**{**ok, **bad})
        assert L.sqmix_gdn_decode(ctypes.byref(a), None) == sqmix_lib.SQMIX_EINVAL, bad


def test_workspace_sizes(sqmix_lib):
    assert sqmix_lib.fa_workspace_bytes(1, 148) >= 148 * 16 * 256 * 4
    assert sqmix_lib.fa_workspace_bytes(2, 148) >= 2 * 148 * 16 * 256 * 4
    assert sqmix_lib.kv_cache_bytes(172032) == 172032 * 288


# ------------------------------------------------- KvCache bookkeeping (kv.rs) --

def _kv(L, n_layers, cap):
    h = ctypes.c_void_p()
    assert L.sqmix_kvcache_create(n_layers, cap, -1, ctypes.byref(h)) == 0
    return h


def test_kvcache_cursor_semantics(sqmix_lib):
    L = sqmix_lib.lib()
    h = _kv(L, 10, 1000)
    try:
        assert L.sqmix_kvcache_capacity(h) == 1000
        assert L.sqmix_kvcache_capacity_alloc(h) == 1024  # kv.rs:119 ceil to 256
        assert L.sqmix_kvcache_bytes_per_token(h) == 10 * 576  # 5.6 KiB/token over 10 layers
        assert L.sqmix_kvcache_n_kv_padded(h) == 0
        assert L.sqmix_kvcache_begin_step(h, 300) == 0
        assert (L.sqmix_kvcache_step_start(h), L.sqmix_kvcache_n_used(h)) == (0, 300)
        assert L.sqmix_kvcache_n_kv_padded(h) == 512
        assert L.sqmix_kvcache_begin_step(h, 2) == 0
        assert (L.sqmix_kvcache_step_start(h), L.sqmix_kvcache_n_used(h)) == (300, 302)
        # overflow is an error and leaves the cursor alone (kv.rs:240-245)
        assert L.sqmix_kvcache_begin_step(h, 699) == sqmix_lib.SQMIX_EOVERFLOW
        assert b"overflow" in L.sqmix_last_error()
        assert L.sqmix_kvcache_n_used(h) == 302
        assert L.sqmix_kvcache_begin_step(h, 698) == 0
        # rewind moves the cursor only, never forward (kv.rs:284-297)
        assert L.sqmix_kvcache_rewind_to(h, 1001) == sqmix_lib.SQMIX_ERANGE
        assert L.sqmix_kvcache_rewind_to(h, 301) == 0
        assert (L.sqmix_kvcache_step_start(h), L.sqmix_kvcache_n_used(h)) == (301, 301)
        assert L.sqmix_kvcache_rewind_to(h, 302) == sqmix_lib.SQMIX_ERANGE
        L.sqmix_kvcache_reset(h)
        assert L.sqmix_kvcache_n_used(h) == 0
        assert L.sqmix_kvcache_upload_step(h, None) == 0  # bookkeeping-only: no device copy
    finally:
        L.sqmix_kvcache_destroy(h)


def test_gdnstate_selector_and_snapshot_header(sqmix_lib):
    L = sqmix_lib.lib()
    h = ctypes.c_void_p()
    assert L.sqmix_gdnstate_create(30, 32, 1, -1, ctypes.byref(h)) == 0
    try:
        assert L.sqmix_gdnstate_n_planes(h) == 2
        # set_recurrent_sel clamps to n_rs (graph.rs:190-196) and is one-shot
        assert L.sqmix_gdnstate_set_sel(h, 5) == 1
        assert L.sqmix_gdnstate_sel(h) == 1
        assert L.sqmix_gdnstate_upload_sel(h, None) == 0
        assert L.sqmix_gdnstate_sel(h) == 0
        plane = 32 * 128 * 128 * 4
        n = L.sqmix_gdnstate_snapshot_bytes(h)
        assert n == 8 + 30 * plane  # no conv history: state planes only
        good = struct.pack("<Q", n - 8) + bytes(n - 8)
        assert L.sqmix_gdnstate_restore(h, good, len(good), None) == 0
        bad_len = struct.pack("<Q", n - 8) + bytes(n - 9)
        assert L.sqmix_gdnstate_restore(h, bad_len, len(bad_len), None) == sqmix_lib.SQMIX_EINVAL
        assert b"length mismatch" in L.sqmix_last_error()
        bad_hdr = struct.pack("<Q", n) + bytes(n - 8)
        assert L.sqmix_gdnstate_restore(h, bad_hdr, len(bad_hdr), None) == sqmix_lib.SQMIX_EINVAL
        assert L.sqmix_gdnstate_restore(h, b"1234", 4, None) == sqmix_lib.SQMIX_EINVAL
    finally:
        L.sqmix_gdnstate_destroy(h)


def test_gdnstate_checkpoint_size_with_conv_history(sqmix_lib):
    # the reference's checkpoint of the 30 GDN layers (graph.rs:301-350): per layer the
    # 2 MiB state plane + the 8192 x 3 conv plane, about 63 MiB, behind a u64 header
    L = sqmix_lib.lib()
    h = ctypes.c_void_p()
    assert L.sqmix_gdnstate_create_conv(30, 32, 1, 8192, 4, -1, ctypes.byref(h)) == 0
    try:
        n = L.sqmix_gdnstate_snapshot_bytes(h)
        assert n == 8 + 30 * (32 * 128 * 128 + 8192 * 3) * 4
        assert 62 * 2**20 < n < 64 * 2**20
        good = struct.pack("<Q", n - 8) + bytes(n - 8)
        assert L.sqmix_gdnstate_restore(h, good, len(good), None) == 0
        no_conv = 8 + 30 * 32 * 128 * 128 * 4
        short = struct.pack("<Q", no_conv - 8) + bytes(no_conv - 8)
        assert L.sqmix_gdnstate_restore(h, short, len(short), None) == sqmix_lib.SQMIX_EINVAL
    finally:
        L.sqmix_gdnstate_destroy(h)
    for bad in ((30, 32, 1, -1, 4), (30, 32, 1, 8192, 1)):
        assert L.sqmix_gdnstate_create_conv(*bad, -1, ctypes.byref(h)) == sqmix_lib.SQMIX_EINVAL


def test_kvcache_rejects_bad_shapes(sqmix_lib):
    L = sqmix_lib.lib()
    h = ctypes.c_void_p()
    assert L.sqmix_kvcache_create(0, 100, -1, ctypes.byref(h)) == sqmix_lib.SQMIX_EINVAL
    assert L.sqmix_kvcache_create(1, 0, -1, ctypes.byref(h)) == sqmix_lib.SQMIX_EINVAL


def header_struct_fields():
    """Field names of every `typedef struct X {...} X;` in sqmix.h, in order."""
    text = open(HEADER).read()
    out = {}
    for m in re.finditer(r"typedef struct (\w+) \{(.*?)\} \w+;", text, re.S):
        body = re.sub(r"/\*.*?\*/", "", m.group(2), flags=re.S)
        out[m.group(1)] = [re.findall(r"(\w+)\s*$", d.strip())[0] for d in body.split(";") if d.strip()]
    return out


def _abi_structs():
    from sqmix import _lib as L

    return {
        "sqmix_kv_append_args": (L.SQMIX_ABI_KV_APPEND_ARGS, L.KvAppendArgs),
        "sqmix_fa_args": (L.SQMIX_ABI_FA_ARGS, L.FaArgs),
        "sqmix_fa_batch_args": (L.SQMIX_ABI_FA_BATCH_ARGS, L.FaBatchArgs),
        "sqmix_peer_merge_args": (L.SQMIX_ABI_PEER_MERGE_ARGS, L.PeerMergeArgs),
        "sqmix_gdn_args": (L.SQMIX_ABI_GDN_ARGS, L.GdnArgs),
        "sqmix_gdn_conv_args": (L.SQMIX_ABI_GDN_CONV_ARGS, L.GdnConvArgs),
        "sqmix_head_norm_args": (L.SQMIX_ABI_HEAD_NORM_ARGS, L.HeadNormArgs),
        "sqmix_gdn_layer_args": (L.SQMIX_ABI_GDN_LAYER_ARGS, L.GdnLayerArgs),
        "sqmix_ggml_fa_op": (L.SQMIX_ABI_GGML_FA_OP, L.GgmlFaOp),
        "sqmix_ggml_gdn_op": (L.SQMIX_ABI_GGML_GDN_OP, L.GgmlGdnOp),
        "sqmix_mul_mat_args": (L.SQMIX_ABI_MUL_MAT_ARGS, L.MulMatArgs),
    }


def test_abi_layout_table_matches_ctypes_mirror(sqmix_lib):
    """Every argument struct: the library's compiled size, field count and offsets equal
    the ctypes declaration's, and the ctypes field names follow the header's order.  A
    field added to one side only fails here."""
    L = sqmix_lib.lib()
    hdr = header_struct_fields()
    structs = _abi_structs()
    assert set(structs) == set(hdr), "every struct of sqmix.h needs an ABI table entry and a ctypes mirror"
    for name, (which, cls) in structs.items():
        names = [f[0] for f in cls._fields_]
        assert names == hdr[name], name
        assert L.sqmix_abi_struct_size(which) == ctypes.sizeof(cls), name
        assert L.sqmix_abi_field_count(which) == len(cls._fields_), name
        for i, (fname, _) in enumerate(cls._fields_):
            assert L.sqmix_abi_field_offset(which, i) == getattr(cls, fname).offset, (name, fname)
        assert L.sqmix_abi_field_offset(which, len(cls._fields_)) == -1
    assert L.sqmix_abi_struct_size(0) == 0 and L.sqmix_abi_field_count(99) == -1


def test_integration_guide_rust_structs_match_header():
    """The Rust #[repr(C)] structs in INTEGRATION.md declare the same fields, in the same
    order, as sqmix.h (a binding copied from the guide must not be shorter than the C
    struct the library reads)."""
    guide = open(os.path.join(REPO, "INTEGRATION.md")).read()
    hdr = header_struct_fields()
    rust = {}
    for m in re.finditer(r"pub struct (\w+) \{\n(.*?)\n\}", guide, re.S):
        rust[m.group(1)] = re.findall(r"pub (\w+):", m.group(2))
    for cname, fields in hdr.items():
        rname = "".join(w.capitalize() for w in cname.split("_"))
        assert rname in rust, f"INTEGRATION.md declares no {rname}"
        assert rust[rname] == fields, rname
    for name in declared_functions():
        assert f"pub fn {name}(" in guide, f"INTEGRATION.md's extern block lacks {name}"


def test_mul_mat_argument_validation_without_gpu(sqmix_lib):
    from sqmix._lib import MulMatArgs

    L = sqmix_lib.lib()
    assert L.sqmix_mul_mat_row_bytes(sqmix_lib.SQMIX_Q4_K, 2048) == 8 * 144
    assert L.sqmix_mul_mat_row_bytes(sqmix_lib.SQMIX_Q6_K, 4096) == 16 * 210
    assert L.sqmix_mul_mat_row_bytes(sqmix_lib.SQMIX_Q8_0, 2048) == 8 * 272
    assert L.sqmix_mul_mat_row_bytes(2, 2048) == 0  # q4_0 weights: not a projection format here
    assert L.sqmix_mul_mat_row_bytes(sqmix_lib.SQMIX_F32, 100) == 0
    fake = ctypes.c_void_p(4096)

    def args(**kw):
        base = dict(w=fake, w_type=sqmix_lib.SQMIX_Q4_K, w_row_bytes=8 * 144, n_in=2048, n_out=64, x=fake,
                    x_dtype=sqmix_lib.SQMIX_F32, x_stride=2048, n_tokens=1, y=fake, y_stride=64)
        base.update(kw)
        return MulMatArgs(**base)

    bad = [
        dict(w_type=2, w_row_bytes=0),                             # unsupported block format
        dict(n_in=8192, w_row_bytes=32 * 144, x_stride=8192),      # n_in above 4096
        dict(n_in=300),                                            # not a multiple of 256
        dict(w_row_bytes=8 * 144 + 16),                            # rows not contiguous
        dict(w_type=sqmix_lib.SQMIX_Q6_K, n_in=512, w_row_bytes=2 * 210, x_stride=512),  # 420-byte rows
        dict(w=ctypes.c_void_p(4096 + 8)),                         # w not 16-byte aligned
        dict(n_tokens=0),
        dict(x_stride=100),
        dict(x_dtype=2),
        dict(y=None),
    ]
    for kw in bad:
        a = args(**kw)
        assert L.sqmix_mul_mat(ctypes.byref(a), None) == sqmix_lib.SQMIX_EINVAL, kw


def test_mul_mat_group_argument_validation_without_gpu(sqmix_lib):
    """A group takes 1..SQMIX_MUL_MAT_MAX_GROUP entries that share x (pointer, dtype,
    stride, tokens, n_in); each entry is checked as sqmix_mul_mat checks it."""
    from sqmix._lib import MulMatArgs

    L = sqmix_lib.lib()
    fake = ctypes.c_void_p(4096)

    def entry(**kw):
        base = dict(w=fake, w_type=sqmix_lib.SQMIX_Q4_K, w_row_bytes=8 * 144, n_in=2048, n_out=64, x=fake,
                    x_dtype=sqmix_lib.SQMIX_F32, x_stride=2048, n_tokens=1, y=fake, y_stride=64)
        base.update(kw)
        return MulMatArgs(**base)

    def group(*entries, n=None):
        arr = (MulMatArgs * max(1, len(entries)))(*entries)
        return L.sqmix_mul_mat_group(arr, len(entries) if n is None else n, None)

    assert sqmix_lib.SQMIX_MUL_MAT_MAX_GROUP == 8
    assert group(entry(), n=0) == sqmix_lib.SQMIX_EINVAL
    assert group(*[entry() for _ in range(9)]) == sqmix_lib.SQMIX_EINVAL
    assert group(entry(), entry(x=ctypes.c_void_p(8192))) == sqmix_lib.SQMIX_EINVAL      # another x
    assert group(entry(), entry(x_stride=4096)) == sqmix_lib.SQMIX_EINVAL               # another stride
    assert group(entry(), entry(n_tokens=2)) == sqmix_lib.SQMIX_EINVAL
    assert group(entry(), entry(x_dtype=sqmix_lib.SQMIX_BF16)) == sqmix_lib.SQMIX_EINVAL
    assert group(entry(), entry(w_row_bytes=8 * 144 + 16)) == sqmix_lib.SQMIX_EINVAL    # a bad second entry
    assert b"mul_mat[1]" in L.sqmix_last_error()
    assert L.sqmix_mul_mat_group(None, 1, None) == sqmix_lib.SQMIX_EINVAL
