"""Engine-side state objects (C++ in host.cpp), mirrored for Python callers.

KvCache  <- src/engine/kv.rs:67-448   (begin_step / rewind_to / reset / n_kv_padded /
                                        append / zero_caches / bytes_per_token)
GdnState <- src/model/gdn.rs:71-120 and src/model/graph.rs:190-350
            (set_recurrent_sel, snapshot_gdn / restore_gdn)

Errors come back as SqmixError with the codes of include/sqmix.h; an overflowing
begin_step or an out-of-range rewind raises instead of returning Err(String).
"""
from __future__ import annotations

import ctypes

import torch

from . import ops
from ._lib import check, lib


class _DevView:
    """Expose a raw device allocation to torch via __cuda_array_interface__."""

    def __init__(self, ptr: int, nbytes: int, typestr: str = "|u1", itemsize: int = 1):
        self.__cuda_array_interface__ = {
            "shape": (nbytes // itemsize,),
            "typestr": typestr,
            "data": (ptr, False),
            "version": 3,
            "strides": None,
        }


def _device_tensor(ptr: int, nbytes: int, dtype=torch.uint8, device=None) -> torch.Tensor:
    typestr, itemsize = {torch.uint8: ("|u1", 1), torch.float32: ("<f4", 4), torch.int64: ("<i8", 8),
                         torch.int32: ("<i4", 4)}[dtype]
    with torch.cuda.device(device):
        return torch.as_tensor(_DevView(ptr, nbytes, typestr, itemsize), device="cuda")


class KvCache:
    """Single-sequence, append-only q4_0 KV cache for the full-attention layers."""

    def __init__(self, n_layers: int, kv_cap: int, device: int | None = None):
        if device is None:
            device = torch.cuda.current_device()
        self.device = int(device)
        h = ctypes.c_void_p()
        check(lib().sqmix_kvcache_create(int(n_layers), int(kv_cap), self.device, ctypes.byref(h)),
              "KvCache")
        self._h = h
        self.n_layers = int(n_layers)
        cap = self.capacity_alloc
        nbytes = ops.kv_cache_bytes(cap)
        self._k = [_device_tensor(lib().sqmix_kvcache_k(h, i), nbytes, device=self.device)
                   for i in range(n_layers)]
        self._v = [_device_tensor(lib().sqmix_kvcache_v(h, i), nbytes, device=self.device)
                   for i in range(n_layers)]
        max_step = int(lib().sqmix_kvcache_max_step_tokens(h))
        self._step = _device_tensor(lib().sqmix_kvcache_device_step(h), 8 * (2 + max_step),
                                    torch.int64, self.device)

    def close(self):
        if getattr(self, "_h", None):
            lib().sqmix_kvcache_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- bookkeeping (kv.rs) -------------------------------------------------
    def begin_step(self, n_tokens: int) -> None:
        check(lib().sqmix_kvcache_begin_step(self._h, int(n_tokens)), "KvCache.begin_step")

    def rewind_to(self, pos: int) -> None:
        check(lib().sqmix_kvcache_rewind_to(self._h, int(pos)), "KvCache.rewind_to")

    def reset(self) -> None:
        lib().sqmix_kvcache_reset(self._h)

    def zero_caches(self, stream=None) -> None:
        check(lib().sqmix_kvcache_zero(self._h, ops._stream(stream)), "KvCache.zero_caches")

    @property
    def n_used(self) -> int:
        return int(lib().sqmix_kvcache_n_used(self._h))

    @property
    def step_start(self) -> int:
        return int(lib().sqmix_kvcache_step_start(self._h))

    def n_kv_padded(self) -> int:
        return int(lib().sqmix_kvcache_n_kv_padded(self._h))

    @property
    def kv_cap(self) -> int:
        return int(lib().sqmix_kvcache_capacity(self._h))

    @property
    def capacity_alloc(self) -> int:
        return int(lib().sqmix_kvcache_capacity_alloc(self._h))

    def bytes_per_token(self) -> int:
        return int(lib().sqmix_kvcache_bytes_per_token(self._h))

    def k_state(self, slot: int) -> torch.Tensor:
        return self._k[slot]

    def v_state(self, slot: int) -> torch.Tensor:
        return self._v[slot]

    # ---- device step inputs (graph.rs fill_inputs) -----------------------------
    def upload_step(self, stream=None) -> None:
        check(lib().sqmix_kvcache_upload_step(self._h, ops._stream(stream)), "KvCache.upload_step")

    @property
    def d_n_kv(self) -> torch.Tensor:
        return self._step[0:1]

    @property
    def d_q_pos0(self) -> torch.Tensor:
        return self._step[1:2]

    def d_rows(self, n_tokens: int) -> torch.Tensor:
        return self._step[2:2 + n_tokens]

    # ---- layer ops --------------------------------------------------------------
    def append(self, slot: int, k_cur: torch.Tensor, v_cur: torch.Tensor, rope_n_rot: int = 0,
               rope_freq_base: float = 1e7, rope_pos_offset: int = 0, stream=None) -> None:
        """Write this step's K/V rows (after upload_step) into layer `slot`."""
        T = k_cur.shape[0]
        ops.set_rows_q4_0(k_cur, v_cur, self.d_rows(T), self._k[slot], self._v[slot], self.capacity_alloc,
                          rope_n_rot=rope_n_rot, rope_freq_base=rope_freq_base,
                          rope_pos_offset=rope_pos_offset, stream=stream)

    def attention(self, slot: int, q: torch.Tensor, gate: torch.Tensor | None = None,
                  scale: float = 1.0 / 16.0, rope_n_rot: int = 0, rope_freq_base: float = 1e7,
                  rope_pos_offset: int = 0, out=None, lse=None, workspace=None, n_splits: int = 0,
                  k_new=None, v_new=None, overlap_prev: bool = False, stream=None) -> torch.Tensor:
        """Causal attention of this step's queries over layer `slot`.

        Either append first (KvCache.append), or pass the step's k_new/v_new to append
        them inside the same launch.  overlap_prev (SQMIX_FA_OVERLAP_PREV) is safe when
        the step's scalars were uploaded (upload_step) and the kernel just before this
        call wrote no cache rows below the step start.
        """
        return ops.flash_attn_ext(q, self._k[slot], self._v[slot], self.capacity_alloc, self.d_n_kv,
                                  self.d_q_pos0, gate=gate, scale=scale, rope_n_rot=rope_n_rot,
                                  rope_freq_base=rope_freq_base, rope_pos_offset=rope_pos_offset, out=out,
                                  lse=lse, workspace=workspace, n_splits=n_splits, k_new=k_new, v_new=v_new,
                                  overlap_prev=overlap_prev, stream=stream)

    def export_rows(self, slot: int, which: str, row0: int, n_rows: int) -> torch.Tensor:
        cache = self._k[slot] if which == "k" else self._v[slot]
        return ops.kv_convert_rows(cache, self.capacity_alloc, which, row0, n_rows)


class GdnState:
    """Recurrent GDN state with 1 + n_rs snapshot planes per layer, and (conv_channels >
    0) the short-conv history planes [1 + n_rs][conv_channels][d_conv - 1] that
    sqmix_gdn_conv reads and writes; snapshots hold plane 0 of both per layer."""

    def __init__(self, n_layers: int, h_v: int = 32, n_rs: int = 0, device: int | None = None,
                 conv_channels: int = 0, d_conv: int = 4):
        if device is None:
            device = torch.cuda.current_device()
        self.device = int(device)
        h = ctypes.c_void_p()
        check(lib().sqmix_gdnstate_create_conv(int(n_layers), int(h_v), int(n_rs), int(conv_channels), int(d_conv),
                                               self.device, ctypes.byref(h)), "GdnState")
        self.conv_channels = int(conv_channels)
        self.d_conv = int(d_conv) if conv_channels > 0 else 0
        self._h = h
        self.n_layers = int(n_layers)
        self.h_v = int(h_v)
        self.n_rs = int(n_rs)
        self.n_planes = int(lib().sqmix_gdnstate_n_planes(h))
        plane = self.h_v * ops.GDN_D * ops.GDN_D
        self._planes = [
            _device_tensor(lib().sqmix_gdnstate_planes(h, i), 4 * plane * self.n_planes, torch.float32,
                           self.device).view(self.n_planes, self.h_v, ops.GDN_D, ops.GDN_D)
            for i in range(n_layers)]
        self._sel = _device_tensor(lib().sqmix_gdnstate_device_sel(h), 4, torch.int32, self.device)
        conv_plane = self.conv_channels * (self.d_conv - 1) if self.conv_channels else 0
        self._conv = [
            _device_tensor(lib().sqmix_gdnstate_conv_planes(h, i), 4 * conv_plane * self.n_planes, torch.float32,
                           self.device).view(self.n_planes, self.conv_channels, self.d_conv - 1)
            for i in range(n_layers)] if conv_plane else []

    def close(self):
        if getattr(self, "_h", None):
            lib().sqmix_gdnstate_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def planes(self, layer: int) -> torch.Tensor:
        return self._planes[layer]

    def conv_planes(self, layer: int) -> torch.Tensor:
        """[1 + n_rs][conv_channels][d_conv - 1] f32 (the `state` argument of gdn_conv)."""
        if not self._conv:
            raise ValueError("this GdnState has no conv history (conv_channels = 0)")
        return self._conv[layer]

    def zero_states(self, stream=None) -> None:
        check(lib().sqmix_gdnstate_zero(self._h, ops._stream(stream)), "GdnState.zero_states")

    def set_recurrent_sel(self, sel: int) -> int:
        return int(lib().sqmix_gdnstate_set_sel(self._h, int(sel)))

    def recurrent_sel(self) -> int:
        return int(lib().sqmix_gdnstate_sel(self._h))

    def upload_sel(self, stream=None) -> None:
        check(lib().sqmix_gdnstate_upload_sel(self._h, ops._stream(stream)), "GdnState.upload_sel")

    @property
    def d_sel(self) -> torch.Tensor:
        return self._sel

    def step(self, layer: int, q, k, v, g, beta, n_tokens: int | None = None, l2_eps: float = 0.0,
             out=None, stream=None) -> torch.Tensor:
        """One gated_delta_net call on `layer`: reads plane sel, writes n_snap planes."""
        T = q.shape[-3] if n_tokens is None else n_tokens
        n_snap = min(T, self.n_rs + 1)
        return ops.gated_delta_net(q, k, v, g, beta, self._planes[layer], n_planes=self.n_planes,
                                   sel=self._sel, n_snap=n_snap, l2_eps=l2_eps, out=out, stream=stream)

    def snapshot_bytes(self) -> int:
        return int(lib().sqmix_gdnstate_snapshot_bytes(self._h))

    def snapshot_gdn(self, stream=None) -> bytes:
        n = self.snapshot_bytes()
        buf = ctypes.create_string_buffer(n)
        check(lib().sqmix_gdnstate_snapshot(self._h, buf, n, ops._stream(stream)), "snapshot_gdn")
        return buf.raw

    def restore_gdn(self, data: bytes, stream=None) -> None:
        buf = ctypes.create_string_buffer(bytes(data), len(data))
        check(lib().sqmix_gdnstate_restore(self._h, buf, len(data), ops._stream(stream)), "restore_gdn")
