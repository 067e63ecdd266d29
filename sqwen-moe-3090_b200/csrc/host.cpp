// host.cpp -- C-ABI host side: error reporting, device queries and the engine-side
// state objects that sit above the kernels.
//
//   sqmix_kvcache   <- KvCache (src/engine/kv.rs:67-448): per-layer q4_0 K/V
//                      caches, a cursor shared by all layers, 256-padding, rewind.
//   sqmix_gdnstate  <- GdnState (src/model/gdn.rs:71-120) and the EngineState
//                      pieces that drive it (src/model/graph.rs:190-350): 1 + n_rs
//                      snapshot planes per layer, the one-shot plane selector, and
//                      the length-prefixed plane-0 checkpoint.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "sqmix.h"

namespace sqmix {

static thread_local std::string g_last_error;

void set_error(const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
}

int cuda_status(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return SQMIX_OK;
    set_error("%s: %s", what, cudaGetErrorString(e));
    return SQMIX_ECUDA;
}

}  // namespace sqmix

using sqmix::cuda_status;
using sqmix::set_error;

extern "C" const char *sqmix_version(void) { return "sqmix 0.1.0 (sm_100a)"; }

extern "C" const char *sqmix_last_error(void) { return sqmix::g_last_error.c_str(); }

extern "C" int sqmix_device_sm_count(int device) {
    if (device < 0 && cudaGetDevice(&device) != cudaSuccess) return 148;
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0)
        return 148;
    return n;
}

namespace {

// Restores the caller's current device on scope exit.
struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (dev >= 0) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

}  // namespace

// ============================================================== KvCache ====

struct sqmix_kvcache {
    int device = 0;
    int32_t n_layers = 0;
    int64_t kv_cap = 0;        // logical capacity
    int64_t kv_cap_alloc = 0;  // padded to SQMIX_KV_PAD
    int64_t n_used = 0;
    int64_t step_start = 0;
    int32_t step_n = 0;
    std::vector<void *> k, v;
    int64_t *d_step = nullptr;  // {n_kv, q_pos0, rows[max_step]}
    int32_t max_step = 0;
    std::vector<int64_t> h_step;
};

extern "C" int sqmix_kvcache_create(int32_t n_layers, int64_t kv_cap, int32_t device,
                                    sqmix_kvcache **out) {
    if (!out || n_layers <= 0 || kv_cap <= 0) {
        set_error("kvcache_create: n_layers=%d kv_cap=%lld", n_layers, (long long)kv_cap);
        return SQMIX_EINVAL;
    }
    *out = nullptr;
    auto *kv = new sqmix_kvcache();
    kv->device = device;
    kv->n_layers = n_layers;
    kv->kv_cap = kv_cap;
    kv->kv_cap_alloc = (kv_cap + SQMIX_KV_PAD - 1) / SQMIX_KV_PAD * SQMIX_KV_PAD;
    kv->max_step = 4096;
    kv->h_step.assign(2 + kv->max_step, 0);
    if (device < 0) {  // bookkeeping only (no device buffers): planning and CPU tests
        *out = kv;
        return SQMIX_OK;
    }
    DeviceGuard guard(device);
    const size_t bytes = sqmix_kv_cache_bytes(kv->kv_cap_alloc);
    int rc = SQMIX_OK;
    for (int32_t l = 0; l < n_layers && rc == SQMIX_OK; ++l) {
        void *pk = nullptr, *pv = nullptr;
        rc = cuda_status(cudaMalloc(&pk, bytes), "kvcache_create: cudaMalloc K");
        if (rc == SQMIX_OK) rc = cuda_status(cudaMalloc(&pv, bytes), "kvcache_create: cudaMalloc V");
        if (pk) kv->k.push_back(pk);
        if (pv) kv->v.push_back(pv);
        // Rows in [n_used, n_kv_padded) are read by attention: they must be zero,
        // not uninitialised memory (kv.rs:150-170).
        if (rc == SQMIX_OK) rc = cuda_status(cudaMemset(pk, 0, bytes), "kvcache_create: memset K");
        if (rc == SQMIX_OK) rc = cuda_status(cudaMemset(pv, 0, bytes), "kvcache_create: memset V");
    }
    if (rc == SQMIX_OK)
        rc = cuda_status(cudaMalloc(&kv->d_step, sizeof(int64_t) * (2 + kv->max_step)),
                         "kvcache_create: cudaMalloc step");
    if (rc != SQMIX_OK) {
        sqmix_kvcache_destroy(kv);
        return rc;
    }
    *out = kv;
    return SQMIX_OK;
}

extern "C" void sqmix_kvcache_destroy(sqmix_kvcache *kv) {
    if (!kv) return;
    if (kv->device < 0) {
        delete kv;
        return;
    }
    DeviceGuard guard(kv->device);
    for (void *p : kv->k) cudaFree(p);
    for (void *p : kv->v) cudaFree(p);
    if (kv->d_step) cudaFree(kv->d_step);
    delete kv;
}

extern "C" int sqmix_kvcache_zero(sqmix_kvcache *kv, sqmix_stream_t stream) {
    if (!kv) return SQMIX_EINVAL;
    if (kv->device < 0) return SQMIX_OK;
    DeviceGuard guard(kv->device);
    const size_t bytes = sqmix_kv_cache_bytes(kv->kv_cap_alloc);
    for (int32_t l = 0; l < kv->n_layers; ++l) {
        int rc = cuda_status(cudaMemsetAsync(kv->k[l], 0, bytes, reinterpret_cast<cudaStream_t>(stream)),
                             "kvcache_zero");
        if (rc == SQMIX_OK)
            rc = cuda_status(cudaMemsetAsync(kv->v[l], 0, bytes, reinterpret_cast<cudaStream_t>(stream)),
                             "kvcache_zero");
        if (rc != SQMIX_OK) return rc;
    }
    return SQMIX_OK;
}

extern "C" int sqmix_kvcache_begin_step(sqmix_kvcache *kv, int32_t n_tokens) {
    if (!kv || n_tokens < 0) {
        set_error("kvcache_begin_step: bad arguments");
        return SQMIX_EINVAL;
    }
    if (kv->n_used + n_tokens > kv->kv_cap) {
        set_error("KV cache overflow: n_used=%lld + n_tokens=%d > kv_cap=%lld", (long long)kv->n_used,
                  n_tokens, (long long)kv->kv_cap);
        return SQMIX_EOVERFLOW;
    }
    if (n_tokens > kv->max_step) {
        set_error("kvcache_begin_step: n_tokens=%d > max step %d", n_tokens, kv->max_step);
        return SQMIX_EINVAL;
    }
    kv->step_start = kv->n_used;
    kv->n_used += n_tokens;
    kv->step_n = n_tokens;
    return SQMIX_OK;
}

extern "C" int sqmix_kvcache_rewind_to(sqmix_kvcache *kv, int64_t pos) {
    if (!kv) return SQMIX_EINVAL;
    if (pos < 0 || pos > kv->n_used) {
        set_error("KV rewind out of range: pos=%lld > written %lld", (long long)pos, (long long)kv->n_used);
        return SQMIX_ERANGE;
    }
    if (pos > kv->kv_cap) {
        set_error("KV rewind out of range: pos=%lld > capacity %lld", (long long)pos, (long long)kv->kv_cap);
        return SQMIX_ERANGE;
    }
    // Cursor only: rows [0, pos) keep their data, [pos, ...) are overwritten later.
    kv->n_used = pos;
    kv->step_start = pos;
    kv->step_n = 0;
    return SQMIX_OK;
}

extern "C" void sqmix_kvcache_reset(sqmix_kvcache *kv) {
    if (!kv) return;
    kv->n_used = 0;
    kv->step_start = 0;
    kv->step_n = 0;
}

extern "C" int64_t sqmix_kvcache_n_used(const sqmix_kvcache *kv) { return kv ? kv->n_used : -1; }
extern "C" int64_t sqmix_kvcache_step_start(const sqmix_kvcache *kv) { return kv ? kv->step_start : -1; }
extern "C" int64_t sqmix_kvcache_n_kv_padded(const sqmix_kvcache *kv) {
    return kv ? (kv->n_used + SQMIX_KV_PAD - 1) / SQMIX_KV_PAD * SQMIX_KV_PAD : -1;
}
extern "C" int64_t sqmix_kvcache_capacity(const sqmix_kvcache *kv) { return kv ? kv->kv_cap : -1; }
extern "C" int64_t sqmix_kvcache_capacity_alloc(const sqmix_kvcache *kv) {
    return kv ? kv->kv_cap_alloc : -1;
}
extern "C" size_t sqmix_kvcache_bytes_per_token(const sqmix_kvcache *kv) {
    // K and V are both q4_0: 512/32 blocks * 18 bytes each, per layer (kv.rs:179-189).
    return kv ? static_cast<size_t>(2 * 288) * kv->n_layers : 0;
}
extern "C" void *sqmix_kvcache_k(sqmix_kvcache *kv, int32_t layer) {
    return (kv && layer >= 0 && layer < kv->n_layers) ? kv->k[layer] : nullptr;
}
extern "C" void *sqmix_kvcache_v(sqmix_kvcache *kv, int32_t layer) {
    return (kv && layer >= 0 && layer < kv->n_layers) ? kv->v[layer] : nullptr;
}
extern "C" const int64_t *sqmix_kvcache_device_step(const sqmix_kvcache *kv) {
    return kv ? kv->d_step : nullptr;
}
extern "C" int32_t sqmix_kvcache_max_step_tokens(const sqmix_kvcache *kv) { return kv ? kv->max_step : 0; }

extern "C" int sqmix_kvcache_upload_step(sqmix_kvcache *kv, sqmix_stream_t stream) {
    if (!kv) return SQMIX_EINVAL;
    kv->h_step[0] = kv->n_used;      // keys visible after this step's append
    kv->h_step[1] = kv->step_start;  // absolute position of the step's first query
    for (int32_t t = 0; t < kv->step_n; ++t) kv->h_step[2 + t] = kv->step_start + t;
    if (kv->device < 0) return SQMIX_OK;
    DeviceGuard guard(kv->device);
    // Pageable source: the call returns once the bytes are staged, so h_step may be
    // reused immediately (this upload is not part of any captured graph).
    return cuda_status(cudaMemcpyAsync(kv->d_step, kv->h_step.data(), sizeof(int64_t) * (2 + kv->step_n),
                                       cudaMemcpyHostToDevice, reinterpret_cast<cudaStream_t>(stream)),
                       "kvcache_upload_step");
}

// ============================================================= GdnState ====

struct sqmix_gdnstate {
    int device = 0;
    int32_t n_layers = 0;
    int32_t h_v = 0;
    int32_t n_rs = 0;
    int32_t sel = 0;
    int32_t conv_channels = 0;  // 0: no conv history
    int32_t d_conv = 0;
    std::vector<float *> planes;
    std::vector<float *> conv_planes;
    int32_t *d_sel = nullptr;
    size_t plane_elems() const { return static_cast<size_t>(h_v) * SQMIX_GDN_D * SQMIX_GDN_D; }
    size_t conv_plane_elems() const {
        return conv_channels > 0 ? static_cast<size_t>(conv_channels) * (d_conv - 1) : 0;
    }
};

extern "C" int sqmix_gdnstate_create_conv(int32_t n_layers, int32_t h_v, int32_t n_rs, int32_t conv_channels,
                                          int32_t d_conv, int32_t device, sqmix_gdnstate **out) {
    if (!out || n_layers <= 0 || h_v <= 0 || n_rs < 0 || conv_channels < 0 ||
        (conv_channels > 0 && d_conv < 2)) {
        set_error("gdnstate_create: n_layers=%d h_v=%d n_rs=%d conv_channels=%d d_conv=%d", n_layers, h_v, n_rs,
                  conv_channels, d_conv);
        return SQMIX_EINVAL;
    }
    *out = nullptr;
    auto *st = new sqmix_gdnstate();
    st->device = device;
    st->n_layers = n_layers;
    st->h_v = h_v;
    st->n_rs = n_rs;
    st->conv_channels = conv_channels;
    st->d_conv = conv_channels > 0 ? d_conv : 0;
    if (device < 0) {  // bookkeeping only
        *out = st;
        return SQMIX_OK;
    }
    DeviceGuard guard(device);
    const size_t bytes = st->plane_elems() * sizeof(float) * (1 + n_rs);
    const size_t conv_bytes = st->conv_plane_elems() * sizeof(float) * (1 + n_rs);
    int rc = SQMIX_OK;
    for (int32_t l = 0; l < n_layers && rc == SQMIX_OK; ++l) {
        float *p = nullptr;
        rc = cuda_status(cudaMalloc(&p, bytes), "gdnstate_create: cudaMalloc");
        if (p) st->planes.push_back(p);
        if (rc == SQMIX_OK) rc = cuda_status(cudaMemset(p, 0, bytes), "gdnstate_create: memset");
        if (rc == SQMIX_OK && conv_bytes > 0) {
            float *c = nullptr;
            rc = cuda_status(cudaMalloc(&c, conv_bytes), "gdnstate_create: cudaMalloc (conv)");
            if (c) st->conv_planes.push_back(c);
            if (rc == SQMIX_OK) rc = cuda_status(cudaMemset(c, 0, conv_bytes), "gdnstate_create: memset (conv)");
        }
    }
    if (rc == SQMIX_OK) rc = cuda_status(cudaMalloc(&st->d_sel, sizeof(int32_t)), "gdnstate_create: sel");
    if (rc == SQMIX_OK) rc = cuda_status(cudaMemset(st->d_sel, 0, sizeof(int32_t)), "gdnstate_create: sel");
    if (rc != SQMIX_OK) {
        sqmix_gdnstate_destroy(st);
        return rc;
    }
    *out = st;
    return SQMIX_OK;
}

extern "C" int sqmix_gdnstate_create(int32_t n_layers, int32_t h_v, int32_t n_rs, int32_t device,
                                     sqmix_gdnstate **out) {
    return sqmix_gdnstate_create_conv(n_layers, h_v, n_rs, 0, 0, device, out);
}

extern "C" void sqmix_gdnstate_destroy(sqmix_gdnstate *st) {
    if (!st) return;
    if (st->device < 0) {
        delete st;
        return;
    }
    DeviceGuard guard(st->device);
    for (float *p : st->planes) cudaFree(p);
    for (float *p : st->conv_planes) cudaFree(p);
    if (st->d_sel) cudaFree(st->d_sel);
    delete st;
}

extern "C" int sqmix_gdnstate_zero(sqmix_gdnstate *st, sqmix_stream_t stream) {
    if (!st) return SQMIX_EINVAL;
    if (st->device < 0) return SQMIX_OK;
    DeviceGuard guard(st->device);
    const size_t bytes = st->plane_elems() * sizeof(float) * (1 + st->n_rs);
    for (float *p : st->planes) {
        int rc = cuda_status(cudaMemsetAsync(p, 0, bytes, reinterpret_cast<cudaStream_t>(stream)),
                             "gdnstate_zero");
        if (rc != SQMIX_OK) return rc;
    }
    const size_t conv_bytes = st->conv_plane_elems() * sizeof(float) * (1 + st->n_rs);
    for (float *p : st->conv_planes) {
        int rc = cuda_status(cudaMemsetAsync(p, 0, conv_bytes, reinterpret_cast<cudaStream_t>(stream)),
                             "gdnstate_zero (conv)");
        if (rc != SQMIX_OK) return rc;
    }
    return SQMIX_OK;
}

extern "C" float *sqmix_gdnstate_planes(sqmix_gdnstate *st, int32_t layer) {
    return (st && layer >= 0 && layer < st->n_layers) ? st->planes[layer] : nullptr;
}
extern "C" float *sqmix_gdnstate_conv_planes(sqmix_gdnstate *st, int32_t layer) {
    return (st && layer >= 0 && layer < static_cast<int32_t>(st->conv_planes.size())) ? st->conv_planes[layer]
                                                                                      : nullptr;
}
extern "C" int32_t sqmix_gdnstate_n_planes(const sqmix_gdnstate *st) { return st ? 1 + st->n_rs : 0; }

extern "C" int32_t sqmix_gdnstate_set_sel(sqmix_gdnstate *st, int32_t sel) {
    if (!st) return -1;
    if (sel < 0) sel = 0;
    st->sel = sel < st->n_rs ? sel : st->n_rs;
    return st->sel;
}
extern "C" int32_t sqmix_gdnstate_sel(const sqmix_gdnstate *st) { return st ? st->sel : -1; }
extern "C" const int32_t *sqmix_gdnstate_device_sel(const sqmix_gdnstate *st) {
    return st ? st->d_sel : nullptr;
}

extern "C" int sqmix_gdnstate_upload_sel(sqmix_gdnstate *st, sqmix_stream_t stream) {
    if (!st) return SQMIX_EINVAL;
    const int32_t v = st->sel;
    // One-shot (graph.rs:187-189): the step that reads this selection consumes it.
    st->sel = 0;
    if (st->device < 0) return SQMIX_OK;
    DeviceGuard guard(st->device);
    return cuda_status(cudaMemcpyAsync(st->d_sel, &v, sizeof(int32_t), cudaMemcpyHostToDevice,
                                       reinterpret_cast<cudaStream_t>(stream)),
                       "gdnstate_upload_sel");
}

extern "C" size_t sqmix_gdnstate_snapshot_bytes(const sqmix_gdnstate *st) {
    return st ? 8 + (st->plane_elems() + st->conv_plane_elems()) * sizeof(float) * st->n_layers : 0;
}

extern "C" int sqmix_gdnstate_snapshot(sqmix_gdnstate *st, void *host_buf, size_t bytes,
                                       sqmix_stream_t stream) {
    if (!st || !host_buf) return SQMIX_EINVAL;
    const size_t need = sqmix_gdnstate_snapshot_bytes(st);
    if (bytes < need) {
        set_error("gdnstate_snapshot: buffer %zu < %zu bytes", bytes, need);
        return SQMIX_ENOSPC;
    }
    if (st->device < 0) {
        set_error("gdnstate_snapshot: bookkeeping-only state has no planes");
        return SQMIX_EINVAL;
    }
    DeviceGuard guard(st->device);
    const uint64_t payload = need - 8;
    uint8_t *dst = static_cast<uint8_t *>(host_buf);
    for (int i = 0; i < 8; ++i) dst[i] = static_cast<uint8_t>(payload >> (8 * i));  // little endian
    const size_t pb = st->plane_elems() * sizeof(float), cb = st->conv_plane_elems() * sizeof(float);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    for (int32_t l = 0; l < st->n_layers; ++l) {
        uint8_t *lay = dst + 8 + l * (pb + cb);
        int rc = cuda_status(cudaMemcpyAsync(lay, st->planes[l], pb, cudaMemcpyDeviceToHost, s), "gdnstate_snapshot");
        if (rc == SQMIX_OK && cb > 0)
            rc = cuda_status(cudaMemcpyAsync(lay + pb, st->conv_planes[l], cb, cudaMemcpyDeviceToHost, s),
                             "gdnstate_snapshot (conv)");
        if (rc != SQMIX_OK) return rc;
    }
    return cuda_status(cudaStreamSynchronize(s), "gdnstate_snapshot sync");
}

extern "C" int sqmix_gdnstate_restore(sqmix_gdnstate *st, const void *host_buf, size_t bytes,
                                      sqmix_stream_t stream) {
    if (!st || !host_buf) return SQMIX_EINVAL;
    const size_t want = sqmix_gdnstate_snapshot_bytes(st) - 8;
    if (bytes < 8) {
        set_error("GDN snapshot too short: %zu bytes", bytes);
        return SQMIX_EINVAL;
    }
    const uint8_t *src = static_cast<const uint8_t *>(host_buf);
    uint64_t declared = 0;
    for (int i = 0; i < 8; ++i) declared |= static_cast<uint64_t>(src[i]) << (8 * i);
    if (declared != want || bytes != want + 8) {
        set_error("GDN snapshot length mismatch: declared %llu + header, got %zu, expected %zu + header",
                  (unsigned long long)declared, bytes, want);
        return SQMIX_EINVAL;
    }
    if (st->device < 0) return SQMIX_OK;  // header validated; nothing to write
    DeviceGuard guard(st->device);
    const size_t pb = st->plane_elems() * sizeof(float), cb = st->conv_plane_elems() * sizeof(float);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    for (int32_t l = 0; l < st->n_layers; ++l) {
        const uint8_t *lay = src + 8 + l * (pb + cb);
        int rc = cuda_status(cudaMemcpyAsync(st->planes[l], lay, pb, cudaMemcpyHostToDevice, s), "gdnstate_restore");
        if (rc == SQMIX_OK && cb > 0)
            rc = cuda_status(cudaMemcpyAsync(st->conv_planes[l], lay + pb, cb, cudaMemcpyHostToDevice, s),
                             "gdnstate_restore (conv)");
        if (rc != SQMIX_OK) return rc;
    }
    return cuda_status(cudaStreamSynchronize(s), "gdnstate_restore sync");
}
