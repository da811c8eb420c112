// C ABI: context, QTensor, QMatMul and op entry points.  Every entry point
// converts exceptions into a status code plus a thread-local message; none of
// them aborts.
#include <cuda_fp16.h>
#include <string.h>

#include <memory>
#include <string>

#include "fb_internal.h"

namespace fb {

static thread_local std::string g_last_error;

void fail(int code, const std::string &msg) { throw Error(code, msg); }
void set_last_error(const std::string &msg) { g_last_error = msg; }

void check_cuda(cudaError_t e, const char *what, const char *file, int line) {
    if (e == cudaSuccess) return;
    const int code = (e == cudaErrorMemoryAllocation) ? FB_ERR_OOM : FB_ERR_CUDA;
    throw Error(code, std::string(what) + " failed: " + cudaGetErrorString(e) + " (" + file + ":" +
                          std::to_string(line) + ")");
}

DevBuf::~DevBuf() { release(); }
void DevBuf::alloc(size_t n) {
    release();
    if (n == 0) return;
    FB_CUDA(cudaMalloc(&ptr, n));
    bytes = n;
}
void DevBuf::release() {
    if (ptr) cudaFree(ptr);
    ptr = nullptr;
    bytes = 0;
}

}  // namespace fb

using namespace fb;

void *fb_ctx::ensure_scratch(size_t n) {
    if (scratch.bytes < n) {
        // scratch may be in use by queued work: drain the stream first
        FB_CUDA(cudaStreamSynchronize(stream));
        scratch.alloc(n);
    }
    return scratch.ptr;
}

size_t fb_qtensor::device_bytes(int dtype, int64_t n, int64_t k) {
    const int64_t nb = k / 256, np = (n + 15) / 16 * 16;  // tile-major, rows padded to 16
    switch (dtype) {
    case FB_Q4_K: return (size_t)(np * nb) * 144;
    case FB_Q6_K: return (size_t)(np * nb) * 210;
    case FB_F32: return (size_t)(n * k) * 4;
    default: return 0;
    }
}

static size_t gguf_bytes(int dtype, int64_t n, int64_t k) {
    const int64_t nb = k / 256;
    switch (dtype) {
    case FB_Q4_K: return (size_t)(n * nb) * 144;
    case FB_Q6_K: return (size_t)(n * nb) * 210;
    case FB_F32: return (size_t)(n * k) * 4;
    default: return 0;
    }
}

static void check_shape(int dtype, int64_t n, int64_t k) {
    FB_REQUIRE(n > 0 && k > 0, "tensor dims must be positive");
    FB_REQUIRE(dtype == FB_Q4_K || dtype == FB_Q6_K || dtype == FB_F32, "dtype must be FB_Q4_K, FB_Q6_K or FB_F32");
    if (dtype != FB_F32) FB_REQUIRE(k % 256 == 0, "k-quant tensors need k % 256 == 0");
}

extern "C" {

const char *fb_last_error(void) { return g_last_error.c_str(); }
int fb_abi_version(void) { return FB_ABI_VERSION; }

int fb_ctx_create(int device, void *stream, fb_ctx **out) {
    return guarded([&] {
        FB_REQUIRE(out != nullptr, "out is null");
        *out = nullptr;
        int ndev = 0;
        FB_CUDA(cudaGetDeviceCount(&ndev));
        FB_REQUIRE(device >= 0 && device < ndev, "device index out of range");
        FB_CUDA(cudaSetDevice(device));
        auto c = std::make_unique<fb_ctx>();
        c->device = device;
        c->stream = (cudaStream_t)stream;  // NULL = CUDA default stream
        FB_CUDA(cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, device));
        FB_CUDA(cudaMalloc(&c->err_word, 64));
        FB_CUDA(cudaMemset(c->err_word, 0, 64));
        *out = c.release();
    });
}

int fb_ctx_destroy(fb_ctx *ctx) {
    return guarded([&] {
        if (!ctx) return;
        cudaSetDevice(ctx->device);
        if (ctx->stream) cudaStreamSynchronize(ctx->stream);
        ctx->scratch.release();
        if (ctx->err_word) cudaFree(ctx->err_word);
        if (ctx->own_stream) cudaStreamDestroy(ctx->stream);
        delete ctx;
    });
}

int fb_ctx_set_stream(fb_ctx *ctx, void *stream) {
    return guarded([&] {
        FB_REQUIRE(ctx, "null ctx");
        FB_CUDA(cudaStreamSynchronize(ctx->stream));
        if (ctx->own_stream) {
            FB_CUDA(cudaStreamSynchronize(ctx->stream));
            FB_CUDA(cudaStreamDestroy(ctx->stream));
            ctx->own_stream = false;
        }
        ctx->stream = (cudaStream_t)stream;
    });
}

void *fb_ctx_stream(fb_ctx *ctx) { return ctx ? (void *)ctx->stream : nullptr; }

int fb_ctx_set_pdl(fb_ctx *ctx, int enable) {
    return guarded([&] {
        FB_REQUIRE(ctx, "null ctx");
        ctx->pdl = enable != 0;
    });
}

int fb_ctx_set_prefill_weight_cache(fb_ctx *ctx, int enable) {
    return guarded([&] {
        FB_REQUIRE(ctx, "null ctx");
        ctx->prefill_cache = enable != 0;
    });
}

int fb_sync(fb_ctx *ctx) {
    return guarded([&] {
        FB_REQUIRE(ctx, "null ctx");
        FB_CUDA(cudaStreamSynchronize(ctx->stream));
    });
}

int fb_ctx_error_word(fb_ctx *ctx, uint32_t *flags) {
    return guarded([&] {
        FB_REQUIRE(ctx && flags, "null argument");
        FB_CUDA(cudaMemcpyAsync(flags, ctx->err_word, 4, cudaMemcpyDeviceToHost, ctx->stream));
        FB_CUDA(cudaStreamSynchronize(ctx->stream));
        FB_CUDA(cudaMemsetAsync(ctx->err_word, 0, 4, ctx->stream));
    });
}

// ---------------------------------------------------------------- QTensor
static fb_qtensor *new_qtensor(fb_ctx *ctx, int dtype, int64_t n, int64_t k, const void *src,
                               cudaMemcpyKind kind) {
    check_shape(dtype, n, k);
    auto t = std::make_unique<fb_qtensor>();
    t->dtype = dtype;
    t->n = n;
    t->k = k;
    const size_t bytes = fb_qtensor::device_bytes(dtype, n, k);
    t->buf.alloc(bytes);
    if (dtype == FB_F32) {
        FB_CUDA(cudaMemcpyAsync(t->buf.ptr, src, bytes, kind, ctx->stream));
    } else {
        DevBuf staging;
        const void *gsrc = src;
        if (t->n_pad() != n) FB_CUDA(cudaMemsetAsync(t->buf.ptr, 0, bytes, ctx->stream));  // zero pad rows
        if (kind == cudaMemcpyHostToDevice) {
            staging.alloc(gguf_bytes(dtype, n, k));
            FB_CUDA(cudaMemcpyAsync(staging.ptr, src, staging.bytes, kind, ctx->stream));
            gsrc = staging.ptr;
        }
        launch_repack(ctx, dtype, n, k, gsrc, t->buf.ptr);
        FB_CUDA(cudaStreamSynchronize(ctx->stream));  // staging is freed on return
    }
    return t.release();
}

int fb_qtensor_upload(fb_ctx *ctx, int dtype, int64_t n, int64_t k, const void *host_blocks, fb_qtensor **out) {
    return guarded([&] {
        FB_REQUIRE(ctx && host_blocks && out, "null argument");
        *out = new_qtensor(ctx, dtype, n, k, host_blocks, cudaMemcpyHostToDevice);
        FB_CUDA(cudaStreamSynchronize(ctx->stream));
    });
}

int fb_qtensor_upload_dev(fb_ctx *ctx, int dtype, int64_t n, int64_t k, const void *dev_blocks, fb_qtensor **out) {
    return guarded([&] {
        FB_REQUIRE(ctx && dev_blocks && out, "null argument");
        *out = new_qtensor(ctx, dtype, n, k, dev_blocks, cudaMemcpyDeviceToDevice);
        FB_CUDA(cudaStreamSynchronize(ctx->stream));
    });
}

int fb_qtensor_synth(fb_ctx *ctx, int dtype, int64_t n, int64_t k, uint64_t seed, float sigma, fb_qtensor **out) {
    return guarded([&] {
        FB_REQUIRE(ctx && out, "null argument");
        check_shape(dtype, n, k);
        FB_REQUIRE(dtype != FB_F32, "synth: use a k-quant dtype");
        DevBuf staging;
        staging.alloc(gguf_bytes(dtype, n, k));
        launch_synth(ctx, dtype, n * (k / 256), seed, sigma, staging.ptr);
        *out = new_qtensor(ctx, dtype, n, k, staging.ptr, cudaMemcpyDeviceToDevice);
        FB_CUDA(cudaStreamSynchronize(ctx->stream));
    });
}

int fb_qtensor_upload_slice(fb_ctx *ctx, int dtype, int64_t n, int64_t k, const void *src_blocks, int src_on_device,
                            int64_t row0, int64_t rows, int64_t col0, int64_t cols, fb_qtensor **out) {
    return guarded([&] {
        FB_REQUIRE(ctx && src_blocks && out, "null argument");
        *out = nullptr;
        check_shape(dtype, n, k);
        FB_REQUIRE(dtype != FB_F32, "slice: use a k-quant dtype");
        FB_REQUIRE(row0 >= 0 && rows > 0 && row0 + rows <= n, "slice: rows out of range");
        FB_REQUIRE(col0 >= 0 && cols > 0 && col0 + cols <= k && col0 % 256 == 0 && cols % 256 == 0,
                   "slice: columns must be whole 256-value super-blocks inside the tensor");
        const size_t bb = dtype == FB_Q4_K ? 144 : 210;
        const size_t pitch = (size_t)(k / 256) * bb, width = (size_t)(cols / 256) * bb;
        const uint8_t *src = static_cast<const uint8_t *>(src_blocks) + (size_t)row0 * pitch + (size_t)(col0 / 256) * bb;
        DevBuf staging;
        staging.alloc(width * (size_t)rows);
        FB_CUDA(cudaMemcpy2DAsync(staging.ptr, width, src, pitch, width, (size_t)rows,
                                  src_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, ctx->stream));
        *out = new_qtensor(ctx, dtype, rows, cols, staging.ptr, cudaMemcpyDeviceToDevice);
        FB_CUDA(cudaStreamSynchronize(ctx->stream));
    });
}

int fb_qtensor_concat_rows(fb_ctx *ctx, const fb_qtensor *const *parts, int nparts, fb_qtensor **out) {
    return guarded([&] {
        FB_REQUIRE(ctx && parts && out && nparts > 0, "null argument");
        const int dtype = parts[0]->dtype;
        const int64_t k = parts[0]->k;
        int64_t n = 0;
        for (int i = 0; i < nparts; i++) {
            FB_REQUIRE(parts[i] && parts[i]->dtype == dtype && parts[i]->k == k, "concat: dtype and k must match");
            n += parts[i]->n;
        }
        for (int i = 0; i + 1 < nparts; i++)
            FB_REQUIRE(dtype == FB_F32 || parts[i]->n % 16 == 0,
                       "concat: all parts but the last need a multiple of 16 rows");
        auto t = std::make_unique<fb_qtensor>();
        t->dtype = dtype;
        t->n = n;
        t->k = k;
        t->buf.alloc(fb_qtensor::device_bytes(dtype, n, k));
        if (t->buf.bytes) FB_CUDA(cudaMemsetAsync(t->buf.ptr, 0, t->buf.bytes, ctx->stream));
        size_t off = 0;
        for (int i = 0; i < nparts; i++) {
            const fb_qtensor *p = parts[i];
            // tile-major records of whole 16-row tiles concatenate as bytes
            const size_t bytes = fb_qtensor::device_bytes(dtype, p->n, k);
            FB_CUDA(cudaMemcpyAsync(t->buf.as<uint8_t>() + off, p->main(), bytes, cudaMemcpyDeviceToDevice,
                                    ctx->stream));
            off += bytes;
        }
        FB_CUDA(cudaStreamSynchronize(ctx->stream));
        *out = t.release();
    });
}

int fb_qtensor_info(const fb_qtensor *t, int *dtype, int64_t *n, int64_t *k, int64_t *device_bytes) {
    return guarded([&] {
        FB_REQUIRE(t, "null tensor");
        if (dtype) *dtype = t->dtype;
        if (n) *n = t->n;
        if (k) *k = t->k;
        if (device_bytes) *device_bytes = (int64_t)t->buf.bytes;
    });
}

int fb_qtensor_download(fb_ctx *ctx, const fb_qtensor *t, void *host_blocks) {
    return guarded([&] {
        FB_REQUIRE(ctx && t && host_blocks, "null argument");
        const size_t bytes = gguf_bytes(t->dtype, t->n, t->k);
        if (t->dtype == FB_F32) {
            FB_CUDA(cudaMemcpyAsync(host_blocks, t->main(), bytes, cudaMemcpyDeviceToHost, ctx->stream));
        } else {
            DevBuf staging;
            staging.alloc(bytes);
            launch_unpack(ctx, t->dtype, t->n, t->k, t->main(), staging.ptr);
            FB_CUDA(cudaMemcpyAsync(host_blocks, staging.ptr, bytes, cudaMemcpyDeviceToHost, ctx->stream));
            FB_CUDA(cudaStreamSynchronize(ctx->stream));
        }
        FB_CUDA(cudaStreamSynchronize(ctx->stream));
    });
}

int fb_qtensor_destroy(fb_qtensor *t) {
    return guarded([&] { delete t; });
}

int fb_dequantize(fb_ctx *ctx, const fb_qtensor *t, void *out_dev, int out_dtype) {
    return guarded([&] {
        FB_REQUIRE(ctx && t && out_dev, "null argument");
        launch_dequantize(ctx, t, out_dev, out_dtype);
    });
}

// ---------------------------------------------------------------- QMatMul
static void qmatmul_q8k(fb_ctx *ctx, const fb_qtensor *w, const float *x, float *y, int64_t m) {
    FB_REQUIRE(w->dtype == FB_Q4_K || w->dtype == FB_Q6_K, "qmatmul: weight must be Q4_K or Q6_K");
    const int64_t chunk = m < 16 ? m : 16;
    void *base = ctx->ensure_scratch(q8act_bytes(chunk, w->k));
    Q8Act a = q8act_view(base, chunk, w->k);
    for (int64_t r = 0; r < m; r += 16) {
        const int64_t mm = (m - r) < 16 ? (m - r) : 16;
        launch_quantize_q8k(ctx, x + r * w->k, mm, w->k, a);
        launch_gemv(ctx, w, a, (int)mm, y + r * w->n, w->n);
    }
}

int fb_qmatmul_q8k(fb_ctx *ctx, const fb_qtensor *w, const float *x_dev, float *y_dev, int64_t m) {
    return guarded([&] {
        FB_REQUIRE(ctx && w && x_dev && y_dev, "null argument");
        FB_REQUIRE(m >= 1, "m must be >= 1");
        qmatmul_q8k(ctx, w, x_dev, y_dev, m);
    });
}

int fb_qmatmul(fb_ctx *ctx, const fb_qtensor *w, const float *x_dev, float *y_dev, int64_t m) {
    return guarded([&] {
        FB_REQUIRE(ctx && w && x_dev && y_dev, "null argument");
        FB_REQUIRE(m >= 1, "m must be >= 1");
        if (m <= 16) qmatmul_q8k(ctx, w, x_dev, y_dev, m);
        else qmatmul_prefill(ctx, w, x_dev, y_dev, m);
    });
}

int fb_quantize_q8k(fb_ctx *ctx, const float *x_dev, int64_t m, int64_t k, void *q8k_dev) {
    return guarded([&] {
        FB_REQUIRE(ctx && x_dev && q8k_dev, "null argument");
        FB_REQUIRE(m >= 1 && k >= 256 && k % 256 == 0, "need m >= 1 and k % 256 == 0");
        launch_quantize_q8k_gguf(ctx, x_dev, m, k, q8k_dev);
    });
}

int fb_block_dots(fb_ctx *ctx, const fb_qtensor *w, const float *x_dev, int32_t *out_sc_dev, int32_t *out_min_dev) {
    return guarded([&] {
        FB_REQUIRE(ctx && w && x_dev && out_sc_dev && out_min_dev, "null argument");
        FB_REQUIRE(w->dtype == FB_Q4_K || w->dtype == FB_Q6_K, "block_dots: weight must be Q4_K or Q6_K");
        void *base = ctx->ensure_scratch(q8act_bytes(1, w->k));
        Q8Act a = q8act_view(base, 1, w->k);
        launch_quantize_q8k(ctx, x_dev, 1, w->k, a);
        launch_block_dots(ctx, w, a, out_sc_dev, out_min_dev);
    });
}

// ---------------------------------------------------------------- ops
int fb_rmsnorm(fb_ctx *ctx, const float *x_dev, const float *g_dev, float *y_dev, int64_t rows, int64_t dim,
               float eps) {
    return guarded([&] {
        FB_REQUIRE(ctx && x_dev && g_dev && y_dev, "null argument");
        FB_REQUIRE(rows >= 1 && dim >= 1, "bad shape");
        launch_rmsnorm(ctx, x_dev, g_dev, y_dev, rows, dim, eps);
    });
}

int fb_rope(fb_ctx *ctx, float *x_dev, int64_t n_tok, int64_t n_heads, int64_t head_dim, int64_t pos0, float theta,
            int mode) {
    return guarded([&] {
        FB_REQUIRE(ctx && x_dev, "null argument");
        FB_REQUIRE(n_tok >= 1 && n_heads >= 1 && head_dim >= 2 && head_dim % 2 == 0 && pos0 >= 0, "bad shape");
        FB_REQUIRE(mode == 0 || mode == 1, "mode must be 0 or 1");
        std::vector<float> ct, st;
        rope_tables((int)(pos0 + n_tok), (int)head_dim, theta, ct, st);
        DevBuf tabs;
        tabs.alloc((ct.size() + st.size()) * 4);
        FB_CUDA(cudaMemcpyAsync(tabs.ptr, ct.data(), ct.size() * 4, cudaMemcpyHostToDevice, ctx->stream));
        FB_CUDA(cudaMemcpyAsync(tabs.as<float>() + ct.size(), st.data(), st.size() * 4, cudaMemcpyHostToDevice,
                                ctx->stream));
        launch_rope(ctx, x_dev, n_tok, n_heads, head_dim, pos0, tabs.as<float>(), tabs.as<float>() + ct.size(), mode);
        FB_CUDA(cudaStreamSynchronize(ctx->stream));
    });
}

int fb_swiglu(fb_ctx *ctx, const float *gate_dev, const float *up_dev, float *out_dev, int64_t m, int64_t f) {
    return guarded([&] {
        FB_REQUIRE(ctx && gate_dev && up_dev && out_dev, "null argument");
        FB_REQUIRE(m >= 1 && f >= 1, "bad shape");
        launch_swiglu(ctx, gate_dev, up_dev, out_dev, m, f);
    });
}

}  // extern "C"
