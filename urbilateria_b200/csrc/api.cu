// api.cu — the C ABI (include/urb_moe.h): contexts, resident matrices, matrix products,
// routing, grouping and the MoE layer.  Host-pointer entry points validate arguments in the
// reference's order, copy inputs to the device, run the device path and copy results back.
#include <cmath>
#include <cstring>

#include "urb_internal.cuh"
#include "urb_moe_internal.cuh"

namespace urb {

int set_error(Ctx *ctx, int status, const std::string &msg) {
    if (ctx) {
        ctx->last_status = status;
        ctx->last_error = msg;
    }
    return status;
}

int cuda_fail(Ctx *ctx, cudaError_t err, const char *what) {
    return set_error(ctx, URB_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(err));
}

void *workspace(Ctx *ctx, size_t bytes, int *status) {
    *status = URB_OK;
    if (bytes <= ctx->ws_size) return ctx->ws;
    size_t want = std::max(bytes, ctx->ws_size * 2);
    if (ctx->ws) cudaFreeAsync(ctx->ws, ctx->stream);
    ctx->ws = nullptr;
    ctx->ws_size = 0;
    cudaError_t e = cudaMallocAsync(&ctx->ws, want, ctx->stream);
    if (e != cudaSuccess) {
        *status = cuda_fail(ctx, e, "workspace allocation");
        return nullptr;
    }
    ctx->ws_size = want;
    return ctx->ws;
}

void *io_buffer(Ctx *ctx, size_t bytes, int *status) {
    *status = URB_OK;
    if (bytes <= ctx->io_size) return ctx->io;
    size_t want = std::max(bytes, ctx->io_size * 2);
    if (ctx->io) cudaFreeAsync(ctx->io, ctx->stream);
    ctx->io = nullptr;
    ctx->io_size = 0;
    cudaError_t e = cudaMallocAsync(&ctx->io, want, ctx->stream);
    if (e != cudaSuccess) {
        *status = cuda_fail(ctx, e, "input/output staging allocation");
        return nullptr;
    }
    ctx->io_size = want;
    return ctx->io;
}

void *pinned_staging(Ctx *ctx, size_t bytes, int *status) {
    *status = URB_OK;
    if (bytes <= ctx->pinned_size) return ctx->pinned;
    size_t want = std::max(bytes, ctx->pinned_size * 2);
    if (ctx->pinned) {
        // A copy on the stream may still read or write the old buffer.
        cudaStreamSynchronize(ctx->stream);
        cudaFreeHost(ctx->pinned);
    }
    ctx->pinned = nullptr;
    ctx->pinned_size = 0;
    cudaError_t e = cudaHostAlloc(&ctx->pinned, want, cudaHostAllocDefault);
    if (e != cudaSuccess) {
        *status = cuda_fail(ctx, e, "pinned staging allocation");
        return nullptr;
    }
    ctx->pinned_size = want;
    return ctx->pinned;
}

static cudaEvent_t prof_event(Ctx *ctx) {
    if (!ctx->prof_free.empty()) {
        cudaEvent_t e = ctx->prof_free.back();
        ctx->prof_free.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
}

void prof_begin(Ctx *ctx, int kind, cudaStream_t st) {
    if (!ctx || !ctx->prof) return;
    ctx->prof_open = kind;
    ctx->prof_open_ev = prof_event(ctx);
    cudaEventRecord(ctx->prof_open_ev, st);
}

void prof_end(Ctx *ctx, cudaStream_t st) {
    if (!ctx || !ctx->prof || ctx->prof_open < 0) return;
    cudaEvent_t b = prof_event(ctx);
    cudaEventRecord(b, st);
    ctx->prof_pending.push_back({ctx->prof_open, ctx->prof_open_ev, b});
    ctx->prof_open = -1;
}

static void prof_drain(Ctx *ctx) {
    for (auto &r : ctx->prof_pending) {
        cudaEventSynchronize(r.b);
        float ms = 0.0f;
        if (cudaEventElapsedTime(&ms, r.a, r.b) == cudaSuccess) {
            ctx->prof_ms[r.kind] += ms;
            ctx->prof_n[r.kind] += 1;
        }
        ctx->prof_free.push_back(r.a);
        ctx->prof_free.push_back(r.b);
    }
    ctx->prof_pending.clear();
}

namespace {

struct Carve {
    uint8_t *base;
    size_t off = 0;
    template <class T>
    T *take(size_t n) {
        off = (off + 255) & ~size_t(255);
        T *p = reinterpret_cast<T *>(base + off);
        off += n * sizeof(T);
        return p;
    }
};

size_t div_ceil(size_t a, size_t b) { return (a + b - 1) / b; }

bool all_finite(const float *v, size_t n) {
    for (size_t i = 0; i < n; ++i)
        if (!std::isfinite(v[i])) return false;
    return true;
}

int pick_ksplit(Ctx *ctx, long total_rows) {
    long per = total_rows / std::max(1, ctx->num_sms);
    return per < 64 ? 8 : (per < 256 ? 2 : 1);
}

// y[batch, out_rows] (stride out_rows) = W[rb_lo*16 .. rb_hi*16) x for a tiled matrix.
int tiled_product(Ctx *ctx, const Mat *m, int rb_lo, int rb_hi, const float *d_x, int batch,
                  const int32_t *d_shift, float *d_y, Carve &cv, cudaStream_t st) {
    const int cap = 8;  // tokens per segment (hi/lo -> 16 activation columns)
    const int nseg = int(div_ceil(batch, cap));
    std::vector<Seg> segs(nseg);
    const int TB = tile_bytes(m->format);
    for (int i = 0; i < nseg; ++i) {
        Seg &s = segs[i];
        s.tiles_a = m->tiles + size_t(rb_lo) * m->kslices * TB;
        s.rexp_a = m->row_exp + size_t(rb_lo) * 16;
        s.tiles_b = nullptr;
        s.rexp_b = nullptr;
        s.rbs = rb_hi - rb_lo;
        s.rows = int(std::min<size_t>(m->rows - size_t(rb_lo) * 16, size_t(s.rbs) * 16));
        s.kslices = m->kslices;
        s.cols = int(m->cols);
        s.col_begin = i * cap;
        s.ntok = std::min(cap, batch - i * cap);
        s.row_begin = i * 16 * s.rbs;
        s.pad = 0;
    }
    Seg *d_segs = cv.take<Seg>(nseg);
    int *d_sc = cv.take<int>(2);
    int sc[2] = {nseg, nseg * 16 * (rb_hi - rb_lo)};
    URB_CUDA(ctx, cudaMemcpyAsync(d_segs, segs.data(), nseg * sizeof(Seg), cudaMemcpyHostToDevice, st));
    URB_CUDA(ctx, cudaMemcpyAsync(d_sc, sc, sizeof(sc), cudaMemcpyHostToDevice, st));
    GroupArgs a{};
    a.segs = d_segs;
    a.nsegs = d_sc;
    a.total_rows = d_sc + 1;
    a.src = d_x;
    a.src_stride = int(m->cols);
    a.col_src = nullptr;
    a.src_shift = d_shift;
    a.src_maxexp = nullptr;
    a.out = d_y;
    a.out_stride = (rb_hi - rb_lo) * 16;
    a.out_maxexp = nullptr;
    a.hilo = 1;
    int max_cols = 2 * std::min(cap, batch);
    // Host-built segment arrays are consumed by the kernel before the pageable sources die:
    // cudaMemcpyAsync from pageable memory returns after staging.
    prof_begin(ctx, URB_K_PRODUCT, st);
    int rc = launch_grouped_ex(ctx, m->format, false, pick_ksplit(ctx, sc[1]), a, max_cols,
                               m->kslices, st);
    prof_end(ctx, st);
    return rc;
}

// URB_MATVEC=cuda_cores selects the CUDA-core single-token kernel over the tensor-core one
// (for comparison; both read resident tiles of the same matrix).
bool matvec_cuda_cores() {
    static const bool on = [] {
        const char *v = std::getenv("URB_MATVEC");
        return v && std::strcmp(v, "cuda_cores") == 0;
    }();
    return on;
}

// Product of rows [start, start+count) for `batch` tokens; d_y is [batch, count].
int device_product(Ctx *ctx, const Mat *m, size_t start, size_t count, const float *d_x,
                   size_t batch, float *d_y, int32_t *d_status, cudaStream_t st) {
    if (is_int_format(m->format)) {
        // Int8Matrix / Int4Matrix: warp-per-row f64 products over the packed payload.
        prof_begin(ctx, URB_K_PRODUCT, st);
        int rc = launch_int_matmul(ctx, m, start, count, d_x, batch, d_y, d_status, st);
        prof_end(ctx, st);
        return rc;
    }
    if (split_tc_applies(m, batch) && start == 0 && count == m->rows) {
        // BF16, 1..32 tokens, whole rows: split-K tcgen05 clusters (split_tc.cu).
        int rc = split_tc_product(ctx, m, d_x, int(batch), d_y, d_status, st);
        if (rc != URB_ERR_UNSUPPORTED) return rc;
    }
    if (m->format == URB_FMT_BF16 && dense_tc_applies(m) && batch > 32) {
        // BF16, more tokens: the grouped tcgen05 pass with every token in one group.
        int rc = dense_tc_product(ctx, m, start, count, d_x, int(batch), d_y, d_status, st);
        if (rc != URB_ERR_UNSUPPORTED) return rc;
    }
    if (bf16_gemv_applies(m, batch)) {
        // BF16 rows for a few tokens (row ranges): one streaming pass on CUDA cores.
        prof_begin(ctx, URB_K_PRODUCT, st);
        int rc = launch_bf16_gemv(ctx, m, start, count, d_x, batch, d_y, d_status, st);
        prof_end(ctx, st);
        if (rc != URB_ERR_UNSUPPORTED) return rc;
    }
    if (matvec_tc_applies(m) && !(batch == 1 && matvec_cuda_cores())) {
        // MX matrices: the resident tcgen05 tiles.  One token: digit-term x, split-K clusters
        // (matvec_tc.cu); more tokens, or K longer than the clusters hold: the grouped
        // tensor-core pass with every token in one group (dense_tc.cu).
        int rc = URB_ERR_UNSUPPORTED;
        if (batch == 1) {
            prof_begin(ctx, URB_K_PRODUCT, st);
            rc = launch_matvec_tc(ctx, m, start, count, d_x, d_y, d_status, st);
            prof_end(ctx, st);
        }
        if (rc == URB_ERR_UNSUPPORTED)
            rc = dense_tc_product(ctx, m, start, count, d_x, int(batch), d_y, d_status, st);
        return rc;
    }
    if (!m->tiled) {
        prof_begin(ctx, URB_K_PRODUCT, st);
        int rc = launch_generic_matmul(ctx, m, start, count, d_x, batch, d_y, st);
        prof_end(ctx, st);
        return rc;
    }
    if (batch == 1 && (m->format == URB_FMT_MXFP4 || m->format == URB_FMT_MXFP8) && !d_status) {
        // URB_MATVEC=cuda_cores: the CUDA-core kernel over the mma.sync tiles (no activation
        // shifts needed; input finiteness is checked by the host entry points, or through
        // d_status below).
        int rc = ensure_mma_tiles(ctx, m, st);
        if (rc) return rc;
        prof_begin(ctx, URB_K_PRODUCT, st);
        rc = launch_matvec1(ctx, m, start, count, d_x, d_y, st);
        prof_end(ctx, st);
        return rc;
    }
    int rc = ensure_mma_tiles(ctx, m, st);  // MX here only under URB_MATVEC=cuda_cores
    if (rc) return rc;
    int rb_lo = int(start / 16), rb_hi = int(div_ceil(start + count, 16));
    size_t out_rows = size_t(rb_hi - rb_lo) * 16;
    size_t need = batch * 4 + batch * out_rows * 4 + 64 * 1024 + 4096;
    uint8_t *ws = static_cast<uint8_t *>(workspace(ctx, need, &rc));
    if (!ws) return rc;
    Carve cv{ws};
    int32_t *d_shift = cv.take<int32_t>(batch);
    bool direct = (start % 16 == 0) && out_rows == count;  // output lands in place
    float *d_tmp = direct ? d_y : cv.take<float>(batch * out_rows);
    prof_begin(ctx, URB_K_ROW_SHIFT, st);
    rc = launch_row_shift(d_x, int(batch), int(m->cols), int(m->cols), d_shift, d_status, st);
    prof_end(ctx, st);
    if (rc) return cuda_fail(ctx, cudaGetLastError(), "row shift");
    rc = tiled_product(ctx, m, rb_lo, rb_hi, d_x, int(batch), d_shift, d_tmp, cv, st);
    if (rc) return rc;
    if (!direct) {
        URB_CUDA(ctx, cudaMemcpy2DAsync(d_y, count * 4, d_tmp + (start - size_t(rb_lo) * 16),
                                        out_rows * 4, count * 4, batch, cudaMemcpyDeviceToDevice, st));
    }
    return URB_OK;
}

// Host-pointer product: x staged through the context's pinned buffer into its device I/O
// buffer, computed, y back the same way (no allocation once the buffers have grown).
int host_product(Ctx *ctx, const Mat *m, size_t start, size_t count, const float *x,
                 size_t batch, float *y) {
    cudaStream_t st = ctx->stream;
    const size_t xb = batch * m->cols * 4, yb = batch * count * 4, xb_al = (xb + 255) & ~size_t(255);
    int rc;
    uint8_t *io = static_cast<uint8_t *>(io_buffer(ctx, xb_al + yb, &rc));
    if (!io) return rc;
    float *hs = static_cast<float *>(pinned_staging(ctx, std::max(xb, yb), &rc));
    if (!hs) return rc;
    float *d_x = reinterpret_cast<float *>(io), *d_y = reinterpret_cast<float *>(io + xb_al);
    // The pinned buffer may still feed an earlier call's copy on this stream.
    URB_CUDA(ctx, cudaStreamSynchronize(st));
    std::memcpy(hs, x, xb);
    URB_CUDA(ctx, cudaMemcpyAsync(d_x, hs, xb, cudaMemcpyHostToDevice, st));
    rc = device_product(ctx, m, start, count, d_x, batch, d_y, nullptr, st);
    if (rc) return rc;
    URB_CUDA(ctx, cudaMemcpyAsync(hs, d_y, yb, cudaMemcpyDeviceToHost, st));
    URB_CUDA(ctx, cudaStreamSynchronize(st));
    std::memcpy(y, hs, yb);
    return URB_OK;
}

int new_mat(urb_ctx *ctx, int fmt, size_t rows, size_t cols, urb_mat **out) {
    if (!ctx || !out) return URB_ERR_INVALID_ARGUMENT;
    *out = nullptr;
    urb_mat *m = new urb_mat();
    m->ctx = ctx;
    m->format = fmt;
    m->rows = rows;
    m->cols = cols;
    *out = m;
    return URB_OK;
}

int finish_upload(urb_ctx *ctx, urb_mat *m, const void *values, const uint8_t *scales,
                  urb_mat **out) {
    int rc = upload_matrix(ctx, m, values, scales);
    if (rc != URB_OK) {
        urb_mat_free(m);
        *out = nullptr;
        return rc;
    }
    *out = m;
    return URB_OK;
}

}  // namespace

int product_device(Ctx *ctx, const Mat *m, size_t start, size_t count, const float *d_x,
                   size_t batch, float *d_y, int32_t *d_status, cudaStream_t st) {
    return device_product(ctx, m, start, count, d_x, batch, d_y, d_status, st);
}

}  // namespace urb

using namespace urb;

extern "C" {

int urb_ctx_create(int device, urb_ctx **out) {
    if (!out) return URB_ERR_INVALID_ARGUMENT;
    *out = nullptr;
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return URB_ERR_CUDA;
    urb_ctx *ctx = new urb_ctx();
    ctx->device = device;
    cudaDeviceGetAttribute(&ctx->num_sms, cudaDevAttrMultiProcessorCount, device);
    if (cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking) != cudaSuccess) {
        delete ctx;
        return URB_ERR_CUDA;
    }
    ctx->own_stream = true;
    if (cudaStreamCreateWithFlags(&ctx->aux, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&ctx->ev_fork, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&ctx->ev_join, cudaEventDisableTiming) != cudaSuccess ||
        cudaMalloc(&ctx->d_status, sizeof(int32_t)) != cudaSuccess || expf_table_init(ctx) != URB_OK) {
        urb_ctx_destroy(ctx);
        return URB_ERR_CUDA;
    }
    *out = ctx;
    return URB_OK;
}

int urb_ctx_destroy(urb_ctx *ctx) {
    if (!ctx) return URB_ERR_INVALID_ARGUMENT;
    cudaSetDevice(ctx->device);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    if (ctx->aux) cudaStreamSynchronize(ctx->aux);
    if (ctx->ws) cudaFree(ctx->ws);
    if (ctx->io) cudaFree(ctx->io);
    if (ctx->d_status) cudaFree(ctx->d_status);
    if (ctx->expf_keys) cudaFree(const_cast<uint32_t *>(ctx->expf_keys));
    if (ctx->log1pf_keys) cudaFree(const_cast<uint32_t *>(ctx->log1pf_keys));
    if (ctx->pinned) cudaFreeHost(ctx->pinned);
    if (ctx->own_stream && ctx->stream) cudaStreamDestroy(ctx->stream);
    if (ctx->aux) cudaStreamDestroy(ctx->aux);
    if (ctx->ev_fork) cudaEventDestroy(ctx->ev_fork);
    if (ctx->ev_join) cudaEventDestroy(ctx->ev_join);
    delete ctx;
    return URB_OK;
}

int urb_ctx_set_stream(urb_ctx *ctx, void *stream) {
    if (!ctx) return URB_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    if (ctx->own_stream && ctx->stream) cudaStreamSynchronize(ctx->stream);
    if (ctx->own_stream && ctx->stream) cudaStreamDestroy(ctx->stream);
    ctx->stream = static_cast<cudaStream_t>(stream);
    ctx->own_stream = false;
    return URB_OK;
}

void *urb_ctx_stream(urb_ctx *ctx) { return ctx ? ctx->stream : nullptr; }

int urb_last_error(urb_ctx *ctx, char *buf, size_t len) {
    if (!ctx) return URB_ERR_INVALID_ARGUMENT;
    if (buf && len) {
        size_t n = std::min(len - 1, ctx->last_error.size());
        std::memcpy(buf, ctx->last_error.data(), n);
        buf[n] = 0;
    }
    return ctx->last_status;
}

int urb_ctx_synchronize(urb_ctx *ctx) {
    if (!ctx) return URB_ERR_INVALID_ARGUMENT;
    URB_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    return URB_OK;
}

int urb_mxfp4_upload(urb_ctx *ctx, size_t rows, size_t cols, size_t group_size,
                     const uint8_t *packed, size_t packed_len, const uint8_t *scales,
                     size_t scales_len, urb_mat **out) {
    if (!ctx || !out || !packed || !scales) return URB_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    cudaSetDevice(ctx->device);
    // mxfp.rs:1415-1430: non-zero dimensions, exact payload sizes.
    if (rows == 0 || cols == 0 || group_size == 0)
        return set_error(ctx, URB_ERR_SHAPE, "dimensions and group size must be non-zero");
    if (packed_len != rows * div_ceil(cols, 2) || scales_len != rows * div_ceil(cols, group_size))
        return set_error(ctx, URB_ERR_SHAPE, "packed/scale byte counts do not match the shape");
    urb_mat *m;
    new_mat(ctx, URB_FMT_MXFP4, rows, cols, &m);
    m->group_size = group_size;
    return finish_upload(ctx, m, packed, scales, out);
}

int urb_mxfp8_upload(urb_ctx *ctx, size_t rows, size_t cols, size_t block_rows,
                     size_t block_cols, const uint8_t *values, size_t values_len,
                     const uint8_t *scales, size_t scales_len, urb_mat **out) {
    if (!ctx || !out || !values || !scales) return URB_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    cudaSetDevice(ctx->device);
    if (rows == 0 || cols == 0 || block_rows == 0 || block_cols == 0)
        return set_error(ctx, URB_ERR_SHAPE, "dimensions and block dimensions must be non-zero");
    if (values_len != rows * cols ||
        scales_len != div_ceil(rows, block_rows) * div_ceil(cols, block_cols))
        return set_error(ctx, URB_ERR_SHAPE, "value/scale counts do not match the shape");
    urb_mat *m;
    new_mat(ctx, URB_FMT_MXFP8, rows, cols, &m);
    m->block_rows = block_rows;
    m->block_cols = block_cols;
    return finish_upload(ctx, m, values, scales, out);
}

int urb_bf16_upload(urb_ctx *ctx, size_t rows, size_t cols, const uint16_t *values,
                    size_t values_len, urb_mat **out) {
    if (!ctx || !out || !values) return URB_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    cudaSetDevice(ctx->device);
    if (rows == 0 || cols == 0 || values_len != rows * cols)
        return set_error(ctx, URB_ERR_SHAPE, "bf16 matrix shape does not match its payload");
    urb_mat *m;
    new_mat(ctx, URB_FMT_BF16, rows, cols, &m);
    return finish_upload(ctx, m, values, nullptr, out);
}

int urb_f32_upload(urb_ctx *ctx, size_t rows, size_t cols, const float *values,
                   size_t values_len, urb_mat **out) {
    if (!ctx || !out || !values) return URB_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    cudaSetDevice(ctx->device);
    if (rows == 0 || cols == 0 || values_len != rows * cols)
        return set_error(ctx, URB_ERR_SHAPE, "f32 matrix shape does not match its payload");
    urb_mat *m;
    new_mat(ctx, URB_FMT_F32, rows, cols, &m);
    return finish_upload(ctx, m, values, nullptr, out);
}

int urb_int8_upload(urb_ctx *ctx, size_t rows, size_t cols, const uint8_t *bytes,
                    size_t bytes_len, const float *scales, size_t scales_len, urb_mat **out) {
    if (!ctx || !out || !bytes || !scales) return URB_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    cudaSetDevice(ctx->device);
    // quant.rs:369-383: non-zero shape with an exact payload, then one scale per row.
    if (rows == 0 || cols == 0 || bytes_len != rows * cols)
        return set_error(ctx, URB_ERR_SHAPE, "INT8 payload does not match the shape");
    if (scales_len != rows) return set_error(ctx, URB_ERR_SHAPE, "INT8 needs one scale per row");
    urb_mat *m;
    new_mat(ctx, URB_FMT_INT8, rows, cols, &m);
    return finish_upload(ctx, m, bytes, reinterpret_cast<const uint8_t *>(scales), out);
}

int urb_int4_upload(urb_ctx *ctx, size_t rows, size_t cols, size_t group_size,
                    const uint8_t *packed, size_t packed_len, const float *scales,
                    size_t scales_len, urb_mat **out) {
    if (!ctx || !out || !packed || !scales) return URB_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    cudaSetDevice(ctx->device);
    // quant.rs:99-118, 575-598: group size, non-zero shape, payload and scale counts.
    if (group_size == 0) return set_error(ctx, URB_ERR_INVALID_GROUP, "INT4 group size must be greater than zero");
    if (rows == 0 || cols == 0) return set_error(ctx, URB_ERR_SHAPE, "rows and columns must be non-zero");
    if (packed_len != rows * div_ceil(cols, 2))
        return set_error(ctx, URB_ERR_SHAPE, "INT4 packed byte count does not match the shape");
    if (scales_len != rows * div_ceil(cols, group_size))
        return set_error(ctx, URB_ERR_SHAPE, "INT4 scale count does not match the shape");
    urb_mat *m;
    new_mat(ctx, URB_FMT_INT4, rows, cols, &m);
    m->group_size = group_size;
    return finish_upload(ctx, m, packed, reinterpret_cast<const uint8_t *>(scales), out);
}

int urb_int4_quantize_grouped(urb_ctx *ctx, size_t rows, size_t cols, size_t group_size,
                              const float *values, size_t values_len, urb_mat **out) {
    if (!ctx || !out || !values) return URB_ERR_INVALID_ARGUMENT;
    *out = nullptr;
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    cudaSetDevice(ctx->device);
    if (group_size == 0) return set_error(ctx, URB_ERR_INVALID_GROUP, "INT4 group size must be greater than zero");
    if (rows == 0 || cols == 0) return set_error(ctx, URB_ERR_SHAPE, "rows and columns must be non-zero");
    if (values_len != rows * cols) return set_error(ctx, URB_ERR_SHAPE, "INT4 source length does not match the shape");
    cudaStream_t st = ctx->stream;
    const size_t nv = rows * cols * sizeof(float), np = rows * div_ceil(cols, 2),
                 ns = rows * div_ceil(cols, group_size) * sizeof(float);
    uint8_t *d = nullptr;
    URB_CUDA(ctx, cudaMallocAsync(&d, nv + ns + np + 64, st));
    float *d_v = reinterpret_cast<float *>(d), *d_s = reinterpret_cast<float *>(d + nv);
    uint8_t *d_p = d + nv + ns;
    int32_t *d_flag = reinterpret_cast<int32_t *>(d + ((nv + ns + np + 15) / 16) * 16);
    int rc = URB_OK;
    cudaError_t e = cudaMemcpyAsync(d_v, values, nv, cudaMemcpyDefault, st);
    if (e != cudaSuccess) rc = cuda_fail(ctx, e, "INT4 source copy");
    if (rc == URB_OK) rc = int4_quantize_device(ctx, rows, cols, group_size, d_v, d_p, d_s, d_flag, st);
    if (rc == URB_OK) rc = urb_int4_upload(ctx, rows, cols, group_size, d_p, np, d_s, ns / sizeof(float), out);
    cudaFreeAsync(d, st);
    cudaStreamSynchronize(st);
    return rc;
}

int urb_int4_payload(urb_ctx *ctx, const urb_mat *m, uint8_t *packed, float *scales) {
    if (!ctx || !m || !packed || !scales) return URB_ERR_INVALID_ARGUMENT;
    if (m->format != URB_FMT_INT4) return set_error(ctx, URB_ERR_UNSUPPORTED, "not an INT4 matrix");
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    cudaSetDevice(ctx->device);
    cudaStream_t st = ctx->stream;
    URB_CUDA(ctx, cudaMemcpyAsync(packed, m->raw_values, m->rows * div_ceil(m->cols, 2), cudaMemcpyDefault, st));
    URB_CUDA(ctx, cudaMemcpyAsync(scales, m->raw_scales,
                                  m->rows * div_ceil(m->cols, m->group_size) * sizeof(float), cudaMemcpyDefault, st));
    URB_CUDA(ctx, cudaStreamSynchronize(st));
    return URB_OK;
}

int urb_mat_free(urb_mat *m) {
    if (!m) return URB_ERR_INVALID_ARGUMENT;
    if (m->ctx) {
        cudaSetDevice(m->ctx->device);
        cudaStreamSynchronize(m->ctx->stream);
    }
    if (m->tiles) cudaFree(m->tiles);
    if (m->tc_tiles) cudaFree(m->tc_tiles);
    if (m->tc_map) cudaFree(m->tc_map);
    if (m->row_exp) cudaFree(m->row_exp);
    if (m->raw_values) cudaFree(m->raw_values);
    if (m->raw_scales) cudaFree(m->raw_scales);
    delete m;
    return URB_OK;
}

int urb_mat_info(const urb_mat *m, int *format, size_t *rows, size_t *cols, size_t *resident) {
    if (!m) return URB_ERR_INVALID_ARGUMENT;
    if (format) *format = m->format;
    if (rows) *rows = m->rows;
    if (cols) *cols = m->cols;
    if (resident) *resident = m->resident_bytes;
    return URB_OK;
}

int urb_matvec_rows(urb_ctx *ctx, const urb_mat *m, size_t start, size_t count, const float *x,
                    size_t x_len, float *y) {
    if (!ctx || !m || !x || (!y && count)) return URB_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    cudaSetDevice(ctx->device);
    // Validation order of every format: input length, input finiteness, row range.
    if (x_len != m->cols) return set_error(ctx, URB_ERR_SHAPE, "matvec input length mismatch");
    if (!all_finite(x, x_len)) return set_error(ctx, URB_ERR_NONFINITE, "matvec input contains NaN or infinity");
    if (start + count < start || start + count > m->rows)
        return set_error(ctx, URB_ERR_SHAPE, "matvec row range is out of bounds");
    if (count == 0) return URB_OK;
    int rc = host_product(ctx, m, start, count, x, 1, y);
    if (rc) return rc;
    // Only MXFP8 rejects non-finite outputs on this path (mxfp.rs:712-714).
    if (m->format == URB_FMT_MXFP8 && !all_finite(y, count))
        return set_error(ctx, URB_ERR_NONFINITE, "MXFP8 matvec produced a non-finite output");
    return URB_OK;
}

static int matmul_common(urb_ctx *ctx, const urb_mat *m, size_t start, size_t count,
                         const float *x, size_t batch, size_t x_len, float *y) {
    if (!ctx || !m || !x || !y) return URB_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    cudaSetDevice(ctx->device);
    if (batch == 0 || x_len != batch * m->cols)
        return set_error(ctx, URB_ERR_SHAPE, "batched matvec expects a non-zero batch of full rows");
    if (!all_finite(x, x_len)) return set_error(ctx, URB_ERR_NONFINITE, "batched input contains NaN or infinity");
    if (start + count < start || start + count > m->rows)
        return set_error(ctx, URB_ERR_SHAPE, "batched matvec row range is out of bounds");
    int rc = host_product(ctx, m, start, count, x, batch, y);
    if (rc) return rc;
    // Output finiteness, chunk by chunk as WeightMatrix::matmul_rows splits (weight.rs:116-146).
    if (m->format == URB_FMT_MXFP4 || m->format == URB_FMT_MXFP8) {
        size_t chunks = div_ceil(batch, 12), base = batch / chunks, larger = batch % chunks, tok = 0;
        for (size_t c = 0; c < chunks; ++c) {
            size_t b = base + (c < larger ? 1 : 0);
            bool checks = m->format == URB_FMT_MXFP8 ||
                          (b >= 2 && b <= 12 && m->group_size >= 8 && m->group_size % 2 == 0);
            if (checks && !all_finite(y + tok * count, b * count))
                return set_error(ctx, URB_ERR_NONFINITE, "batched matvec produced a non-finite output");
            tok += b;
        }
    }
    return URB_OK;
}

int urb_matmul_rows(urb_ctx *ctx, const urb_mat *m, const float *x, size_t batch, size_t x_len,
                    float *y) {
    if (!m) return URB_ERR_INVALID_ARGUMENT;
    return matmul_common(ctx, m, 0, m->rows, x, batch, x_len, y);
}

int urb_matmul_row_range(urb_ctx *ctx, const urb_mat *m, size_t start, size_t count,
                         const float *x, size_t batch, size_t x_len, float *y) {
    return matmul_common(ctx, m, start, count, x, batch, x_len, y);
}

int urb_matmul_rows_fp32_accum(urb_ctx *ctx, const urb_mat *m, const float *x, size_t batch,
                               size_t x_len, float *y) {
    if (!m) return URB_ERR_INVALID_ARGUMENT;
    int rc = matmul_common(ctx, m, 0, m->rows, x, batch, x_len, y);
    if (rc) return rc;
    // The FP32-accumulation entry points reject non-finite outputs (mxfp.rs:1658-1723); the INT
    // formats take plain matvec there (weight.rs:213-220), which does not check outputs.
    if (!is_int_format(m->format) && !all_finite(y, batch * m->rows))
        return set_error(ctx, URB_ERR_NONFINITE, "fp32-accumulated product is non-finite");
    return URB_OK;
}

int urb_matmul_rows_device(urb_ctx *ctx, const urb_mat *m, const float *d_x, size_t batch,
                           float *d_y, int32_t *d_status) {
    if (!ctx || !m || !d_x || !d_y) return URB_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    cudaSetDevice(ctx->device);
    if (batch == 0) return set_error(ctx, URB_ERR_SHAPE, "batch must be non-zero");
    return device_product(ctx, m, 0, m->rows, d_x, batch, d_y, d_status, ctx->stream);
}

int urb_profile_enable(urb_ctx *ctx, int on) {
    if (!ctx) return URB_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    ctx->prof = on != 0;
    return URB_OK;
}

int urb_profile_read(urb_ctx *ctx, int kind, double *total_ms, int64_t *launches) {
    if (!ctx || kind < 0 || kind >= URB_K_COUNT) return URB_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    cudaSetDevice(ctx->device);
    prof_drain(ctx);
    if (total_ms) *total_ms = ctx->prof_ms[kind];
    if (launches) *launches = ctx->prof_n[kind];
    return URB_OK;
}

int urb_profile_reset(urb_ctx *ctx) {
    if (!ctx) return URB_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    cudaSetDevice(ctx->device);
    prof_drain(ctx);
    for (int k = 0; k < URB_K_COUNT; ++k) { ctx->prof_ms[k] = 0; ctx->prof_n[k] = 0; }
    return URB_OK;
}

int urb_status_read(urb_ctx *ctx, const int32_t *d_status, int32_t *out) {
    if (!ctx || !d_status || !out) return URB_ERR_INVALID_ARGUMENT;
    URB_CUDA(ctx, cudaMemcpyAsync(out, d_status, 4, cudaMemcpyDeviceToHost, ctx->stream));
    URB_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    return URB_OK;
}

// ---- routing -------------------------------------------------------------------------------

static int check_noaux_geometry(urb_ctx *ctx, size_t experts, const urb_moe_geometry *g) {
    // routing.rs:63-99, in the reference's order (after the finiteness checks).
    if (!std::isfinite(g->routed_scaling_factor)) return set_error(ctx, URB_ERR_NONFINITE, "routed_scaling_factor is not finite");
    if (g->routed_scaling_factor <= 0.0f) return set_error(ctx, URB_ERR_INVALID_GEOMETRY, "routed_scaling_factor must be positive");
    if (g->n_group == 0 || experts % g->n_group != 0) return set_error(ctx, URB_ERR_INVALID_GEOMETRY, "experts cannot be divided into equal groups");
    if (g->top_k == 0 || g->top_k > experts) return set_error(ctx, URB_ERR_INVALID_GEOMETRY, "top_k outside 1..=experts");
    if (g->topk_group == 0 || g->topk_group > g->n_group) return set_error(ctx, URB_ERR_INVALID_GEOMETRY, "topk_group outside 1..=n_group");
    if (experts / g->n_group < 2) return set_error(ctx, URB_ERR_INVALID_GEOMETRY, "noaux_tc needs two experts per group");
    return URB_OK;
}

int urb_route_noaux_tc(urb_ctx *ctx, const float *logits, const float *bias, size_t tokens,
                       size_t experts, const urb_moe_geometry *g, int32_t *out_expert,
                       float *out_weight, float *out_score) {
    if (!ctx || !logits || !bias || !g || !out_expert || !out_weight) return URB_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    cudaSetDevice(ctx->device);
    if (experts == 0) return set_error(ctx, URB_ERR_INVALID_GEOMETRY, "no experts");
    if (!all_finite(logits, tokens * experts) || !all_finite(bias, experts))
        return set_error(ctx, URB_ERR_NONFINITE, "router logits or bias contain NaN/infinity");
    int rc = check_noaux_geometry(ctx, experts, g);
    if (rc) return rc;
    if (tokens == 0) return URB_OK;
    cudaStream_t st = ctx->stream;
    size_t K = g->top_k;
    size_t need = tokens * experts * 4 + experts * 4 + tokens * K * 12 + 4096;
    uint8_t *ws = static_cast<uint8_t *>(workspace(ctx, need, &rc));
    if (!ws) return rc;
    Carve cv{ws};
    float *d_l = cv.take<float>(tokens * experts);
    float *d_b = cv.take<float>(experts);
    int32_t *d_e = cv.take<int32_t>(tokens * K);
    float *d_w = cv.take<float>(tokens * K);
    float *d_s = cv.take<float>(tokens * K);
    URB_CUDA(ctx, cudaMemsetAsync(ctx->d_status, 0, 4, st));
    URB_CUDA(ctx, cudaMemcpyAsync(d_l, logits, tokens * experts * 4, cudaMemcpyDefault, st));
    URB_CUDA(ctx, cudaMemcpyAsync(d_b, bias, experts * 4, cudaMemcpyDefault, st));
    rc = launch_route_noaux(ctx, d_l, d_b, int(tokens), int(experts), *g, d_e, d_w, d_s,
                            ctx->d_status, st);
    if (rc) return rc;
    int32_t status = 0;
    URB_CUDA(ctx, cudaMemcpyAsync(out_expert, d_e, tokens * K * 4, cudaMemcpyDefault, st));
    URB_CUDA(ctx, cudaMemcpyAsync(out_weight, d_w, tokens * K * 4, cudaMemcpyDefault, st));
    if (out_score) URB_CUDA(ctx, cudaMemcpyAsync(out_score, d_s, tokens * K * 4, cudaMemcpyDefault, st));
    URB_CUDA(ctx, cudaMemcpyAsync(&status, ctx->d_status, 4, cudaMemcpyDeviceToHost, st));
    URB_CUDA(ctx, cudaStreamSynchronize(st));
    if (status) return set_error(ctx, status, "route_noaux_tc rejected the logits");
    return URB_OK;
}

int urb_route_sqrt_softplus(urb_ctx *ctx, const float *logits, const float *bias, size_t tokens,
                            size_t experts, const int32_t *hash_experts, uint32_t top_k,
                            float routed_scaling_factor, int32_t *out_expert, float *out_weight,
                            float *out_score) {
    if (!ctx || !logits || !out_expert || !out_weight) return URB_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    cudaSetDevice(ctx->device);
    // deepseek_v4/math.rs:458-480: geometry, scale, finiteness, hash range.
    if (experts == 0 || top_k == 0 || top_k > experts)
        return set_error(ctx, URB_ERR_SHAPE, "router logits/bias/hash/top-k geometry is inconsistent");
    if (!std::isfinite(routed_scaling_factor) || routed_scaling_factor <= 0.0f)
        return set_error(ctx, URB_ERR_INVALID_ARGUMENT, "routed_scaling_factor must be finite and positive");
    if (!all_finite(logits, tokens * experts) || (bias && !all_finite(bias, experts)))
        return set_error(ctx, URB_ERR_NONFINITE, "router logits or bias contain NaN/infinity");
    if (hash_experts)
        for (size_t i = 0; i < tokens * top_k; ++i)
            if (hash_experts[i] < 0 || size_t(hash_experts[i]) >= experts)
                return set_error(ctx, URB_ERR_INVALID_ARGUMENT, "hash expert IDs must be in range");
    if (tokens == 0) return URB_OK;
    cudaStream_t st = ctx->stream;
    const size_t K = top_k;
    int rc;
    size_t need = tokens * experts * 4 + experts * 4 + tokens * K * 16 + 4096;
    uint8_t *ws = static_cast<uint8_t *>(workspace(ctx, need, &rc));
    if (!ws) return rc;
    Carve cv{ws};
    float *d_l = cv.take<float>(tokens * experts);
    float *d_b = cv.take<float>(experts);
    int32_t *d_h = cv.take<int32_t>(tokens * K);
    int32_t *d_e = cv.take<int32_t>(tokens * K);
    float *d_w = cv.take<float>(tokens * K);
    float *d_s = cv.take<float>(tokens * K);
    URB_CUDA(ctx, cudaMemsetAsync(ctx->d_status, 0, 4, st));
    URB_CUDA(ctx, cudaMemcpyAsync(d_l, logits, tokens * experts * 4, cudaMemcpyDefault, st));
    if (bias) URB_CUDA(ctx, cudaMemcpyAsync(d_b, bias, experts * 4, cudaMemcpyDefault, st));
    if (hash_experts) URB_CUDA(ctx, cudaMemcpyAsync(d_h, hash_experts, tokens * K * 4, cudaMemcpyDefault, st));
    rc = launch_route_sqrt_softplus(ctx, d_l, bias ? d_b : nullptr, hash_experts ? d_h : nullptr,
                                    int(tokens), int(experts), int(K), routed_scaling_factor, d_e,
                                    d_w, d_s, ctx->d_status, st);
    if (rc) return rc;
    int32_t status = 0;
    URB_CUDA(ctx, cudaMemcpyAsync(out_expert, d_e, tokens * K * 4, cudaMemcpyDefault, st));
    URB_CUDA(ctx, cudaMemcpyAsync(out_weight, d_w, tokens * K * 4, cudaMemcpyDefault, st));
    if (out_score) URB_CUDA(ctx, cudaMemcpyAsync(out_score, d_s, tokens * K * 4, cudaMemcpyDefault, st));
    URB_CUDA(ctx, cudaMemcpyAsync(&status, ctx->d_status, 4, cudaMemcpyDeviceToHost, st));
    URB_CUDA(ctx, cudaStreamSynchronize(st));
    if (status) return set_error(ctx, status, "route_sqrt_softplus rejected the logits");
    return URB_OK;
}

int urb_route_softmax_top_k(urb_ctx *ctx, const float *logits, size_t tokens, size_t experts,
                            uint32_t top_k, int32_t *out_expert, float *out_weight) {
    if (!ctx || !logits || !out_expert || !out_weight) return URB_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    cudaSetDevice(ctx->device);
    // qwen3_8/moe.rs:95-106.
    if (experts == 0 || top_k == 0 || top_k > experts)
        return set_error(ctx, URB_ERR_INVALID_GEOMETRY, "top_k outside 1..=experts");
    if (!all_finite(logits, tokens * experts))
        return set_error(ctx, URB_ERR_NONFINITE, "router logits contain NaN/infinity");
    if (tokens == 0) return URB_OK;
    cudaStream_t st = ctx->stream;
    int rc;
    size_t need = tokens * experts * 4 + tokens * top_k * 8 + 4096;
    uint8_t *ws = static_cast<uint8_t *>(workspace(ctx, need, &rc));
    if (!ws) return rc;
    Carve cv{ws};
    float *d_l = cv.take<float>(tokens * experts);
    int32_t *d_e = cv.take<int32_t>(tokens * top_k);
    float *d_w = cv.take<float>(tokens * top_k);
    URB_CUDA(ctx, cudaMemsetAsync(ctx->d_status, 0, 4, st));
    URB_CUDA(ctx, cudaMemcpyAsync(d_l, logits, tokens * experts * 4, cudaMemcpyDefault, st));
    rc = launch_route_softmax(ctx, d_l, int(tokens), int(experts), int(top_k), d_e, d_w,
                              ctx->d_status, st);
    if (rc) return rc;
    int32_t status = 0;
    URB_CUDA(ctx, cudaMemcpyAsync(out_expert, d_e, tokens * top_k * 4, cudaMemcpyDefault, st));
    URB_CUDA(ctx, cudaMemcpyAsync(out_weight, d_w, tokens * top_k * 4, cudaMemcpyDefault, st));
    URB_CUDA(ctx, cudaMemcpyAsync(&status, ctx->d_status, 4, cudaMemcpyDeviceToHost, st));
    URB_CUDA(ctx, cudaStreamSynchronize(st));
    if (status) return set_error(ctx, status, "route_softmax_top_k rejected the logits");
    return URB_OK;
}

int urb_group_routes(urb_ctx *ctx, const int32_t *expert_ids, size_t tokens, uint32_t top_k,
                     size_t experts, int32_t *counts, int32_t *offsets, int32_t *perm_token,
                     int32_t *perm_slot) {
    if (!ctx || !expert_ids || !counts || !offsets || !perm_token || !perm_slot)
        return URB_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    cudaSetDevice(ctx->device);
    if (experts == 0 || top_k == 0) return set_error(ctx, URB_ERR_SHAPE, "empty grouping geometry");
    cudaStream_t st = ctx->stream;
    size_t TK = tokens * top_k;
    int rc;
    uint8_t *ws = static_cast<uint8_t *>(workspace(ctx, TK * 16 + experts * 8 + 8192, &rc));
    if (!ws) return rc;
    Carve cv{ws};
    int32_t *d_ids = cv.take<int32_t>(TK + 1);
    int32_t *d_cnt = cv.take<int32_t>(experts);
    int32_t *d_off = cv.take<int32_t>(experts + 1);
    int32_t *d_pt = cv.take<int32_t>(TK + 1);
    int32_t *d_ps = cv.take<int32_t>(TK + 1);
    int32_t *d_inv = cv.take<int32_t>(TK + 1);
    URB_CUDA(ctx, cudaMemsetAsync(ctx->d_status, 0, 4, st));
    if (TK) URB_CUDA(ctx, cudaMemcpyAsync(d_ids, expert_ids, TK * 4, cudaMemcpyDefault, st));
    PermArgs p{};
    p.ids = d_ids;
    p.tokens = int(tokens);
    p.top_k = int(top_k);
    p.experts = int(experts);
    p.cap = 1;
    p.counts = d_cnt;
    p.offsets = d_off;
    p.perm_token = d_pt;
    p.perm_slot = d_ps;
    p.inv = d_inv;
    p.status = ctx->d_status;
    rc = launch_permute(ctx, p, st);
    if (rc) return rc;
    int32_t status = 0;
    URB_CUDA(ctx, cudaMemcpyAsync(counts, d_cnt, experts * 4, cudaMemcpyDefault, st));
    URB_CUDA(ctx, cudaMemcpyAsync(offsets, d_off, (experts + 1) * 4, cudaMemcpyDefault, st));
    if (TK) {
        URB_CUDA(ctx, cudaMemcpyAsync(perm_token, d_pt, TK * 4, cudaMemcpyDefault, st));
        URB_CUDA(ctx, cudaMemcpyAsync(perm_slot, d_ps, TK * 4, cudaMemcpyDefault, st));
    }
    URB_CUDA(ctx, cudaMemcpyAsync(&status, ctx->d_status, 4, cudaMemcpyDeviceToHost, st));
    URB_CUDA(ctx, cudaStreamSynchronize(st));
    if (status) return set_error(ctx, status, "expert id out of range");
    return URB_OK;
}

}  // extern "C"
