// transpose.cu — WeightMatrix::transpose_rows_matvec (src/model/weight.rs:332-343): y[cols] =
// W[start .. start + n]^T x[n], the product MLA absorption applies to MXFP8 projections
// (mxfp.rs:785-858) and the other formats provide alike (mxfp.rs:1782-1821 MXFP4,
// bf16.rs:430-475, matrix.rs:276-313).
//
// Every format sums each output column over the rows in order, in f64, from +0.0, the product
// f64(weight) * f64(x) being exact (a weight carries at most 24 significant bits and x 24), and
// rounds the sum to f32 once.  So a thread per column running the same ordered chain of f64
// FMAs is bit-exact against the reference.  Int4Matrix (quant.rs:236-283) is the same chain
// over its f32 weights (code - 8) * scale; Int8Matrix (quant.rs:512-553) adds, per row,
// (f64(x) * f64(row scale)) * f64(i8), a product that is rounded, so that chain multiplies and
// adds separately.  Weights are read from whichever copy the matrix
// keeps on the device: the row-major upload (F32, BF16, and MX layouts that are not tiled) or
// the block-scaled tensor-core tiles (MXFP4 with 32-column groups, MXFP8 with 32-column
// blocks), decoding one element at a time; consecutive threads read consecutive columns of
// one row, so each warp's loads stay within one 128-byte row segment.
#include "urb_internal.cuh"
#include "urb_tc.cuh"

namespace urb {
namespace {

__device__ __forceinline__ float tr_e8m0(uint32_t s) {
    return s ? __uint_as_float(s << 23) : __uint_as_float(1u << 22);
}

__device__ __forceinline__ float tr_e4m3(uint32_t code) {
    const uint32_t e = (code >> 3) & 0xfu, m = code & 7u;
    const float mag = e == 0 ? float(m) * 0.001953125f : __uint_as_float(((e + 120u) << 23) | (m << 20));
    return (code & 0x80u) ? -mag : mag;
}

__device__ __forceinline__ float tr_e2m1(uint32_t code) {
    const uint32_t m = code & 7u;
    const float mag = m < 2 ? 0.5f * float(m) : __uint_as_float(((((m >> 1) + 126u) << 23)) | ((m & 1u) << 22));
    return ((code & 8u) && m) ? -mag : mag;  // code 8 decodes to +0.0 (mxfp.rs:73-79)
}

struct TrArgs {
    int format;
    int rows, cols;
    int group, block_rows, block_cols;  // MX scale geometry of the row-major copy
    const void *values;                 // row-major copy (nullptr: tiles)
    const uint8_t *scales;
    const uint8_t *tiles;               // block-scaled tiles (tile (mt, ks) at ks * mts + mt)
    int mts;
    const float *fscales;               // INT8 [rows] / INT4 [rows, groups] f32 scales
};

// Weight (row, col) of the matrix, exactly as the reference decodes it (f32).
__device__ __forceinline__ float tr_weight(const TrArgs &a, int row, int col) {
    if (a.values) {
        const size_t i = size_t(row) * a.cols + col;
        switch (a.format) {
        case URB_FMT_F32: return static_cast<const float *>(a.values)[i];
        case URB_FMT_BF16: return __uint_as_float(uint32_t(static_cast<const uint16_t *>(a.values)[i]) << 16);
        case URB_FMT_MXFP8: {
            const int sc = (a.cols + a.block_cols - 1) / a.block_cols;
            return tr_e4m3(static_cast<const uint8_t *>(a.values)[i]) *
                   tr_e8m0(a.scales[size_t(row / a.block_rows) * sc + col / a.block_cols]);
        }
        case URB_FMT_INT8:  // quant.rs:430: f32(i8) * scale
            return __fmul_rn(float(static_cast<const int8_t *>(a.values)[i]), a.fscales[row]);
        default: {
            const int rb = (a.cols + 1) / 2, groups = (a.cols + a.group - 1) / a.group;
            const uint8_t byte = static_cast<const uint8_t *>(a.values)[size_t(row) * rb + col / 2];
            const uint32_t code = (col & 1) ? byte >> 4 : byte & 15;
            if (a.format == URB_FMT_INT4)  // quant.rs:343-350: (code - 8) * scale in f32
                return __fmul_rn(float(int(code) - 8), a.fscales[size_t(row) * groups + col / a.group]);
            return tr_e2m1(code) * tr_e8m0(a.scales[size_t(row) * groups + col / a.group]);
        }
        }
    }
    // Block-scaled tile layout: 128 rows x one stage (256 E2M1 / 128 E4M3 columns), 128-byte
    // rows in 16-byte chunks swizzled by row % 8, then the stage's E8M0 bytes per 32 columns.
    const bool fp4 = a.format == URB_FMT_MXFP4;
    const int sc = fp4 ? 256 : 128;
    const int mt = row >> 7, rr = row & 127, ks = col / sc, cs = col - ks * sc;
    const uint8_t *t = a.tiles + (size_t(ks) * a.mts + mt) * size_t(fp4 ? bs_tile_bytes(URB_FMT_MXFP4)
                                                                     : bs_tile_bytes(URB_FMT_MXFP8));
    const int b = fp4 ? cs >> 1 : cs;
    const uint8_t byte = t[(rr >> 3) * 1024 + (rr & 7) * 128 + ((((b >> 4) ^ (rr & 7))) << 4) + (b & 15)];
    const int kb = cs >> 5;
    const uint8_t s = t[16384 + 512 * (kb >> 2) + 16 * (rr & 31) + 4 * (rr >> 5) + (kb & 3)];
    return (fp4 ? tr_e2m1((cs & 1) ? byte >> 4 : byte & 15) : tr_e4m3(byte)) * tr_e8m0(s);
}

__global__ void k_transpose_rows(TrArgs a, int start, const float *x, int n, float *y) {
    const int col = blockIdx.x * blockDim.x + threadIdx.x;
    if (col >= a.cols) return;
    double sum = 0.0;
    if (a.format == URB_FMT_INT8) {
        const int8_t *v = static_cast<const int8_t *>(a.values);
        for (int i = 0; i < n; ++i) {
            const double scaled = __dmul_rn(double(__ldg(x + i)), double(a.fscales[start + i]));
            sum = __dadd_rn(sum, __dmul_rn(scaled, double(v[size_t(start + i) * a.cols + col])));
        }
    } else {
#pragma unroll 4
        for (int i = 0; i < n; ++i)
            sum = fma(double(__ldg(x + i)), double(tr_weight(a, start + i, col)), sum);
    }
    y[col] = float(sum);
}

// Thread per element: out[i, c] = weight (start + i, c).
__global__ void k_write_rows(TrArgs a, int start, int count, float *out) {
    const size_t idx = blockIdx.x * size_t(blockDim.x) + threadIdx.x;
    if (idx >= size_t(count) * a.cols) return;
    const int i = int(idx / a.cols), c = int(idx % a.cols);
    out[idx] = tr_weight(a, start + i, c);
}

// Kernel arguments for a matrix, or URB_ERR_UNSUPPORTED when no device copy can be read.
int tr_args(Ctx *ctx, const Mat *m, TrArgs &a) {
    a = TrArgs{};
    a.format = m->format;
    a.rows = int(m->rows);
    a.cols = int(m->cols);
    a.group = int(m->group_size ? m->group_size : 32);
    a.block_rows = int(m->block_rows ? m->block_rows : 1);
    a.block_cols = int(m->block_cols ? m->block_cols : 32);
    a.values = m->raw_values;
    a.scales = m->raw_scales;
    a.fscales = reinterpret_cast<const float *>(m->raw_scales);
    a.tiles = m->tc_tiles;
    a.mts = m->tc_mts;
    const bool mx = m->format == URB_FMT_MXFP4 || m->format == URB_FMT_MXFP8;
    if (!a.values && !(mx && a.tiles))
        return set_error(ctx, URB_ERR_UNSUPPORTED, "no device copy of the weights to read");
    if (a.values && (mx || is_int_format(m->format)) && !a.scales)
        return set_error(ctx, URB_ERR_UNSUPPORTED, "scales missing");
    return URB_OK;
}

}  // namespace
}  // namespace urb

using namespace urb;

extern "C" int urb_transpose_rows_matvec(urb_ctx *ctx, const urb_mat *m, size_t start,
                                         const float *x, size_t n, float *y) {
    if (!ctx || !m || !y || (n && !x)) return URB_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    cudaSetDevice(ctx->device);
    // Validation order of the reference: input finiteness, then the row range.
    for (size_t i = 0; i < n; ++i)
        if (!std::isfinite(x[i])) return set_error(ctx, URB_ERR_NONFINITE, "transpose input is not finite");
    if (start + n < start || start + n > m->rows)
        return set_error(ctx, URB_ERR_SHAPE, "transpose matvec row range is out of bounds");
    TrArgs a;
    if (int rc = tr_args(ctx, m, a)) return rc;
    const size_t C = m->cols;
    cudaStream_t st = ctx->stream;
    float *d = nullptr;
    URB_CUDA(ctx, cudaMallocAsync(&d, (n + C) * sizeof(float) + 16, st));
    float *d_x = d, *d_y = d + n;
    if (n) URB_CUDA(ctx, cudaMemcpyAsync(d_x, x, n * sizeof(float), cudaMemcpyDefault, st));
    prof_begin(ctx, URB_K_PRODUCT, st);
    k_transpose_rows<<<unsigned((C + 127) / 128), 128, 0, st>>>(a, int(start), d_x, int(n), d_y);
    prof_end(ctx, st);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaMemcpyAsync(y, d_y, C * sizeof(float), cudaMemcpyDefault, st);
    cudaFreeAsync(d, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "transpose matvec");
    if (m->format == URB_FMT_MXFP8)  // mxfp.rs:851-856: MXFP8 rejects non-finite outputs
        for (size_t c = 0; c < C; ++c)
            if (!std::isfinite(y[c])) return set_error(ctx, URB_ERR_NONFINITE, "transpose output is not finite");
    return URB_OK;
}

extern "C" int urb_mat_write_rows(urb_ctx *ctx, const urb_mat *m, size_t start, size_t count,
                                  float *out) {
    if (!ctx || !m || (count && !out)) return URB_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    cudaSetDevice(ctx->device);
    if (start + count < start || start + count > m->rows)
        return set_error(ctx, URB_ERR_SHAPE, "row is outside the matrix");
    if (count == 0) return URB_OK;
    TrArgs a;
    if (int rc = tr_args(ctx, m, a)) return rc;
    const size_t n = count * m->cols;
    cudaStream_t st = ctx->stream;
    float *d = nullptr;
    URB_CUDA(ctx, cudaMallocAsync(&d, n * sizeof(float), st));
    k_write_rows<<<unsigned((n + 255) / 256), 256, 0, st>>>(a, int(start), int(count), d);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaMemcpyAsync(out, d, n * sizeof(float), cudaMemcpyDefault, st);
    cudaFreeAsync(d, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "write rows");
    return URB_OK;
}
