// generic.cu — CUDA-core kernels that need no tiled layout: the fallback product for matrices
// the tiled path cannot hold exactly (F32 weights, MX group sizes other than 32, rows whose
// scale range exceeds the f16 window) and the per-row activation pre-pass.
#include "urb_internal.cuh"

namespace urb {
namespace {

__device__ __forceinline__ float e8m0_dev(uint8_t code) {
    uint32_t bits = uint32_t(code) << 23;
    return __uint_as_float(bits == 0 ? 0x00400000u : bits);
}

// src/math/mxfp.rs:60-71.
__device__ __forceinline__ float e4m3_dev(uint8_t v) {
    float sign = (v & 0x80) ? -1.0f : 1.0f;
    int e = (v >> 3) & 0x0f, m = v & 7;
    if (e == 0) return sign * float(m) * 0.001953125f;  // 2^-9
    return sign * (1.0f + float(m) * 0.125f) * ldexpf(1.0f, e - 7);
}

__device__ __forceinline__ float e2m1_dev(uint8_t c) {
    const float mag[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
    float v = mag[c & 7];
    return (c & 8) && (c & 7) ? -v : v;
}

struct RawMat {
    int format;
    size_t rows, cols, group, block_rows, block_cols;
    const void *values;
    const uint8_t *scales;
};

__device__ __forceinline__ float weight_at(const RawMat &m, size_t r, size_t c) {
    switch (m.format) {
    case URB_FMT_F32:
        return static_cast<const float *>(m.values)[r * m.cols + c];
    case URB_FMT_BF16:
        return __uint_as_float(uint32_t(static_cast<const uint16_t *>(m.values)[r * m.cols + c]) << 16);
    case URB_FMT_MXFP8: {
        size_t sc = (m.cols + m.block_cols - 1) / m.block_cols;
        float s = e8m0_dev(m.scales[(r / m.block_rows) * sc + c / m.block_cols]);
        return e4m3_dev(static_cast<const uint8_t *>(m.values)[r * m.cols + c]) * s;
    }
    default: {
        size_t rb = (m.cols + 1) / 2, groups = (m.cols + m.group - 1) / m.group;
        uint8_t byte = static_cast<const uint8_t *>(m.values)[r * rb + c / 2];
        uint8_t code = (c & 1) ? (byte >> 4) : (byte & 15);
        return e2m1_dev(code) * e8m0_dev(m.scales[r * groups + c / m.group]);
    }
    }
}

// One warp per (output row, token): f64 accumulation of widened products, then f32.
__global__ void k_generic(RawMat m, size_t start, size_t count, const float *x, size_t batch,
                          float *y) {
    size_t wid = (blockIdx.x * size_t(blockDim.x) + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (wid >= count * batch) return;
    size_t t = wid / count, i = wid % count, r = start + i;
    const float *xt = x + t * m.cols;
    double acc = 0.0;
    for (size_t c = lane; c < m.cols; c += 32) acc += double(weight_at(m, r, c)) * double(xt[c]);
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) y[t * count + i] = float(acc);
}

// One block per row: shift = 14 - ilogb(max|v|) (0 for an all-zero row); flags non-finite;
// with lofree, checks that every shifted value is exact in one f16 (or bf16) column.
__global__ void k_row_shift(const float *src, int cols, int stride, int32_t *shift,
                            int32_t *status, int32_t *lofree, int bf16_check) {
    const float *p = src + size_t(blockIdx.x) * stride;
    float m = 0.0f;
    bool bad = false;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) {
        float v = p[c];
        bad |= !isfinite(v);
        m = fmaxf(m, fabsf(v));
    }
    __shared__ float red[32];
    __shared__ int badf, sh, inexact;
    if (threadIdx.x == 0) { badf = 0; inexact = 0; }
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    __syncthreads();
    if (bad) badf = 1;
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        float mm = 0.0f;
        for (int w = 0; w < int(blockDim.x >> 5); ++w) mm = fmaxf(mm, red[w]);
        sh = (mm > 0.0f && isfinite(mm)) ? 14 - ilogbf(mm) : 0;
        shift[blockIdx.x] = sh;
        if (badf && status) atomicCAS(status, 0, int32_t(URB_ERR_NONFINITE));
    }
    if (!lofree) return;
    __syncthreads();
    bool ok = true;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) {
        float v = ldexpf(p[c], sh);
        float r = bf16_check ? __bfloat162float(__float2bfloat16_rn(v)) : __half2float(__float2half_rn(v));
        ok &= (r == v);
    }
    if (!ok) inexact = 1;
    __syncthreads();
    if (threadIdx.x == 0 && inexact) atomicAnd(lofree, 0);
}

}  // namespace

int launch_generic_matmul(Ctx *ctx, const Mat *mt, size_t start, size_t count, const float *d_x,
                          size_t batch, float *d_y, cudaStream_t st) {
    RawMat m{mt->format, mt->rows, mt->cols, mt->group_size, mt->block_rows, mt->block_cols,
             mt->raw_values, mt->raw_scales};
    size_t warps = count * batch;
    if (warps == 0) return URB_OK;
    k_generic<<<unsigned((warps + 7) / 8), 256, 0, st>>>(m, start, count, d_x, batch, d_y);
    URB_CUDA(ctx, cudaGetLastError());
    return URB_OK;
}

int launch_row_shift(const float *d_src, int rows, int cols, int stride, int32_t *d_shift,
                     int32_t *d_status, cudaStream_t st, int32_t *d_lofree, int bf16_check) {
    if (rows <= 0) return URB_OK;
    k_row_shift<<<rows, 256, 0, st>>>(d_src, cols, stride, d_shift, d_status, d_lofree, bf16_check);
    // The launch error is left for the caller to read (cudaPeekAtLastError does not clear it).
    return cudaPeekAtLastError() == cudaSuccess ? URB_OK : URB_ERR_CUDA;
}

}  // namespace urb
