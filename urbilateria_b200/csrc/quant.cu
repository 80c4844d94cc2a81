// quant.cu — Int8Matrix / Int4Matrix (src/math/quant.rs), the weight formats of GLM's converted
// checkpoints, on the device: the row products behind WeightMatrix::{matvec_rows, matmul_rows,
// matmul_row_range} (src/model/weight.rs:92-153, 305-320) and Int4Matrix::quantize_grouped.
//
// Products.  The reference sums exact f64 products in column order: INT8
// `sum(f64(i8) * f64(x))` from -0.0, times f64(row scale), rounded to f32 (quant.rs:448-499);
// INT4 `sum(f64(f32((code - 8) * scale)) * f64(x))` from +0.0 (quant.rs:304-318).  One dependent
// f64 chain per row would leave the GPU latency-bound, so a warp takes a row: its lanes stream
// the row's 16-byte chunks (coalesced, the packed payload read once per token block), keep the
// exact products in f64 chains of their own, and the chains meet in a fixed xor tree.  Products
// are exact and only the f64 rounding order differs from the reference, so results agree to
// the f64 summation error (far below one f32 ulp except where the row sum cancels), and are
// deterministic.  A warp holds up to 8 tokens so the weights are read once per 8 tokens.
//
// Quantiser.  quant.rs:46-90: per (row, group) scale = max(max|v| / 7, 1e-8) in f32, codes
// round_ties_even(v / scale) clamped to [-8, 7] + 8, low nibble first, 0x88 padding.
#include "urb_internal.cuh"

namespace urb {
namespace {

struct IntArgs {
    const uint8_t *values;  // INT8: [rows, cols] two's-complement bytes; INT4: [rows, row_bytes]
    const float *scales;    // INT8: [rows]; INT4: [rows, groups]
    int cols, group, groups;
    size_t row_bytes;
};

__device__ __forceinline__ float4 ld_x4(const float *p) { return __ldg(reinterpret_cast<const float4 *>(p)); }

__device__ __forceinline__ bool finite4(float4 v) {
    return isfinite(v.x) && isfinite(v.y) && isfinite(v.z) && isfinite(v.w);
}

// acc[t] += w * x[t] for 4 consecutive columns (weights already widened, exact products).
template <int T>
__device__ __forceinline__ void acc4(double (&acc)[T], const double (&w)[4], const float *x, size_t xs,
                                     int nt, bool &bad) {
#pragma unroll
    for (int t = 0; t < T; ++t) {
        if (t < nt) {
            const float4 v = ld_x4(x + t * xs);
            bad |= !finite4(v);
            acc[t] = fma(w[0], double(v.x), acc[t]);
            acc[t] = fma(w[1], double(v.y), acc[t]);
            acc[t] = fma(w[2], double(v.z), acc[t]);
            acc[t] = fma(w[3], double(v.w), acc[t]);
        }
    }
}

// Warp per (row, block of T tokens).  VEC: 16-byte row chunks (row_bytes % 16 == 0 and
// cols % 4 == 0, so every chunk column is in range and x rows are 16-byte aligned); otherwise
// lanes take single bytes.  GROUPED (INT4): a 32-column chunk lies inside one scale group.
template <int FMT, int T, bool VEC, bool GROUPED>
__global__ void __launch_bounds__(256) k_int_rows(IntArgs a, size_t start, size_t count,
                                                  const float *x, int batch, float *y,
                                                  int32_t *status) {
    const size_t wid = (blockIdx.x * size_t(blockDim.x) + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const size_t ntb = (size_t(batch) + T - 1) / T;
    if (wid >= count * ntb) return;
    const size_t i = wid % count, tb = wid / count;  // consecutive warps take consecutive rows
    const size_t r = start + i;
    const int t0 = int(tb) * T, nt = min(T, batch - t0);
    const uint8_t *row = a.values + r * a.row_bytes;
    const float *xt = x + size_t(t0) * a.cols;
    const size_t xs = size_t(a.cols);
    double acc[T];
#pragma unroll
    for (int t = 0; t < T; ++t) acc[t] = FMT == URB_FMT_INT8 ? -0.0 : 0.0;
    bool bad = false;
    if (VEC) {
        const int chunks = int(a.row_bytes / 16);
#pragma unroll 2
        for (int j = lane; j < chunks; j += 32) {
            const uint4 v = __ldg(reinterpret_cast<const uint4 *>(row) + j);
            const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
            if (FMT == URB_FMT_INT8) {
                const int c0 = j * 16;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    double w[4];
#pragma unroll
                    for (int k = 0; k < 4; ++k) w[k] = double(int8_t((wd[q] >> (8 * k)) & 0xffu));
                    acc4<T>(acc, w, xt + c0 + 4 * q, xs, nt, bad);
                }
            } else {
                const int c0 = j * 32;
                const float *srow = a.scales + r * a.groups;
                const float sc = GROUPED ? __ldg(srow + c0 / a.group) : 0.0f;
#pragma unroll
                for (int q = 0; q < 8; ++q) {  // 4 columns (one half word) at a time
                    double w[4];
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const int c = c0 + 4 * q + k;
                        const uint32_t code = (wd[q >> 1] >> (4 * (4 * (q & 1) + k))) & 15u;
                        const float s = GROUPED ? sc : __ldg(srow + c / a.group);
                        w[k] = double(__fmul_rn(float(int(code) - 8), s));
                    }
                    acc4<T>(acc, w, xt + c0 + 4 * q, xs, nt, bad);
                }
            }
        }
    } else {
        for (size_t b = lane; b < a.row_bytes; b += 32) {
            const uint8_t byte = __ldg(row + b);
            const int ncol = FMT == URB_FMT_INT8 ? 1 : 2;
#pragma unroll
            for (int h = 0; h < ncol; ++h) {
                const int c = FMT == URB_FMT_INT8 ? int(b) : int(2 * b) + h;
                if (c >= a.cols) break;
                double w;
                if (FMT == URB_FMT_INT8) {
                    w = double(int8_t(byte));
                } else {
                    const uint32_t code = h ? byte >> 4 : byte & 15u;
                    w = double(__fmul_rn(float(int(code) - 8), __ldg(a.scales + r * a.groups + c / a.group)));
                }
#pragma unroll
                for (int t = 0; t < T; ++t) {
                    if (t < nt) {
                        const float xv = __ldg(xt + t * xs + c);
                        bad |= !isfinite(xv);
                        acc[t] = fma(w, double(xv), acc[t]);
                    }
                }
            }
        }
    }
    // Each input element is read by the first row's warp of every token block: report once.
    if (status && i == 0 && __any_sync(0xffffffffu, bad) && lane == 0)
        atomicCAS(status, 0, int32_t(URB_ERR_NONFINITE));
#pragma unroll
    for (int t = 0; t < T; ++t)
        for (int o = 16; o > 0; o >>= 1) acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], o);
    if (lane == 0) {
        const double rs = FMT == URB_FMT_INT8 ? double(__ldg(a.scales + r)) : 1.0;
#pragma unroll
        for (int t = 0; t < T; ++t)
            if (t < nt)
                y[size_t(t0 + t) * count + i] =
                    FMT == URB_FMT_INT8 ? float(__dmul_rn(acc[t], rs)) : float(acc[t]);
    }
}

template <int FMT, int T>
int launch_int_t(const IntArgs &a, size_t start, size_t count, const float *d_x, int batch,
                 float *d_y, int32_t *d_status, cudaStream_t st) {
    const bool vec = a.row_bytes % 16 == 0 && a.cols % 4 == 0 &&
                     (reinterpret_cast<uintptr_t>(d_x) & 15) == 0;
    const bool grouped = FMT == URB_FMT_INT4 && a.group % 32 == 0;
    const size_t warps = count * ((size_t(batch) + T - 1) / T);
    const unsigned blocks = unsigned((warps + 7) / 8);
    if (vec && grouped)
        k_int_rows<FMT, T, true, true><<<blocks, 256, 0, st>>>(a, start, count, d_x, batch, d_y, d_status);
    else if (vec)
        k_int_rows<FMT, T, true, false><<<blocks, 256, 0, st>>>(a, start, count, d_x, batch, d_y, d_status);
    else
        k_int_rows<FMT, T, false, false><<<blocks, 256, 0, st>>>(a, start, count, d_x, batch, d_y, d_status);
    return cudaGetLastError() == cudaSuccess ? URB_OK : URB_ERR_CUDA;
}

template <int FMT>
int launch_int_fmt(const IntArgs &a, size_t start, size_t count, const float *d_x, int batch,
                   float *d_y, int32_t *d_status, cudaStream_t st) {
    if (batch <= 1) return launch_int_t<FMT, 1>(a, start, count, d_x, batch, d_y, d_status, st);
    if (batch <= 2) return launch_int_t<FMT, 2>(a, start, count, d_x, batch, d_y, d_status, st);
    if (batch <= 4) return launch_int_t<FMT, 4>(a, start, count, d_x, batch, d_y, d_status, st);
    return launch_int_t<FMT, 8>(a, start, count, d_x, batch, d_y, d_status, st);
}

// One warp per (row, group): the group's largest magnitude -> its scale; flags non-finite
// values (quant.rs:53-55, 59-68).
__global__ void k_int4_scales(const float *v, size_t rows, int cols, int group, int groups,
                              float *scales, int32_t *flag) {
    const size_t wid = (blockIdx.x * size_t(blockDim.x) + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (wid >= rows * size_t(groups)) return;
    const size_t r = wid / groups;
    const int g = int(wid % groups);
    const int c0 = g * group, c1 = min(cols, c0 + group);
    float m = 0.0f;
    bool bad = false;
    for (int c = c0 + lane; c < c1; c += 32) {
        const float x = v[r * cols + c];
        bad |= !isfinite(x);
        m = fmaxf(m, fabsf(x));
    }
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (__any_sync(0xffffffffu, bad) && lane == 0) atomicOr(flag, 1);
    if (lane == 0) scales[wid] = fmaxf(__fdiv_rn(m, 7.0f), 1e-8f);
}

// quant.rs:600-617 round_ties_even of the quotient, then clamp (quant.rs:71-72).
__device__ __forceinline__ uint32_t int4_code(float value, float scale) {
    const float q = __fdiv_rn(value, scale);
    const float fl = floorf(q);
    const float fraction = __fsub_rn(q, fl);
    const int lower = int(fl);
    int k = fraction < 0.5f ? lower : (fraction > 0.5f ? lower + 1 : (lower % 2 == 0 ? lower : lower + 1));
    k = min(max(k, -8), 7);
    return uint32_t(k + 8);
}

// One thread per packed byte (two columns; an odd tail keeps the 0x8 padding nibble).
__global__ void k_int4_pack(const float *v, size_t rows, int cols, int group, int groups,
                            size_t row_bytes, const float *scales, uint8_t *packed) {
    const size_t idx = blockIdx.x * size_t(blockDim.x) + threadIdx.x;
    if (idx >= rows * row_bytes) return;
    const size_t r = idx / row_bytes;
    const int c = int(idx % row_bytes) * 2;
    const float *sr = scales + r * groups;
    const uint32_t lo = int4_code(v[r * cols + c], sr[c / group]);
    const uint32_t hi = c + 1 < cols ? int4_code(v[r * cols + c + 1], sr[(c + 1) / group]) : 8u;
    packed[idx] = uint8_t(lo | (hi << 4));
}

}  // namespace

int launch_int_matmul(Ctx *ctx, const Mat *m, size_t start, size_t count, const float *d_x,
                      size_t batch, float *d_y, int32_t *d_status, cudaStream_t st) {
    if (count == 0 || batch == 0) return URB_OK;
    IntArgs a{};
    a.values = static_cast<const uint8_t *>(m->raw_values);
    a.scales = reinterpret_cast<const float *>(m->raw_scales);
    a.cols = int(m->cols);
    a.group = int(m->format == URB_FMT_INT4 ? m->group_size : m->cols);
    a.groups = int((m->cols + a.group - 1) / a.group);
    a.row_bytes = m->format == URB_FMT_INT4 ? (m->cols + 1) / 2 : m->cols;
    const int rc = m->format == URB_FMT_INT8
                       ? launch_int_fmt<URB_FMT_INT8>(a, start, count, d_x, int(batch), d_y, d_status, st)
                       : launch_int_fmt<URB_FMT_INT4>(a, start, count, d_x, int(batch), d_y, d_status, st);
    if (rc) return cuda_fail(ctx, cudaGetLastError(), "int matvec");
    return URB_OK;
}

// Int4Matrix::quantize_grouped on device buffers: d_values [rows, cols] -> d_packed, d_scales.
// Returns URB_ERR_NONFINITE (after a stream synchronisation) when a value is not finite.
int int4_quantize_device(Ctx *ctx, size_t rows, size_t cols, size_t group, const float *d_values,
                         uint8_t *d_packed, float *d_scales, int32_t *d_flag, cudaStream_t st) {
    const int groups = int((cols + group - 1) / group);
    const size_t row_bytes = (cols + 1) / 2;
    URB_CUDA(ctx, cudaMemsetAsync(d_flag, 0, sizeof(int32_t), st));
    const size_t warps = rows * size_t(groups);
    k_int4_scales<<<unsigned((warps + 7) / 8), 256, 0, st>>>(d_values, rows, int(cols), int(group),
                                                             groups, d_scales, d_flag);
    URB_CUDA(ctx, cudaGetLastError());
    int32_t flag = 0;
    URB_CUDA(ctx, cudaMemcpyAsync(&flag, d_flag, sizeof(flag), cudaMemcpyDeviceToHost, st));
    URB_CUDA(ctx, cudaStreamSynchronize(st));
    if (flag) return set_error(ctx, URB_ERR_NONFINITE, "INT4 source contains NaN or infinity");
    const size_t n = rows * row_bytes;
    k_int4_pack<<<unsigned((n + 255) / 256), 256, 0, st>>>(d_values, rows, int(cols), int(group), groups,
                                                          row_bytes, d_scales, d_packed);
    URB_CUDA(ctx, cudaGetLastError());
    return URB_OK;
}

}  // namespace urb
