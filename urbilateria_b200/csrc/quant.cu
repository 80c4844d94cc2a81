// quant.cu — Int8Matrix / Int4Matrix (src/math/quant.rs), the weight formats of GLM's converted
// checkpoints, on the device: the row products behind WeightMatrix::{matvec_rows, matmul_rows,
// matmul_row_range} (src/model/weight.rs:92-153, 305-320) and Int4Matrix::quantize_grouped.
//
// Products.  The reference sums exact f64 products in column order: INT8
// `sum(f64(i8) * f64(x))` from -0.0, times f64(row scale), rounded to f32 (quant.rs:448-499);
// INT4 `sum(f64(f32((code - 8) * scale)) * f64(x))` from +0.0 (quant.rs:304-318).  B200's FP64
// pipe sustains about 2e12 operations per second, so any scheme with an f64 operation per weight
// and token is compute-bound far below HBM speed.  The fast path therefore sums in integers:
// each token's activations become 38-bit fixed-point integers X = rint(x * 2^shift) (shift set
// per 32-column block by the block's largest magnitude) split into five byte limbs, and the integer weights meet the
// limbs in dp4a byte dot products, so sum(w * X) is exact in int64.  INT8 rows scale that sum by
// 2^-shift in f64 per chunk and by the row scale at the end (quant.rs:497); INT4 rows scale each
// 32-column group's exact sum by its group scale and 2^-shift in f64 and add, in f32, the rounding of the reference's f32 weights,
// (code - 8) * scale - f32((code - 8) * scale), an exact FMA residue, times x.  The only
// departures from the reference are x's rounding to the 2^-shift grid (at most 2^-38 of its
// block's largest magnitude per element) and f64 rounding in a different order; both sit far
// below one f32 ulp of a typical output.  Shapes without 16-byte rows (or INT4 groups that are
// not whole 32-column chunks) take a warp-per-row kernel of exact f64 products.
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

// ---- fixed-point activation limbs -------------------------------------------------------

constexpr int kLimbs = 5;

// Thread per 4 columns; the 8 threads of a 32-column block share its shift = 37 - ilogb(block
// max|x|) (0 for an all-zero block), so |X| <= 2^38 and the top limb X >> 32 lies in [-64, 64].
// limbs[t][k][c] = byte k of X = rint(x * 2^shift) for k < 4 (unsigned) and X >> 32 for k = 4
// (signed), zero past cols up to cols32; shift[t][c / 32].  Flags non-finite inputs.
__global__ void __launch_bounds__(256) k_x_limbs(const float *x, int cols, int cols32, int batch,
                                                 uint8_t *limbs, int32_t *shift, int32_t *status) {
    const size_t idx = blockIdx.x * size_t(blockDim.x) + threadIdx.x;
    const int per_tok = cols32 / 4;
    if (idx >= size_t(batch) * per_tok) return;  // whole 8-thread groups leave together
    const int t = int(idx / per_tok), c0 = int(idx % per_tok) * 4;
    const unsigned gmask = 0xffu << (threadIdx.x & 24);
    float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (c0 < cols) v = __ldg(reinterpret_cast<const float4 *>(x + size_t(t) * cols + c0));
    const float vs[4] = {v.x, v.y, v.z, v.w};
    bool bad = false;
    float m = 0.0f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        bad |= !isfinite(vs[e]);
        m = fmaxf(m, fabsf(vs[e]));
    }
    for (int o = 4; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(gmask, m, o));
    const int sh = (m > 0.0f && isfinite(m)) ? 37 - ilogbf(m) : 0;
    if ((threadIdx.x & 7) == 0) shift[size_t(t) * (cols32 / 32) + c0 / 32] = sh;
    if (bad && status) atomicCAS(status, 0, int32_t(URB_ERR_NONFINITE));
    uint32_t word[kLimbs] = {0, 0, 0, 0, 0};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const long long X = isfinite(vs[e]) ? __double2ll_rn(ldexp(double(vs[e]), sh)) : 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) word[k] |= uint32_t((X >> (8 * k)) & 0xff) << (8 * e);
        word[4] |= uint32_t((X >> 32) & 0xff) << (8 * e);
    }
    uint8_t *lt = limbs + size_t(t) * kLimbs * cols32 + c0;
#pragma unroll
    for (int k = 0; k < kLimbs; ++k) *reinterpret_cast<uint32_t *>(lt + size_t(k) * cols32) = word[k];
}

// 2^-sh as a double (sh within [-1022, 1022]).
__device__ __forceinline__ double pow2_neg(int sh) {
    return __longlong_as_double((long long)(1023 - sh) << 52);
}

__device__ __forceinline__ int dp4a_su(int a_signed, uint32_t b_unsigned, int c) {
    int d;
    asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a_signed), "r"(b_unsigned), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_uu(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_ss(int a, int b, int c) {
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Exact int64 value of sum_k 2^(8k) a[k].  An exact zero comes out as +0.0 where the
// reference's sum from -0.0 of products that are all -0.0 keeps -0.0 (numerically equal).
__device__ __forceinline__ long long limb_sum(const int (&a)[kLimbs]) {
    return (long long)a[0] + ((long long)a[1] << 8) + ((long long)a[2] << 16) +
           ((long long)a[3] << 24) + ((long long)a[4] << 32);
}

// Four INT4 codes (nibbles 4h .. 4h+3 of w) as four unsigned bytes.
__device__ __forceinline__ uint32_t nib4(uint32_t w, int h) {
    uint32_t t = (w >> (16 * h)) & 0xffffu;
    t = (t | (t << 8)) & 0x00ff00ffu;
    return (t | (t << 4)) & 0x0f0f0f0fu;
}

// CTA per (R rows, T tokens): its KS warps split the row's 16-byte chunks (INT8: 16 columns;
// INT4: 32 columns, one scale group) into KS slices, each lane taking every 32nd chunk of its
// warp's slice, U chunks per round of loads.  A chunk's exact integer sum, scaled by 2^-shift
// (and the INT4 group scale), enters an f64 accumulator; lanes and then warps are added in a
// fixed order.  Requires row_bytes % 16 == 0, cols % 4 == 0 and 16-byte aligned payloads.
template <int FMT, int R, int T, int KS, int U>
__global__ void __launch_bounds__(32 * KS) k_int_limbs(IntArgs a, size_t start, size_t count,
                                                       const uint8_t *limbs, int cols32,
                                                       const int32_t *shift, const float *x,
                                                       int batch, float *y) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const size_t nrg = (count + R - 1) / R;
    const size_t rg = blockIdx.x % nrg, tb = blockIdx.x / nrg;
    const int t0 = int(tb) * T, nt = min(T, batch - t0);
    size_t row[R];
#pragma unroll
    for (int r = 0; r < R; ++r) row[r] = start + min(rg * R + r, count - 1);
    constexpr int COLS = FMT == URB_FMT_INT8 ? 16 : 32;  // columns per 16-byte chunk
    const int chunks = int(a.row_bytes / 16);
    const int per = (chunks + KS - 1) / KS;
    const int j_begin = warp * per, j_end = min(chunks, j_begin + per);
    const int nsh = cols32 / 32;
    double acc[R][T];
    float corr[R][T];  // INT4: sum of (f32 weight - exact weight) * x
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int t = 0; t < T; ++t) { acc[r][t] = 0.0; corr[r][t] = 0.0f; }
    for (int j0 = j_begin + lane; j0 < j_end; j0 += 32 * U) {
        uint4 w[U][R];
#pragma unroll
        for (int u = 0; u < U; ++u)
            if (j0 + 32 * u < j_end)
#pragma unroll
                for (int r = 0; r < R; ++r)
                    w[u][r] = __ldg(reinterpret_cast<const uint4 *>(a.values + row[r] * a.row_bytes) + j0 + 32 * u);
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int j = j0 + 32 * u;
            if (j >= j_end) break;
            float sc[R];
            if (FMT == URB_FMT_INT4) {
#pragma unroll
                for (int r = 0; r < R; ++r) sc[r] = __ldg(a.scales + row[r] * a.groups + (j * COLS) / a.group);
            }
#pragma unroll
            for (int t = 0; t < T; ++t) {
                if (t >= nt) break;
                const uint8_t *lt = limbs + size_t(t0 + t) * kLimbs * cols32 + size_t(j) * COLS;
                const double p2 = pow2_neg(__ldg(shift + size_t(t0 + t) * nsh + (j * COLS) / 32));
                if (FMT == URB_FMT_INT8) {
                    uint4 L[kLimbs];
#pragma unroll
                    for (int k = 0; k < kLimbs; ++k) L[k] = __ldg(reinterpret_cast<const uint4 *>(lt + size_t(k) * cols32));
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        const uint32_t wq[4] = {w[u][r].x, w[u][r].y, w[u][r].z, w[u][r].w};
                        int d[kLimbs] = {0, 0, 0, 0, 0};
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
#pragma unroll
                            for (int k = 0; k < 4; ++k) d[k] = dp4a_su(int(wq[q]), (&L[k].x)[q], d[k]);
                            d[4] = dp4a_ss(int(wq[q]), int((&L[4].x)[q]), d[4]);
                        }
                        acc[r][t] = fma(double(limb_sum(d)), p2, acc[r][t]);
                    }
                } else {
                    uint4 L[kLimbs][2];
#pragma unroll
                    for (int k = 0; k < kLimbs; ++k)
#pragma unroll
                        for (int h = 0; h < 2; ++h)
                            L[k][h] = __ldg(reinterpret_cast<const uint4 *>(lt + size_t(k) * cols32) + h);
                    // Limb sums over the chunk: the codes carry +8, so sum (u - 8) X = sum u X - 8 sum X.
                    int ls[kLimbs] = {0, 0, 0, 0, 0};
#pragma unroll
                    for (int h = 0; h < 2; ++h)
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
#pragma unroll
                            for (int k = 0; k < 4; ++k) ls[k] = dp4a_uu(0x01010101u, (&L[k][h].x)[q], ls[k]);
                            ls[4] = dp4a_ss(int((&L[4][h].x)[q]), 0x01010101, ls[4]);
                        }
                    const float4 *xc = reinterpret_cast<const float4 *>(x + size_t(t0 + t) * a.cols + size_t(j) * COLS);
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        const uint32_t wq[4] = {w[u][r].x, w[u][r].y, w[u][r].z, w[u][r].w};
                        int d[kLimbs] = {0, 0, 0, 0, 0};
                        float cr = 0.0f;
#pragma unroll
                        for (int g = 0; g < 8; ++g) {  // columns 4g .. 4g+3: nibbles of word g >> 1
                            const uint32_t u4 = nib4(wq[g >> 1], g & 1);
                            const int h = g >> 2, q = g & 3;
#pragma unroll
                            for (int k = 0; k < 4; ++k) d[k] = dp4a_uu((&L[k][h].x)[q], u4, d[k]);
                            d[4] = dp4a_su(int((&L[4][h].x)[q]), u4, d[4]);
                            const float4 xv = __ldg(xc + g);
                            const float xs[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                // code - 8 exactly: (2^23 + code) - (2^23 + 8).
                                const float kf = __fsub_rn(__uint_as_float(0x4b000000u | ((u4 >> (8 * e)) & 0xffu)), 8388616.0f);
                                const float w32 = __fmul_rn(kf, sc[r]);
                                const float res = fmaf(kf, sc[r], -w32);  // exact: k*s - f32(k*s)
                                cr = fmaf(-res, xs[e], cr);
                            }
                        }
#pragma unroll
                        for (int k = 0; k < kLimbs; ++k) d[k] -= 8 * ls[k];
                        acc[r][t] = fma(double(limb_sum(d)), double(sc[r]) * p2, acc[r][t]);
                        corr[r][t] += cr;
                    }
                }
            }
        }
    }
    __shared__ double s_acc[KS][R][T];
    __shared__ float s_corr[KS][R][T];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int t = 0; t < T; ++t) {
            for (int o = 16; o > 0; o >>= 1) {
                acc[r][t] += __shfl_xor_sync(0xffffffffu, acc[r][t], o);
                if (FMT == URB_FMT_INT4) corr[r][t] += __shfl_xor_sync(0xffffffffu, corr[r][t], o);
            }
            if (lane == 0) { s_acc[warp][r][t] = acc[r][t]; s_corr[warp][r][t] = corr[r][t]; }
        }
    __syncthreads();
    if (threadIdx.x < R * T) {
        const int r = threadIdx.x / T, t = threadIdx.x % T;
        const size_t i = rg * R + r;
        if (i < count && t < nt) {
            double v = s_acc[0][r][t];
            float c = s_corr[0][r][t];
#pragma unroll
            for (int k = 1; k < KS; ++k) { v += s_acc[k][r][t]; c += s_corr[k][r][t]; }
            y[size_t(t0 + t) * count + i] = FMT == URB_FMT_INT8
                                                ? float(__dmul_rn(v, double(__ldg(a.scales + row[r]))))
                                                : float(__dadd_rn(v, double(c)));
        }
    }
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

template <int FMT, int R, int T>
void launch_limbs_t(const IntArgs &a, size_t start, size_t count, const uint8_t *limbs, int cols32,
                    const int32_t *shift, const float *d_x, int batch, float *d_y, cudaStream_t st) {
    const size_t ctas = ((count + R - 1) / R) * ((size_t(batch) + T - 1) / T);
    k_int_limbs<FMT, R, T, 4, 2><<<unsigned(ctas), 128, 0, st>>>(a, start, count, limbs, cols32, shift,
                                                                d_x, batch, d_y);
}

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
    const bool limbs_ok = a.row_bytes % 16 == 0 && a.cols % 4 == 0 &&
                          (reinterpret_cast<uintptr_t>(d_x) & 15) == 0 &&
                          (m->format == URB_FMT_INT8 || a.group % 32 == 0);
    if (limbs_ok) {
        const int cols32 = int((m->cols + 31) / 32 * 32);
        const size_t limb_bytes = batch * size_t(kLimbs) * cols32;
        int rc = URB_OK;
        uint8_t *ws = static_cast<uint8_t *>(workspace(ctx, limb_bytes + batch * size_t(cols32 / 32) * 4 + 256, &rc));
        if (!ws) return rc;
        uint8_t *limbs = ws;
        int32_t *shift = reinterpret_cast<int32_t *>(ws + limb_bytes);
        const size_t threads = batch * size_t(cols32 / 4);
        k_x_limbs<<<unsigned((threads + 255) / 256), 256, 0, st>>>(d_x, a.cols, cols32, int(batch), limbs,
                                                                   shift, d_status);
        const int b = int(batch);
        // 4 rows share each load of a token's limbs; up to 4 tokens share each weight load.
        if (m->format == URB_FMT_INT8) {
            if (batch == 1) launch_limbs_t<URB_FMT_INT8, 4, 1>(a, start, count, limbs, cols32, shift, d_x, b, d_y, st);
            else if (batch == 2) launch_limbs_t<URB_FMT_INT8, 4, 2>(a, start, count, limbs, cols32, shift, d_x, b, d_y, st);
            else launch_limbs_t<URB_FMT_INT8, 4, 4>(a, start, count, limbs, cols32, shift, d_x, b, d_y, st);
        } else {
            // (INT4 with 4 rows and 2+ tokens would spill: 2 rows there.)
            if (batch == 1) launch_limbs_t<URB_FMT_INT4, 4, 1>(a, start, count, limbs, cols32, shift, d_x, b, d_y, st);
            else launch_limbs_t<URB_FMT_INT4, 2, 2>(a, start, count, limbs, cols32, shift, d_x, b, d_y, st);
        }
        const cudaError_t e = cudaGetLastError();
        return e == cudaSuccess ? URB_OK : cuda_fail(ctx, e, "int limb matvec");
    }
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
