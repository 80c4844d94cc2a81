// bs_terms.cuh — residual-term encoding of f32 activations for the block-scaled tcgen05 MMAs
// (kind::mxf4 / kind::mxf8f6f4): x ~= t0 + t1 + ..., each term a block of 32 E2M1 or E4M3
// elements with its own E8M0 scale, built by a lane quad (8 values per lane).
#pragma once
#include <cuda_fp4.h>
#include <cuda_fp8.h>

#include "urb_internal.cuh"

namespace urb {
namespace {

// 2^e as a float for -149 <= e <= 127 (exact; subnormal below -126).
__device__ __forceinline__ float pow2f(int e) {
    return e >= -126 ? __int_as_float((e + 127) << 23) : __int_as_float(1 << (e + 149));
}

// One residual term of a 32-value block held by a lane quad (8 values per lane): the E8M0
// exponent e that fits the block's max|r| into the element range, the element codes of
// r * 2^-e (round to nearest even, by the hardware conversion to E2M1 / E4M3) and
// r -= decode * 2^e (exact: the decoded value times a power of two is a float, and r minus it
// is the rounding error of r, a float).  Every lane of the warp must call it (quad shuffles).
// Returns the scale byte; q receives this lane's 8 codes (E2M1: one word, element 0 in the low
// nibble; E4M3: two words, element 0 in the low byte).
template <int FMT>
__device__ __forceinline__ int make_term8(float *r, uint32_t *q) {
    float m = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) m = fmaxf(m, fabsf(r[i]));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
    q[0] = 0;
    if (FMT == URB_FMT_MXFP8) q[1] = 0;
    if (m == 0.0f) return 0;
    const int e0 = ilogbf(m);
    // Largest element magnitude: 6 = 1.5 * 2^2 (E2M1), 448 = 1.75 * 2^8 (E4M3).
    int e = FMT == URB_FMT_MXFP4 ? (m <= 1.5f * pow2f(e0) ? e0 - 2 : e0 - 1)
                                 : (m <= 1.75f * pow2f(e0) ? e0 - 8 : e0 - 7);
    e = max(-127, min(127, e));
    const float inv = pow2f(-e), sc = pow2f(e);
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
        const float2 v = make_float2(r[i] * inv, r[i + 1] * inv);
        __half2_raw d;
        if (FMT == URB_FMT_MXFP4) {
            const __nv_fp4x2_storage_t c = __nv_cvt_float2_to_fp4x2(v, __NV_E2M1, cudaRoundNearest);
            d = __nv_cvt_fp4x2_to_halfraw2(c, __NV_E2M1);
            q[0] |= uint32_t(c) << (4 * i);
        } else {
            const __nv_fp8x2_storage_t c = __nv_cvt_float2_to_fp8x2(v, __NV_SATFINITE, __NV_E4M3);
            d = __nv_cvt_fp8x2_to_halfraw2(c, __NV_E4M3);
            q[i >> 2] |= uint32_t(c) << (8 * (i & 3));
        }
        const float2 dq = __half22float2(*reinterpret_cast<const __half2 *>(&d));
        r[i] -= dq.x * sc;
        r[i + 1] -= dq.y * sc;
    }
    return e + 127;
}

}  // namespace
}  // namespace urb
