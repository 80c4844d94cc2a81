// bs_terms.cuh — residual-term encoding of f32 activations for the block-scaled tcgen05 MMAs
// (kind::mxf4 / kind::mxf8f6f4): x ~= t0 + t1 + ..., each term a block of 32 E2M1 or E4M3
// elements with its own E8M0 scale, built by a lane quad (8 values per lane).
#pragma once
#include "urb_internal.cuh"

namespace urb {
namespace {

// 2^e as a float for -149 <= e <= 127 (exact; subnormal below -126).
__device__ __forceinline__ float pow2f(int e) {
    return e >= -126 ? __int_as_float((e + 127) << 23) : __int_as_float(1 << (e + 149));
}

// Round to nearest (ties to even code) of |v| onto the E2M1 grid {0, .5, 1, 1.5, 2, 3, 4, 6}
// for |v| <= 6: returns the magnitude code (0..7) and the grid value.
__device__ __forceinline__ int e2m1_round(float a, float *dq) {
    float q;
    int idx;
    if (a < 2.0f) {
        q = rintf(a * 2.0f) * 0.5f;  // spacing 0.5; 2.0 lands in the next binade
    } else if (a < 4.0f) {
        q = rintf(a);                // spacing 1
    } else {
        q = 2.0f * rintf(a * 0.5f);  // spacing 2
    }
    if (q < 2.0f) idx = int(q * 2.0f);
    else if (q < 4.0f) idx = int(q) + 2;
    else idx = int(q * 0.5f) + 4;
    *dq = q;
    return idx;
}

// Round to nearest even of |v| onto E4M3 (finite, |v| <= 448): magnitude code and value.
__device__ __forceinline__ int e4m3_round(float a, float *dq) {
    if (a < 0.015625f) {             // subnormal binade, spacing 2^-9 (m = 8 is 2^-6, code 8)
        const float m = rintf(a * 512.0f);
        *dq = m * (1.0f / 512.0f);
        return int(m);
    }
    int k = ilogbf(a);
    float m = rintf(a * pow2f(3 - k));  // 8..16 steps of 2^(k-3)
    if (m == 16.0f) { ++k; m = 8.0f; }
    *dq = m * pow2f(k - 3);
    return ((k + 7) << 3) | (int(m) - 8);
}

// One residual term of a 32-value block held by a lane quad (8 values per lane): the E8M0
// exponent e that fits the block's max|r| into the element range, the element codes of
// r * 2^-e (round to nearest even) and r -= decode * 2^e (exact).  Every lane of the warp must
// call it (quad shuffles).  Returns the scale byte; q receives this lane's 8 codes (E2M1: one
// word, element 0 in the low nibble; E4M3: two words, element 0 in the low byte).
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
    for (int i = 0; i < 8; ++i) {
        const float v = r[i] * inv;
        float dq;
        if (FMT == URB_FMT_MXFP4) {
            int code = e2m1_round(fabsf(v), &dq);
            if (v < 0.0f && code) code |= 8;
            q[0] |= uint32_t(code) << (4 * i);
        } else {
            int code = e4m3_round(fabsf(v), &dq);
            if (v < 0.0f && code) code |= 0x80;
            q[i >> 2] |= uint32_t(code) << (8 * (i & 3));
        }
        r[i] -= copysignf(dq, v) * sc;
    }
    return e + 127;
}

}  // namespace
}  // namespace urb
