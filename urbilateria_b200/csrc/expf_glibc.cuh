// expf_glibc.cuh — device evaluation of the libm expf the reference links.
//
// The reference's router sigmoid (src/math/routing.rs:101-104) and softmax
// (src/models/qwen3_8/moe.rs:113) call Rust's f32::exp, i.e. libm `expf`.  The device computes
// (float)exp((double)x), a single rounding of a double exponential, and overrides it with the
// libm result for the inputs recorded by the build step gen_expf_table.c (where libm is not
// correctly rounded, or where e^x sits within 2^-48 of a float midpoint).  Lookup: a
// (2^20+1)-entry index over the top 20 bits of the input (0.16 keys per bucket on average),
// then a short scan of the sorted keys.
#pragma once
#include <stdint.h>

#include "urb_internal.cuh"

namespace urb {

// expf_libm with the bucket's key range [lo, hi) already loaded from t.index.
__device__ __forceinline__ float expf_libm_range(float x, const ExpfTable &t, uint32_t lo,
                                                 uint32_t hi) {
    const uint32_t k = __float_as_uint(x);
    for (uint32_t i = lo; i < hi; ++i)
        if (t.keys[i] == k) return __uint_as_float(t.vals[i]);
    return float(exp(double(x)));
}

__device__ __forceinline__ float expf_libm(float x, const ExpfTable &t) {
    uint32_t k = __float_as_uint(x);
    if (t.index) {
        uint32_t b = k >> 12;
        for (uint32_t i = t.index[b], e = t.index[b + 1]; i < e; ++i)
            if (t.keys[i] == k) return __uint_as_float(t.vals[i]);
    }
    return float(exp(double(x)));
}

// libm log1pf (Rust's f32::ln_1p) on [0, 1]: (float)log1p((double)x) unless the build step
// gen_log1pf_table.c recorded the input (libm not correctly rounded there, or log1p(x) within
// 2^-48 of a float midpoint).  Same table layout as ExpfTable.
__device__ __forceinline__ float log1pf_libm(float x, const ExpfTable &t) {
    uint32_t k = __float_as_uint(x);
    if (t.index && k <= 0x3F800000u) {
        uint32_t b = k >> 12;
        for (uint32_t i = t.index[b], e = t.index[b + 1]; i < e; ++i)
            if (t.keys[i] == k) return __uint_as_float(t.vals[i]);
    }
    return float(log1p(double(x)));
}

}  // namespace urb
