// numerics.cuh — checkpoint numerics of the DeepSeek-V4 expert path, on the device:
//  * E4M3 activation simulation (src/math/mxfp.rs:91-115): per block, scale = the power of two
//    at or above max(|v|, 1e-4) / 448 (power_of_two_ceiling, :300-319), v -> decode(encode(v /
//    scale)) * scale with the round-to-nearest-even, saturating E4M3FN encoder of :247-275;
//  * round_to_bf16 (deepseek_v4/math.rs:90-101): round to nearest even on the upper 16 bits;
//  * bounded SwiGLU (deepseek_v4/math.rs:518-549): min(g, L) / (1 + exp(-min(g, L))) *
//    clamp(u, -L, L).
// and of the Qwen3.6 expert path:
//  * fine-grained E4M3 activation simulation (src/math/mxfp.rs:122-149): per block the exact
//    scale max|v| / 448, v -> decode(encode(v / scale)) * scale; all-zero blocks stay zero;
//  * silu (src/math/ops.rs:36-38) with the libm expf: v / (1 + exp(-v)).
#pragma once
#include <stdint.h>

#include "expf_glibc.cuh"

namespace urb {

// E4M3FN code of a finite value (RNE, saturating at 448; mxfp.rs:247-275).
__device__ __forceinline__ uint32_t num_e4m3_encode(float value) {
    value = fminf(fmaxf(value, -448.0f), 448.0f);
    const float magnitude = fabsf(value);
    if (magnitude == 0.0f) return 0;
    uint32_t code;
    if (magnitude < 0.015625f) {  // 2^-6: subnormals on an exact 2^-9 grid
        code = uint32_t(__float2int_rn(magnitude * 512.0f));
    } else {
        const uint32_t bits = __float_as_uint(magnitude);
        const uint32_t rounded = (bits + ((1u << 19) - 1) + ((bits >> 20) & 1u)) & ~((1u << 20) - 1);
        const uint32_t e = (rounded >> 23) & 0xffu;
        const uint32_t exponent = e > 120 ? e - 120 : 0;
        code = min(((exponent << 3) | ((rounded >> 20) & 7u)), 0x7eu);
    }
    return (signbit(value) && code) ? (code | 0x80u) : code;
}

// Value of a finite E4M3FN code (exact).
__device__ __forceinline__ float num_e4m3_decode(uint32_t code) {
    const uint32_t e = (code >> 3) & 0xfu, m = code & 7u;
    const float mag = e == 0 ? float(m) * 0.001953125f  // m * 2^-9
                             : __uint_as_float(((e + 120u) << 23) | (m << 20));
    return (code & 0x80u) ? -mag : mag;
}

// power_of_two_ceiling (mxfp.rs:300-319) of a finite positive value.  Interior mantissas step
// the exponent; within 4,096 mantissa units of a power of two the reference evaluates
// 2^ceil(log2f(v)): log2 is formed in f64 and rounded once to f32 (the correctly rounded f32
// logarithm for these inputs, whose distance from an f32 rounding midpoint exceeds the f64
// error by many orders of magnitude), then ceiled.
__device__ __forceinline__ float num_pow2_ceil(float value) {
    const uint32_t bits = __float_as_uint(value);
    const uint32_t exponent = bits & 0x7f800000u, mantissa = bits & 0x007fffffu;
    if (mantissa == 0) return value;
    const uint32_t band = 4096;
    if (exponent == 0 || mantissa <= band || mantissa >= 0x007fffffu - band) {
        const float l = __double2float_rn(log2(double(value)));
        const int k = int(ceilf(l));
        return ldexpf(1.0f, k);
    }
    return __uint_as_float(exponent + 0x00800000u);
}

// E4M3 round trip of one value with a block scale (a power of two, so the division is exact).
__device__ __forceinline__ float num_e4m3_sim(float v, float scale) {
    return num_e4m3_decode(num_e4m3_encode(__fdiv_rn(v, scale))) * scale;
}

// Block scale of the simulation from the block's max |v| (the fold starts at 1e-4).
__device__ __forceinline__ float num_e4m3_scale(float amax) {
    return num_pow2_ceil(__fdiv_rn(fmaxf(amax, 1.0e-4f), 448.0f));
}

// Fine-grained E4M3 round trip of one value of a block whose max |v| is amax.
__device__ __forceinline__ float num_e4m3_sim_fine(float v, float amax) {
    if (amax == 0.0f) return 0.0f;
    const float scale = __fdiv_rn(amax, 448.0f);
    return __fmul_rn(num_e4m3_decode(num_e4m3_encode(__fdiv_rn(v, scale))), scale);
}

__device__ __forceinline__ float num_silu_libm(float v, const ExpfTable &tab) {
    return __fdiv_rn(v, __fadd_rn(1.0f, expf_libm(-v, tab)));
}

__device__ __forceinline__ float num_round_bf16(float v) {
    const uint32_t bits = __float_as_uint(v);
    return __uint_as_float((bits + 0x7fffu + ((bits >> 16) & 1u)) & 0xffff0000u);
}

__device__ __forceinline__ float num_bounded_swiglu(float gate, float up, float limit) {
    const float g = fminf(gate, limit);
    const float u = fminf(fmaxf(up, -limit), limit);
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
}

}  // namespace urb
