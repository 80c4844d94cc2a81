// urb_oracle.cpp — CPU restatement of Urbilateria v0.2.4's routed-expert arithmetic.
//
// TEST INFRASTRUCTURE ONLY (see urb_oracle.h).  Build flags must keep IEEE semantics:
// -O2 -ffp-contract=off, no -ffast-math.  Floating-point operations are spelled out in the
// order and precision the Rust reference uses; comments cite the reference file:line.
//
// Rayon row parallelism (src/execution.rs:154 `should_parallelize`) is mirrored with OpenMP
// over output rows.  Parallelism never changes a row's arithmetic, only which thread runs it.

#include "urb_oracle.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

constexpr size_t kParallelMinWork = 64 * 1024;  // src/execution.rs:18 PARALLEL_MIN_WORK

inline float bits_f32(uint32_t b) { float f; std::memcpy(&f, &b, 4); return f; }
inline uint32_t f32_bits(float f) { uint32_t b; std::memcpy(&b, &f, 4); return b; }
inline bool finite(float v) { return std::isfinite(v); }

bool should_parallelize(size_t tasks, size_t work, int threads) {
    return tasks > 1 && work >= kParallelMinWork && threads > 1;
}

// src/math/mxfp.rs:54-57 decode_e8m0_unchecked: code<<23, code 0 -> 2^-127 (0x00400000).
inline float e8m0(uint8_t code) {
    uint32_t bits = uint32_t(code) << 23;
    return bits_f32(bits == 0 ? 0x00400000u : bits);
}

// src/math/mxfp.rs:60-71 decode_e4m3fn, evaluated in f32 exactly as written there.
float e4m3(uint8_t v) {
    float sign = (v & 0x80) == 0 ? 1.0f : -1.0f;
    int exponent = (v >> 3) & 0x0f;
    int mantissa = v & 0x07;
    if (exponent == 0) return sign * float(mantissa) * std::ldexp(1.0f, -9);
    if (exponent == 0x0f && mantissa == 0x07) return NAN;
    return sign * (1.0f + float(mantissa) / 8.0f) * std::ldexp(1.0f, exponent - 7);
}

// src/math/mxfp.rs:73-79 E2M1_TABLE.  Code 8 decodes to +0.0.
const float kE2M1[16] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f,
                         0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f};

inline float bf16f(uint16_t b) { return bits_f32(uint32_t(b) << 16); }

struct Tables {
    float e4m3[256];
    Tables() { for (int c = 0; c < 256; ++c) e4m3[c] = ::e4m3(uint8_t(c)); }
};
const Tables &tables() { static Tables t; return t; }

size_t div_ceil(size_t a, size_t b) { return (a + b - 1) / b; }

// ---------------------------------------------------------------------------------------
// Row dot products.

// src/math/mxfp.rs:1850-1873 dot_e2m1_e8m0_f64_ordered (bit-identical to the AVX2 form
// :1905-1971): f32 weight = e2m1 * scale, widened product, sequential f64 adds from +0.0.
float dot_mxfp4_f64(const uint8_t *packed, const uint8_t *scales, const float *x, size_t cols,
                    size_t group) {
    double sum = 0.0;
    size_t column = 0;
    for (size_t g = 0; column < cols; ++g) {
        float scale = e8m0(scales[g]);
        size_t end = std::min(cols, column + group);
        for (; column < end; ++column) {
            uint8_t byte = packed[column / 2];
            uint8_t code = (column % 2 == 0) ? (byte & 15) : (byte >> 4);
            float weight = kE2M1[code] * scale;
            sum += double(weight) * double(x[column]);
        }
    }
    return float(sum);
}

// src/math/mxfp.rs:1876-1898 dot_e2m1_e8m0_fp32_ordered: `sum += e2m1 * scale * x` in f32.
float dot_mxfp4_f32(const uint8_t *packed, const uint8_t *scales, const float *x, size_t cols,
                    size_t group) {
    float sum = 0.0f;
    size_t column = 0;
    for (size_t g = 0; column < cols; ++g) {
        float scale = e8m0(scales[g]);
        size_t end = std::min(cols, column + group);
        for (; column < end; ++column) {
            uint8_t byte = packed[column / 2];
            uint8_t code = (column % 2 == 0) ? (byte & 15) : (byte >> 4);
            float product = kE2M1[code] * scale;
            product = product * x[column];
            sum = sum + product;
        }
    }
    return sum;
}

// Rust 1.88 `Iterator::sum::<f32>` folds from -0.0 (the reference pins toolchain 1.88.0).
inline float rust_sum_f32(const float *v, size_t n) {
    float s = -0.0f;
    for (size_t i = 0; i < n; ++i) s = s + v[i];
    return s;
}

// MXFP8 scalar / ordered-AVX2 F64 path (src/math/mxfp.rs:754-765, 964-1006).
float dot_mxfp8_f64(const urbo_matrix *m, size_t row, const float *x) {
    const uint8_t *values = static_cast<const uint8_t *>(m->values) + row * m->cols;
    size_t scale_cols = div_ceil(m->cols, m->block_cols);
    const uint8_t *scales = m->scales + (row / m->block_rows) * scale_cols;
    const float *table = tables().e4m3;
    double sum = 0.0;
    size_t column = 0;
    for (size_t b = 0; column < m->cols; ++b) {
        float scale = e8m0(scales[b]);
        size_t end = std::min(m->cols, column + m->block_cols);
        for (; column < end; ++column) {
            float weight = table[values[column]] * scale;
            sum += double(weight) * double(x[column]);
        }
    }
    return float(sum);
}

// MXFP8 ModelOpt 1x32 on an AVX2+FMA host (src/math/mxfp.rs:1076-1158): eight FP32 FMA lanes
// over columns (lane = column % 8 within complete 8-chunks of each 32-block), lanes summed in
// order 0..7 by `Iterator::sum`, plus an FP32 scalar tail for partial blocks.
float dot_mxfp8_fma_lanes(const urbo_matrix *m, size_t row, const float *x) {
    const uint8_t *values = static_cast<const uint8_t *>(m->values) + row * m->cols;
    size_t scale_cols = div_ceil(m->cols, 32);
    const uint8_t *scales = m->scales + row * scale_cols;
    const float *table = tables().e4m3;
    float lanes[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    float scalar_tail = 0.0f;
    size_t column = 0;
    for (size_t b = 0; column < m->cols; ++b) {
        float scale = e8m0(scales[b]);
        size_t len = std::min<size_t>(32, m->cols - column);
        size_t complete = len / 8 * 8;
        for (size_t off = 0; off < complete; ++off) {
            float weight = table[values[column + off]] * scale;
            lanes[off % 8] = std::fma(weight, x[column + off], lanes[off % 8]);
        }
        for (size_t off = complete; off < len; ++off) {
            float weight = table[values[column + off]] * scale;
            float product = weight * x[column + off];
            scalar_tail = scalar_tail + product;
        }
        column += len;
    }
    return rust_sum_f32(lanes, 8) + scalar_tail;
}

// src/model/bf16.rs:494-525 dot_bf16_f64_ordered_avx2 (and scalar :481-486): from -0.0.
float dot_bf16_f64(const uint16_t *row, const float *x, size_t cols) {
    double sum = -0.0;
    for (size_t c = 0; c < cols; ++c) sum += double(bf16f(row[c])) * double(x[c]);
    return float(sum);
}

// src/model/matrix.rs:235-241 DenseMatrix: `sum::<f64>()` of widened products, from -0.0.
float dot_f32_f64(const float *row, const float *x, size_t cols) {
    double sum = -0.0;
    for (size_t c = 0; c < cols; ++c) sum += double(row[c]) * double(x[c]);
    return float(sum);
}

// src/math/quant.rs:448-499 Int8Matrix::matvec_rows: `sum::<f64>()` of f64(i8) * f64(x) (Rust
// 1.88 folds from -0.0), times f64(row scale), rounded to f32.
float dot_int8_f64(const urbo_matrix *m, size_t row, const float *x) {
    const int8_t *w = static_cast<const int8_t *>(m->values) + row * m->cols;
    double sum = -0.0;
    for (size_t c = 0; c < m->cols; ++c) sum += double(w[c]) * double(x[c]);
    return float(sum * double(m->fscales[row]));
}

// f32 weight (row, col) of an Int4Matrix (quant.rs:343-350): (code - 8) * scale in f32.
inline float int4_value(const urbo_matrix *m, size_t row, size_t col) {
    const uint8_t byte = static_cast<const uint8_t *>(m->values)[row * div_ceil(m->cols, 2) + col / 2];
    const uint8_t code = col % 2 == 0 ? (byte & 15) : (byte >> 4);
    return float(int(code) - 8) * m->fscales[row * div_ceil(m->cols, m->group_size) + col / m->group_size];
}

// src/math/quant.rs:304-318 Int4Matrix::dot_row: ordered f64 sum from +0.0 of the widened f32
// weights times the widened inputs, group by group in column order.
float dot_int4_f64(const urbo_matrix *m, size_t row, const float *x) {
    double sum = 0.0;
    for (size_t c = 0; c < m->cols; ++c) sum += double(int4_value(m, row, c)) * double(x[c]);
    return float(sum);
}

bool mxfp8_is_compact(const urbo_matrix *m) { return m->block_rows == 1 && m->block_cols == 32; }

// One row of WeightMatrix::matvec for the single-input dispatch of each format.
float dot_row(const urbo_matrix *m, size_t row, const float *x) {
    switch (m->format) {
    case URBO_F32:
        return dot_f32_f64(static_cast<const float *>(m->values) + row * m->cols, x, m->cols);
    case URBO_BF16:
        return dot_bf16_f64(static_cast<const uint16_t *>(m->values) + row * m->cols, x, m->cols);
    case URBO_MXFP8:
        // mxfp.rs:672-703: compact AVX2/FMA for 1x32 E8M0, else ordered F64.
        return mxfp8_is_compact(m) ? dot_mxfp8_fma_lanes(m, row, x) : dot_mxfp8_f64(m, row, x);
    case URBO_MXFP4: {
        size_t row_bytes = div_ceil(m->cols, 2), groups = div_ceil(m->cols, m->group_size);
        return dot_mxfp4_f64(static_cast<const uint8_t *>(m->values) + row * row_bytes,
                             m->scales + row * groups, x, m->cols, m->group_size);
    }
    case URBO_INT8:
        return dot_int8_f64(m, row, x);
    case URBO_INT4:
        return dot_int4_f64(m, row, x);
    }
    return NAN;
}

bool any_nonfinite(const float *v, size_t n) {
    for (size_t i = 0; i < n; ++i)
        if (!finite(v[i])) return true;
    return false;
}

template <class F>
void for_rows(size_t count, size_t work, int threads, F &&f) {
#ifdef _OPENMP
    if (should_parallelize(count, work, threads)) {
#pragma omp parallel for schedule(static) num_threads(threads)
        for (long long i = 0; i < (long long)count; ++i) f(size_t(i));
        return;
    }
#endif
    (void)work; (void)threads;
    for (size_t i = 0; i < count; ++i) f(i);
}

}  // namespace

extern "C" {

float urbo_decode_e8m0(uint8_t code) { return e8m0(code); }
float urbo_decode_e4m3fn(uint8_t code) { return e4m3(code); }
float urbo_decode_e2m1(uint8_t code) { return kE2M1[code & 15]; }
float urbo_expf(float v) { return std::exp(v); }  // glibc expf, as Rust's f32::exp on linux-gnu

// src/math/mxfp.rs:247-275 encode_e4m3fn_finite (RNE, saturating at 448).
uint8_t urbo_encode_e4m3fn(float value) {
    value = std::min(std::max(value, -448.0f), 448.0f);
    float magnitude = std::fabs(value);
    if (magnitude == 0.0f) return 0;
    uint32_t code;
    if (magnitude < std::ldexp(1.0f, -6)) {
        code = uint32_t(std::nearbyint(magnitude * 512.0f));  // ties-to-even (default mode)
    } else {
        const uint32_t discard = 20, round_bias = (1u << (discard - 1)) - 1;
        uint32_t bits = f32_bits(magnitude);
        uint32_t retained_lsb = (bits >> discard) & 1;
        uint32_t rounded = (bits + round_bias + retained_lsb) & ~((1u << discard) - 1);
        uint32_t e = (rounded >> 23) & 0xff;
        uint32_t exponent = e > 120 ? e - 120 : 0;
        uint32_t mantissa = (rounded >> discard) & 0x07;
        code = std::min<uint32_t>((exponent << 3) | mantissa, 0x7e);
    }
    if (std::signbit(value) && code != 0) code |= 0x80;
    return uint8_t(code);
}

int urbo_validate(const urbo_matrix *m) {
    if (m && m->format == URBO_INT4 && m->group_size == 0) return URBO_ERR_INVALID_GROUP;
    if (!m || m->rows == 0 || m->cols == 0) return URBO_ERR_SHAPE;
    size_t n = m->rows * m->cols;
    switch (m->format) {
    case URBO_F32:
    case URBO_BF16:
        return URBO_OK;
    case URBO_MXFP8: {  // mxfp.rs:394-425: shape, E4M3 NaN codes, then 0xFF scales
        if (m->block_rows == 0 || m->block_cols == 0) return URBO_ERR_SHAPE;
        const uint8_t *v = static_cast<const uint8_t *>(m->values);
        for (size_t i = 0; i < n; ++i)
            if ((v[i] & 0x7f) == 0x7f) return URBO_ERR_NONFINITE;
        size_t ns = div_ceil(m->rows, m->block_rows) * div_ceil(m->cols, m->block_cols);
        for (size_t i = 0; i < ns; ++i)
            if (m->scales[i] == 0xff) return URBO_ERR_INVALID_SCALE;
        return URBO_OK;
    }
    case URBO_MXFP4: {  // mxfp.rs:1415-1435: shape, then every scale != 0xFF
        if (m->group_size == 0) return URBO_ERR_SHAPE;
        size_t ns = m->rows * div_ceil(m->cols, m->group_size);
        for (size_t i = 0; i < ns; ++i)
            if (m->scales[i] == 0xff) return URBO_ERR_INVALID_SCALE;
        return URBO_OK;
    }
    case URBO_INT8:    // quant.rs:363-396: shape, then every scale finite and > 0
    case URBO_INT4: {  // quant.rs:92-131 (group size checked before the shape)
        size_t ns = m->format == URBO_INT8 ? m->rows : m->rows * div_ceil(m->cols, m->group_size);
        for (size_t i = 0; i < ns; ++i)
            if (!finite(m->fscales[i]) || !(m->fscales[i] > 0.0f)) return URBO_ERR_NONFINITE;
        return URBO_OK;
    }
    }
    return URBO_ERR_SHAPE;
}

int urbo_matvec_rows(const urbo_matrix *m, size_t start, size_t count, const float *x, float *y,
                     int threads) {
    // Validation order of every format: input finiteness, then row range
    // (mxfp.rs:1731-1743, 667-676; bf16.rs:127-145; matrix.rs:216-233).
    if (any_nonfinite(x, m->cols)) return URBO_ERR_NONFINITE;
    if (start + count < start || start + count > m->rows) return URBO_ERR_SHAPE;
    for_rows(count, count * m->cols, threads, [&](size_t i) { y[i] = dot_row(m, start + i, x); });
    // Only MXFP8 checks outputs on this path (mxfp.rs:712-714); MXFP4 does not (:1779).
    if (m->format == URBO_MXFP8 && any_nonfinite(y, count)) return URBO_ERR_NONFINITE;
    return URBO_OK;
}

// WeightMatrix::transpose_rows_matvec (src/model/weight.rs:332-343): per column, the ordered
// f64 sum over rows start..start+n of f64(weight) * f64(x[row - start]) from +0.0, rounded to
// f32 (mxfp.rs:785-858 MXFP8, whose AVX2 form :1308-1360 is the same sequence of exactly
// rounded adds of exact products; mxfp.rs:1782-1821 MXFP4; bf16.rs:430-475; matrix.rs:276-313).
// Input finiteness, then the row range; only MXFP8 rejects non-finite outputs (:851-856).
int urbo_transpose_rows_matvec(const urbo_matrix *m, size_t start, const float *x, size_t n,
                               float *y) {
    if (any_nonfinite(x, n)) return URBO_ERR_NONFINITE;
    if (start + n < start || start + n > m->rows) return URBO_ERR_SHAPE;
    const float *e4 = tables().e4m3;
    for (size_t c = 0; c < m->cols; ++c) {
        double sum = 0.0;
        for (size_t i = 0; i < n; ++i) {
            const size_t r = start + i;
            float w;
            switch (m->format) {
            case URBO_F32: w = static_cast<const float *>(m->values)[r * m->cols + c]; break;
            case URBO_BF16: w = bf16f(static_cast<const uint16_t *>(m->values)[r * m->cols + c]); break;
            case URBO_MXFP8: {
                const size_t sc = div_ceil(m->cols, m->block_cols);
                w = e4[static_cast<const uint8_t *>(m->values)[r * m->cols + c]] *
                    e8m0(m->scales[(r / m->block_rows) * sc + c / m->block_cols]);
                break;
            }
            case URBO_INT8: {
                // quant.rs:512-553: (f64(x) * f64(row scale)) * f64(i8), each product rounded.
                const double scaled = double(x[i]) * double(m->fscales[r]);
                sum += scaled * double(static_cast<const int8_t *>(m->values)[r * m->cols + c]);
                continue;
            }
            case URBO_INT4: w = int4_value(m, r, c); break;  // quant.rs:236-283
            default: {  // MXFP4
                const uint8_t byte = static_cast<const uint8_t *>(m->values)[r * div_ceil(m->cols, 2) + c / 2];
                w = kE2M1[(c % 2 == 0 ? byte : byte >> 4) & 15] *
                    e8m0(m->scales[r * div_ceil(m->cols, m->group_size) + c / m->group_size]);
            }
            }
            sum += double(x[i]) * double(w);
        }
        y[c] = float(sum);
    }
    if (m->format == URBO_MXFP8 && any_nonfinite(y, m->cols)) return URBO_ERR_NONFINITE;
    return URBO_OK;
}

// src/math/quant.rs:600-617 round_ties_even of an f32, as an integer.
static int32_t round_ties_even_i32(float value) {
    const float fl = std::floor(value);
    const float fraction = value - fl;
    const int32_t lower = int32_t(fl);
    if (fraction < 0.5f) return lower;
    if (fraction > 0.5f) return lower + 1;
    return lower % 2 == 0 ? lower : lower + 1;
}

int urbo_int4_quantize_grouped(size_t rows, size_t cols, size_t group, const float *values,
                               uint8_t *packed, float *scales) {
    // quant.rs:575-598 validate_geometry, then finiteness (:53-55).
    if (group == 0) return URBO_ERR_INVALID_GROUP;
    if (rows == 0 || cols == 0) return URBO_ERR_SHAPE;
    if (any_nonfinite(values, rows * cols)) return URBO_ERR_NONFINITE;
    const size_t row_bytes = div_ceil(cols, 2), groups = div_ceil(cols, group);
    std::fill(packed, packed + rows * row_bytes, uint8_t(0x88));
    for (size_t r = 0; r < rows; ++r) {
        const float *v = values + r * cols;
        for (size_t g = 0; g < groups; ++g) {
            float maximum = 0.0f;  // fold of f32::max over |v| (no NaN: inputs are finite)
            for (size_t c = g * group; c < std::min(cols, (g + 1) * group); ++c)
                maximum = std::max(maximum, std::fabs(v[c]));
            scales[r * groups + g] = std::max(maximum / 7.0f, 1e-8f);
        }
        for (size_t c = 0; c < cols; ++c) {
            const float scale = scales[r * groups + c / group];
            const int32_t q = std::min(std::max(round_ties_even_i32(v[c] / scale), -8), 7);
            const uint8_t code = uint8_t(q + 8);
            uint8_t &byte = packed[r * row_bytes + c / 2];
            byte = c % 2 == 0 ? uint8_t((byte & 0xf0) | code) : uint8_t((byte & 0x0f) | (code << 4));
        }
    }
    return URBO_OK;
}

int urbo_write_row(const urbo_matrix *m, size_t row, float *out) {
    if (row >= m->rows) return URBO_ERR_SHAPE;
    const float *e4 = tables().e4m3;
    for (size_t c = 0; c < m->cols; ++c) {
        switch (m->format) {
        case URBO_F32: out[c] = static_cast<const float *>(m->values)[row * m->cols + c]; break;
        case URBO_BF16: out[c] = bf16f(static_cast<const uint16_t *>(m->values)[row * m->cols + c]); break;
        case URBO_MXFP8: {
            const size_t sc = div_ceil(m->cols, m->block_cols);
            out[c] = e4[static_cast<const uint8_t *>(m->values)[row * m->cols + c]] *
                     e8m0(m->scales[(row / m->block_rows) * sc + c / m->block_cols]);
            break;
        }
        case URBO_MXFP4: {
            const uint8_t byte = static_cast<const uint8_t *>(m->values)[row * div_ceil(m->cols, 2) + c / 2];
            out[c] = kE2M1[(c % 2 == 0 ? byte : byte >> 4) & 15] *
                     e8m0(m->scales[row * div_ceil(m->cols, m->group_size) + c / m->group_size]);
            break;
        }
        case URBO_INT8:  // quant.rs:414-436
            out[c] = float(static_cast<const int8_t *>(m->values)[row * m->cols + c]) * m->fscales[row];
            break;
        default: out[c] = int4_value(m, row, c);
        }
    }
    return URBO_OK;
}

int urbo_mxfp4_matvec_rows_fp32(const urbo_matrix *m, size_t start, size_t count,
                                const float *x, float *y, int threads) {
    if (m->format != URBO_MXFP4) return URBO_ERR_SHAPE;
    if (any_nonfinite(x, m->cols)) return URBO_ERR_NONFINITE;
    if (start + count < start || start + count > m->rows) return URBO_ERR_SHAPE;
    size_t row_bytes = div_ceil(m->cols, 2), groups = div_ceil(m->cols, m->group_size);
    for_rows(count, count * m->cols, threads, [&](size_t i) {
        size_t r = start + i;
        y[i] = dot_mxfp4_f32(static_cast<const uint8_t *>(m->values) + r * row_bytes,
                             m->scales + r * groups, x, m->cols, m->group_size);
    });
    // mxfp.rs:1719-1721: the FP32 variant rejects non-finite outputs.
    return any_nonfinite(y, count) ? URBO_ERR_NONFINITE : URBO_OK;
}

// One chunk of MxFp4Matrix::matmul_rows / MxFp8Matrix::matmul_row_range.
static int matmul_chunk(const urbo_matrix *m, const float *x, size_t batch, float *y, int threads) {
    if (any_nonfinite(x, batch * m->cols)) return URBO_ERR_NONFINITE;
    bool batched = batch >= 2 && batch <= 12;
    if (m->format == URBO_MXFP4 && batched && m->group_size >= 8 && m->group_size % 2 == 0) {
        // mxfp.rs:1488-1555: decoded once, per-token ordered F64 (bit-equal to matvec), then
        // token-major transpose and an output finiteness check.
        for_rows(m->rows, batch * m->rows * m->cols, threads, [&](size_t r) {
            for (size_t t = 0; t < batch; ++t) y[t * m->rows + r] = dot_row(m, r, x + t * m->cols);
        });
        return any_nonfinite(y, batch * m->rows) ? URBO_ERR_NONFINITE : URBO_OK;
    }
    if (m->format == URBO_MXFP8 && batched) {
        bool compact = mxfp8_is_compact(m) && m->cols % 32 == 0;  // mxfp.rs:596-601
        bool ordered = m->block_cols >= 8;                           // mxfp.rs:602-605
        if (compact || ordered) {
            for_rows(m->rows, batch * m->rows * m->cols, threads, [&](size_t r) {
                for (size_t t = 0; t < batch; ++t)
                    y[t * m->rows + r] = compact ? dot_mxfp8_fma_lanes(m, r, x + t * m->cols)
                                                 : dot_mxfp8_f64(m, r, x + t * m->cols);
            });
            return any_nonfinite(y, batch * m->rows) ? URBO_ERR_NONFINITE : URBO_OK;
        }
    }
    for (size_t t = 0; t < batch; ++t) {  // per-token matvec fallback (mxfp.rs:1557-1560, :653-656)
        int rc = urbo_matvec_rows(m, 0, m->rows, x + t * m->cols, y + t * m->rows, threads);
        if (rc != URBO_OK) return rc;
    }
    return URBO_OK;
}

int urbo_matmul_rows(const urbo_matrix *m, const float *x, size_t batch, float *y, int threads) {
    if (batch == 0) return URBO_ERR_SHAPE;
    if (m->format == URBO_MXFP4 || m->format == URBO_MXFP8) {
        // src/model/weight.rs:116-146: split evenly into ceil(batch/12) chunks, the first
        // `batch % chunks` one token larger.
        size_t chunks = div_ceil(batch, 12), base = batch / chunks, larger = batch % chunks;
        size_t token = 0;
        for (size_t c = 0; c < chunks; ++c) {
            size_t b = base + (c < larger ? 1 : 0);
            int rc = matmul_chunk(m, x + token * m->cols, b, y + token * m->rows, threads);
            if (rc != URBO_OK) return rc;
            token += b;
        }
        return URBO_OK;
    }
    for (size_t t = 0; t < batch; ++t) {  // weight.rs:147-151
        int rc = urbo_matvec_rows(m, 0, m->rows, x + t * m->cols, y + t * m->rows, threads);
        if (rc != URBO_OK) return rc;
    }
    return URBO_OK;
}

// ---------------------------------------------------------------------------------------
// Routing.

// Rust f32::total_cmp as a signed-integer key (IEEE totalOrder on the bit pattern).
static inline int32_t total_key(float v) {
    int32_t b = int32_t(f32_bits(v));
    return b ^ int32_t(uint32_t(b >> 31) >> 1);
}

int urbo_route_noaux_tc(const float *logits, const float *bias, size_t n, size_t top_k,
                        size_t n_group, size_t topk_group, int normalize, float scaling,
                        int32_t *out_expert, float *out_weight, float *out_score) {
    // routing.rs:47-99 validation, in the reference's order.
    if (n == 0) return URBO_ERR_INVALID_GEOMETRY;
    for (size_t i = 0; i < n; ++i)
        if (!finite(logits[i]) || !finite(bias[i])) return URBO_ERR_NONFINITE;
    if (!finite(scaling)) return URBO_ERR_NONFINITE;
    if (scaling <= 0.0f) return URBO_ERR_INVALID_GEOMETRY;
    if (n_group == 0 || n % n_group != 0) return URBO_ERR_INVALID_GEOMETRY;
    if (top_k == 0 || top_k > n) return URBO_ERR_INVALID_GEOMETRY;
    if (topk_group == 0 || topk_group > n_group) return URBO_ERR_INVALID_GEOMETRY;
    size_t per_group = n / n_group;
    if (per_group < 2) return URBO_ERR_INVALID_GEOMETRY;

    // routing.rs:101-110: gate = 1 / (1 + exp(-logit)) in f32; selection = gate + bias.
    std::vector<float> gates(n), selection(n);
    for (size_t i = 0; i < n; ++i) {
        float e = std::exp(-logits[i]);
        gates[i] = 1.0f / (1.0f + e);
        selection[i] = gates[i] + bias[i];
    }
    // routing.rs:112-129: group score = sum of the two largest selections; rank groups.
    std::vector<std::pair<size_t, float>> groups;
    for (size_t g = 0; g < n_group; ++g) {
        std::vector<float> s(selection.begin() + g * per_group,
                             selection.begin() + (g + 1) * per_group);
        std::stable_sort(s.begin(), s.end(),
                         [](float a, float b) { return total_key(a) > total_key(b); });
        groups.push_back({g, s[0] + s[1]});
    }
    std::stable_sort(groups.begin(), groups.end(), [](const auto &a, const auto &b) {
        int32_t ka = total_key(a.second), kb = total_key(b.second);
        return ka != kb ? ka > kb : a.first < b.first;
    });
    std::vector<char> allowed(n, 0);
    for (size_t i = 0; i < topk_group; ++i)
        std::fill(allowed.begin() + groups[i].first * per_group,
                  allowed.begin() + (groups[i].first + 1) * per_group, 1);
    // routing.rs:131-141: rank allowed experts by selection desc, lower ID wins ties.
    std::vector<size_t> ranking;
    for (size_t i = 0; i < n; ++i)
        if (allowed[i]) ranking.push_back(i);
    std::stable_sort(ranking.begin(), ranking.end(), [&](size_t a, size_t b) {
        int32_t ka = total_key(selection[a]), kb = total_key(selection[b]);
        return ka != kb ? ka > kb : a < b;
    });
    if (ranking.size() < top_k) return URBO_ERR_INVALID_GEOMETRY;
    ranking.resize(top_k);
    // routing.rs:143-146: f32 sum (Rust 1.88 folds from -0.0) of gates in ranking order + 1e-20.
    float den = -0.0f;
    for (size_t e : ranking) den = den + gates[e];
    den = den + 1e-20f;
    if (normalize && !finite(den)) return URBO_ERR_NONFINITE;
    for (size_t i = 0; i < top_k; ++i) {  // routing.rs:147-160
        size_t e = ranking[i];
        float w = normalize ? gates[e] / den : gates[e];
        out_expert[i] = int32_t(e);
        out_weight[i] = w * scaling;
        if (out_score) out_score[i] = selection[e];
    }
    return URBO_OK;
}

int urbo_route_softmax_top_k(const float *logits, size_t n, size_t top_k, int32_t *out_expert,
                             float *out_weight) {
    // src/models/qwen3_8/moe.rs:95-159.
    if (n == 0 || top_k == 0 || top_k > n) return URBO_ERR_INVALID_GEOMETRY;
    for (size_t i = 0; i < n; ++i)
        if (!finite(logits[i])) return URBO_ERR_NONFINITE;
    float maximum = -INFINITY;
    for (size_t i = 0; i < n; ++i) maximum = std::fmax(maximum, logits[i]);
    std::vector<float> p(n);
    float den = 0.0f;
    for (size_t i = 0; i < n; ++i) {
        p[i] = std::exp(logits[i] - maximum);
        den = den + p[i];
    }
    if (!finite(den) || den <= 0.0f) return URBO_ERR_NONFINITE;
    for (size_t i = 0; i < n; ++i) p[i] = p[i] / den;
    std::vector<size_t> ranking(n);
    for (size_t i = 0; i < n; ++i) ranking[i] = i;
    std::stable_sort(ranking.begin(), ranking.end(), [&](size_t a, size_t b) {
        int32_t ka = total_key(p[a]), kb = total_key(p[b]);
        return ka != kb ? ka > kb : a < b;
    });
    float selected = 0.0f;
    for (size_t i = 0; i < top_k; ++i) selected = selected + p[ranking[i]];
    if (!finite(selected) || selected <= 0.0f) return URBO_ERR_NONFINITE;
    for (size_t i = 0; i < top_k; ++i) {
        out_expert[i] = int32_t(ranking[i]);
        out_weight[i] = p[ranking[i]] / selected;
        if (!finite(out_weight[i])) return URBO_ERR_NONFINITE;
    }
    return URBO_OK;
}

// ---------------------------------------------------------------------------------------
// SwiGLU expert and the MoE layer.

float urbo_silu(float v) {  // src/math/ops.rs:36-38
    float e = std::exp(-v);
    return v / (1.0f + e);
}

int urbo_gated_mlp_forward(const urbo_matrix *gate, const urbo_matrix *up,
                           const urbo_matrix *down, const float *x, float *y, int threads) {
    // src/model/mlp.rs:60-81 shape contract, then :90-99.
    if (gate->rows != up->rows || gate->cols != up->cols) return URBO_ERR_SHAPE;
    if (down->cols != gate->rows || down->rows != gate->cols) return URBO_ERR_SHAPE;
    std::vector<float> g(gate->rows), u(up->rows);
    int rc = urbo_matvec_rows(gate, 0, gate->rows, x, g.data(), threads);
    if (rc) return rc;
    rc = urbo_matvec_rows(up, 0, up->rows, x, u.data(), threads);
    if (rc) return rc;
    for (size_t i = 0; i < g.size(); ++i) g[i] = urbo_silu(g[i]) * u[i];
    return urbo_matvec_rows(down, 0, down->rows, g.data(), y, threads);
}

int urbo_group_routes(const int32_t *ids, size_t tokens, size_t top_k, size_t experts,
                      int32_t *counts, int32_t *offsets, int32_t *perm_token,
                      int32_t *perm_slot) {
    // qwen3_6/runtime.rs:1095,1123-1132: routes are visited token-major and appended to a
    // BTreeMap keyed by expert, so groups are experts ascending and tokens ascending inside.
    for (size_t e = 0; e < experts; ++e) counts[e] = 0;
    for (size_t i = 0; i < tokens * top_k; ++i) {
        if (ids[i] < 0 || size_t(ids[i]) >= experts) return URBO_ERR_SHAPE;
        counts[ids[i]]++;
    }
    offsets[0] = 0;
    for (size_t e = 0; e < experts; ++e) offsets[e + 1] = offsets[e] + counts[e];
    std::vector<int32_t> cursor(offsets, offsets + experts);
    for (size_t t = 0; t < tokens; ++t)
        for (size_t k = 0; k < top_k; ++k) {
            int32_t e = ids[t * top_k + k];
            int32_t p = cursor[e]++;
            perm_token[p] = int32_t(t);
            perm_slot[p] = int32_t(k);
        }
    return URBO_OK;
}

int urbo_moe_layer_forward(const urbo_moe_layer *L, const float *x, size_t tokens, float *out,
                           int32_t *route_expert, float *route_weight, float *route_score,
                           float *router_logits, int threads) {
    size_t hidden = L->router->cols, n = L->experts, k = L->top_k;
    if (L->router->rows != n) return URBO_ERR_SHAPE;
    std::vector<float> logits(n), shared(hidden), expert_out(hidden);
    std::vector<double> acc(hidden);
    for (size_t t = 0; t < tokens; ++t) {
        const float *xt = x + t * hidden;
        // glm/runtime/moe.rs:154-163
        int rc = urbo_matvec_rows(L->router, 0, n, xt, logits.data(), threads);
        if (rc) return rc;
        if (router_logits) std::copy(logits.begin(), logits.end(), router_logits + t * n);
        rc = urbo_route_noaux_tc(logits.data(), L->bias, n, k, L->n_group, L->topk_group,
                                 L->normalize, L->routed_scaling_factor, route_expert + t * k,
                                 route_weight + t * k, route_score ? route_score + t * k : nullptr);
        if (rc) return rc;
        // :164-175 shared expert, then routed experts in selection order, combined in f64.
        rc = urbo_gated_mlp_forward(L->shared_gate, L->shared_up, L->shared_down, xt,
                                    shared.data(), threads);
        if (rc) return rc;
        for (size_t h = 0; h < hidden; ++h) acc[h] = double(shared[h]);
        for (size_t r = 0; r < k; ++r) {
            size_t e = size_t(route_expert[t * k + r]);
            rc = urbo_gated_mlp_forward(&L->gate[e], &L->up[e], &L->down[e], xt,
                                        expert_out.data(), threads);
            if (rc) return rc;
            double w = double(route_weight[t * k + r]);
            for (size_t h = 0; h < hidden; ++h) acc[h] += w * double(expert_out[h]);
        }
        for (size_t h = 0; h < hidden; ++h) out[t * hidden + h] = float(acc[h]);
    }
    return URBO_OK;
}

// ---------------------------------------------------------------------------------------
// Checkpoint numerics (DeepSeek-V4): MX activation simulation, BF16 boundaries, bounded SwiGLU.

// src/math/mxfp.rs:300-319 power_of_two_ceiling: the exponent increment for interior mantissas;
// the band near powers of two keeps the log2 / ceil / powf formula (glibc log2f and powf, the
// libm Rust's f32::log2 / f32::powf call on linux-gnu).
float urbo_power_of_two_ceiling(float value) {
    const uint32_t bits = f32_bits(value);
    const uint32_t exponent = bits & 0x7f800000u, mantissa = bits & 0x007fffffu;
    if (mantissa == 0) return value;
    const uint32_t band = 4096;
    if (exponent == 0 || mantissa <= band || mantissa >= 0x007fffffu - band)
        return std::pow(2.0f, std::ceil(std::log2(value)));
    return bits_f32(exponent + 0x00800000u);
}

// src/math/mxfp.rs:91-115 simulate_e4m3_activation_in_place: per block, the scale is the power
// of two at or above max(|v|, 1e-4 start of the fold) / 448; values round-trip through E4M3.
int urbo_simulate_e4m3_activation(float *values, size_t n, size_t block) {
    if (n == 0 || block == 0) return URBO_ERR_SHAPE;
    if (any_nonfinite(values, n)) return URBO_ERR_NONFINITE;
    for (size_t b = 0; b < n; b += block) {
        const size_t e = std::min(n, b + block);
        float amax = 1.0e-4f;
        for (size_t i = b; i < e; ++i) amax = std::max(amax, std::fabs(values[i]));
        const float scale = urbo_power_of_two_ceiling(amax / 448.0f);
        for (size_t i = b; i < e; ++i) values[i] = e4m3(urbo_encode_e4m3fn(values[i] / scale)) * scale;
    }
    return URBO_OK;
}

// deepseek_v4/math.rs:90-101 round_to_bf16 (round to nearest even on the upper 16 bits).
float urbo_round_bf16(float value) {
    const uint32_t bits = f32_bits(value);
    return bits_f32((bits + 0x7fffu + ((bits >> 16) & 1u)) & 0xffff0000u);
}

// deepseek_v4/math.rs:518-549 bounded SwiGLU of one element.
float urbo_bounded_swiglu(float gate, float up, float limit) {
    const float g = std::min(gate, limit);
    const float u = std::min(std::max(up, -limit), limit);
    return g / (1.0f + std::exp(-g)) * u;
}

// WeightMatrix::uses_mx_activation_quantization (src/model/weight.rs:408-410).
static bool uses_mx(const urbo_matrix *m) { return m->format == URBO_MXFP8 || m->format == URBO_MXFP4; }

// DeepExpert::forward_with_mx_input (deepseek_v4/runtime.rs:3081-3104), per projection as
// linear_with_mx_activation / linear (deepseek_v4/math.rs:106-141): an MX gate / up reads the
// simulated input mx_x and its output rounds to BF16, a plain (F32 / BF16 / INT) one reads x
// unrounded; bounded SwiGLU, the route weight applied to the activation (none for the shared
// expert), BF16; an MX down projection simulates the activation as E4M3 per 128 and rounds its
// output to BF16, a plain one multiplies the activation as it is.
int urbo_deepseek_expert_forward(const urbo_matrix *gate, const urbo_matrix *up,
                                 const urbo_matrix *down, const float *x, const float *mx_x,
                                 const float *route_weight, float limit, float *y, int threads) {
    const size_t I = gate->rows;
    std::vector<float> g(I), u(I);
    int rc = urbo_matvec_rows(gate, 0, I, uses_mx(gate) ? mx_x : x, g.data(), threads);
    if (rc) return rc;
    rc = urbo_matvec_rows(up, 0, I, uses_mx(up) ? mx_x : x, u.data(), threads);
    if (rc) return rc;
    if (route_weight && (!finite(*route_weight) || *route_weight < 0.0f)) return URBO_ERR_INVALID;
    for (size_t i = 0; i < I; ++i) {
        const float gv = uses_mx(gate) ? urbo_round_bf16(g[i]) : g[i];
        const float uv = uses_mx(up) ? urbo_round_bf16(u[i]) : u[i];
        float a = urbo_bounded_swiglu(gv, uv, limit);
        if (route_weight) a *= *route_weight;
        g[i] = urbo_round_bf16(a);
        if (!finite(g[i])) return URBO_ERR_NONFINITE;
    }
    if (uses_mx(down)) {
        rc = urbo_simulate_e4m3_activation(g.data(), I, 128);
        if (rc) return rc;
    }
    rc = urbo_matvec_rows(down, 0, down->rows, g.data(), y, threads);
    if (rc) return rc;
    if (uses_mx(down))
        for (size_t h = 0; h < down->rows; ++h) y[h] = urbo_round_bf16(y[h]);
    return URBO_OK;
}

// The DeepSeek-V4 MoE composition for given routes (deepseek_v4/runtime.rs:2500-2650 with
// prepare_routes :2651-2700): the input simulated once (E4M3, blocks of 128), routed experts in
// ascending expert id accumulated in f32, the shared expert added last, the sum cast to BF16.
int urbo_moe_deepseek_forward(const urbo_moe_layer *L, const float *x, size_t tokens,
                              const int32_t *route_expert, const float *route_weight, float limit,
                              float *out, int threads) {
    const size_t H = L->router->cols, k = L->top_k;
    std::vector<float> mx(H), y(H), acc(H), shared(H);
    std::vector<std::pair<int32_t, float>> order(k);
    for (size_t t = 0; t < tokens; ++t) {
        std::copy(x + t * H, x + (t + 1) * H, mx.begin());
        int rc = urbo_simulate_e4m3_activation(mx.data(), H, 128);
        if (rc) return rc;
        for (size_t r = 0; r < k; ++r) order[r] = {route_expert[t * k + r], route_weight[t * k + r]};
        std::stable_sort(order.begin(), order.end(),
                         [](const std::pair<int32_t, float> &a, const std::pair<int32_t, float> &b) {
                             return a.first < b.first;
                         });
        std::fill(acc.begin(), acc.end(), 0.0f);
        for (size_t r = 0; r < k; ++r) {
            const size_t e = size_t(order[r].first);
            if (e >= L->experts) return URBO_ERR_SHAPE;
            rc = urbo_deepseek_expert_forward(&L->gate[e], &L->up[e], &L->down[e], x + t * H,
                                              mx.data(), &order[r].second, limit, y.data(), threads);
            if (rc) return rc;
            for (size_t h = 0; h < H; ++h) acc[h] += y[h];
        }
        rc = urbo_deepseek_expert_forward(L->shared_gate, L->shared_up, L->shared_down, x + t * H,
                                          mx.data(), nullptr, limit, shared.data(), threads);
        if (rc) return rc;
        for (size_t h = 0; h < H; ++h) out[t * H + h] = urbo_round_bf16(acc[h] + shared[h]);
    }
    return URBO_OK;
}

// deepseek_v4/math.rs:604-610 softplus (libm expf / log1pf, as Rust's f32::exp / ln_1p).
static float softplus(float v) {
    return v > 0.0f ? v + std::log1p(std::exp(-v)) : std::log1p(std::exp(v));
}

// deepseek_v4/math.rs:451-516 route_sqrt_softplus for one row of logits.
int urbo_route_sqrt_softplus(const float *logits, const float *bias, size_t n,
                             const int32_t *hash, size_t top_k, float scaling, int32_t *out_expert,
                             float *out_weight, float *out_score) {
    if (n == 0 || top_k == 0 || top_k > n) return URBO_ERR_SHAPE;
    if (!(scaling > 0.0f) || !finite(scaling)) return URBO_ERR_INVALID;
    if (any_nonfinite(logits, n) || (bias && any_nonfinite(bias, n))) return URBO_ERR_NONFINITE;
    std::vector<float> score(n), sel(n);
    for (size_t i = 0; i < n; ++i) {
        score[i] = std::sqrt(softplus(logits[i]));
        sel[i] = score[i] + (bias ? bias[i] : 0.0f);
    }
    std::vector<int32_t> experts(top_k);
    if (hash) {
        for (size_t r = 0; r < top_k; ++r) {
            if (hash[r] < 0 || size_t(hash[r]) >= n) return URBO_ERR_INVALID;
            experts[r] = hash[r];
        }
    } else {
        std::vector<int32_t> ranking(n);
        for (size_t i = 0; i < n; ++i) ranking[i] = int32_t(i);
        std::stable_sort(ranking.begin(), ranking.end(), [&](int32_t a, int32_t b) {
            const int32_t ka = total_key(sel[a]), kb = total_key(sel[b]);
            return ka != kb ? ka > kb : a < b;
        });
        std::copy(ranking.begin(), ranking.begin() + long(top_k), experts.begin());
    }
    float den = -0.0f;  // Iterator::sum over f32
    for (int32_t e : experts) den += score[e];
    if (!finite(den) || den <= 0.0f) return URBO_ERR_NONFINITE;
    for (size_t r = 0; r < top_k; ++r) {
        out_expert[r] = experts[r];
        out_weight[r] = score[experts[r]] / den * scaling;
        if (out_score) out_score[r] = sel[experts[r]];
    }
    return URBO_OK;
}

// MoeWeights::forward of DeepSeek-V4 (deepseek_v4/runtime.rs:2484-2700): router logits (the
// layer's router matvec), route_sqrt_softplus with the layer bias and scaling (or the given hash
// experts), then urbo_moe_deepseek_forward for the routes.
int urbo_moe_deepseek_layer_forward(const urbo_moe_layer *L, const float *x, size_t tokens,
                                    const int32_t *hash, float limit, float *out,
                                    int32_t *route_expert, float *route_weight, int threads) {
    const size_t H = L->router->cols, n = L->experts, k = L->top_k;
    std::vector<float> logits(n);
    for (size_t t = 0; t < tokens; ++t) {
        int rc = urbo_matvec_rows(L->router, 0, n, x + t * H, logits.data(), threads);
        if (rc) return rc;
        rc = urbo_route_sqrt_softplus(logits.data(), L->bias, n, hash ? hash + t * k : nullptr, k,
                                      L->routed_scaling_factor, route_expert + t * k,
                                      route_weight + t * k, nullptr);
        if (rc) return rc;
    }
    return urbo_moe_deepseek_forward(L, x, tokens, route_expert, route_weight, limit, out, threads);
}

// ---------------------------------------------------------------------------------------
// Checkpoint numerics (Qwen3.6): FP32-lane BF16 linear, fine-grained E4M3 activations, BF16
// boundaries, softmax routing, expert-order BF16 accumulation, sigmoid-gated shared expert.

// src/model/bf16.rs:591-613 dot_bf16_fp32_avx2_fma: eight FMA lanes over the columns
// (column c in lane c % 8, from +0.0), lanes summed in order (Iterator::sum from -0.0), the
// columns past the last multiple of eight added by separate multiply and add.
float urbo_dot_bf16_fp32_lanes(const uint16_t *row, const float *x, size_t cols) {
    float lanes[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    const size_t complete = cols / 8 * 8;
    for (size_t c = 0; c < complete; ++c) lanes[c % 8] = std::fma(bf16f(row[c]), x[c], lanes[c % 8]);
    float sum = rust_sum_f32(lanes, 8);
    for (size_t c = complete; c < cols; ++c) {
        const float product = bf16f(row[c]) * x[c];
        sum = sum + product;
    }
    return sum;
}

// src/math/mxfp.rs:122-149 simulate_finegrained_e4m3_activation: per block the exact scale
// max|v| / 448 (all-zero blocks stay zero).
int urbo_simulate_finegrained_e4m3(float *values, size_t n, size_t block) {
    if (n == 0 || block == 0) return URBO_ERR_SHAPE;
    if (any_nonfinite(values, n)) return URBO_ERR_NONFINITE;
    for (size_t b = 0; b < n; b += block) {
        const size_t e = std::min(n, b + block);
        float amax = 0.0f;
        for (size_t i = b; i < e; ++i) amax = std::max(amax, std::fabs(values[i]));
        if (amax == 0.0f) {
            for (size_t i = b; i < e; ++i) values[i] = 0.0f;
            continue;
        }
        const float scale = amax / 448.0f;
        for (size_t i = b; i < e; ++i) values[i] = e4m3(urbo_encode_e4m3fn(values[i] / scale)) * scale;
    }
    return URBO_OK;
}

// qwen3_8/math.rs:10-26 linear: MX weights see the fine-grained E4M3 activation (groups of
// 128) and the output rounds to BF16; BF16 weights use the FP32 lanes and round to BF16.
static int qwen_linear(const urbo_matrix *m, const float *x, float *y, int threads) {
    std::vector<float> xq(x, x + m->cols);
    int rc;
    if (m->format == URBO_MXFP4 || m->format == URBO_MXFP8) {
        rc = urbo_simulate_finegrained_e4m3(xq.data(), m->cols, 128);
        if (rc) return rc;
        rc = urbo_matvec_rows(m, 0, m->rows, xq.data(), y, threads);
        if (rc) return rc;
    } else if (m->format == URBO_BF16) {
        const uint16_t *w = static_cast<const uint16_t *>(m->values);
        for (size_t r = 0; r < m->rows; ++r) y[r] = urbo_dot_bf16_fp32_lanes(w + r * m->cols, x, m->cols);
    } else {
        return urbo_matvec_rows(m, 0, m->rows, x, y, threads);  // plain F32: no rounding
    }
    for (size_t r = 0; r < m->rows; ++r) {
        y[r] = urbo_round_bf16(y[r]);
        if (!finite(y[r])) return URBO_ERR_NONFINITE;
    }
    return URBO_OK;
}

// Qwen38Expert::forward_projections (qwen3_8/expert.rs:137-200) with BF16 boundaries.
static int qwen_expert(const urbo_matrix *gate, const urbo_matrix *up, const urbo_matrix *down,
                       const float *x, float *y, int threads) {
    const size_t I = gate->rows;
    std::vector<float> g(I), u(I);
    int rc = qwen_linear(gate, x, g.data(), threads);
    if (rc) return rc;
    rc = qwen_linear(up, x, u.data(), threads);
    if (rc) return rc;
    for (size_t i = 0; i < I; ++i) {
        const float a = urbo_round_bf16(urbo_silu(g[i]));
        const float v = a * u[i];
        if (!finite(v)) return URBO_ERR_NONFINITE;
        g[i] = urbo_round_bf16(v);
    }
    return qwen_linear(down, g.data(), y, threads);
}

// execute_batched_moe (qwen3_6/runtime.rs:1067-1215) for one token at a time: BF16 router
// (FP32 lanes, BF16 logits), softmax top-k with BF16 weights, routed experts accumulated in
// ascending expert id with BF16 contributions and sums, then the shared expert scaled by the
// sigmoid of its BF16 gate logit, all BF16.
int urbo_moe_qwen_layer_forward(const urbo_moe_layer *L, const urbo_matrix *shared_gate_vec,
                                const float *x, size_t tokens, float *out, int32_t *route_expert,
                                float *route_weight, int threads) {
    const size_t H = L->router->cols, n = L->experts, k = L->top_k;
    std::vector<float> logits(n), y(H), acc(H), shared(H);
    std::vector<std::pair<int32_t, float>> order(k);
    for (size_t t = 0; t < tokens; ++t) {
        const float *xt = x + t * H;
        int rc = qwen_linear(L->router, xt, logits.data(), threads);
        if (rc) return rc;
        rc = urbo_route_softmax_top_k(logits.data(), n, k, route_expert + t * k, route_weight + t * k);
        if (rc) return rc;
        for (size_t r = 0; r < k; ++r) {
            route_weight[t * k + r] = urbo_round_bf16(route_weight[t * k + r]);
            order[r] = {route_expert[t * k + r], route_weight[t * k + r]};
        }
        std::stable_sort(order.begin(), order.end(),
                         [](const std::pair<int32_t, float> &a, const std::pair<int32_t, float> &b) {
                             return a.first < b.first;
                         });
        std::fill(acc.begin(), acc.end(), 0.0f);
        for (size_t r = 0; r < k; ++r) {
            const size_t e = size_t(order[r].first);
            rc = qwen_expert(&L->gate[e], &L->up[e], &L->down[e], xt, y.data(), threads);
            if (rc) return rc;
            for (size_t h = 0; h < H; ++h) {
                const float c = urbo_round_bf16(order[r].second * y[h]);
                acc[h] = urbo_round_bf16(acc[h] + c);
            }
        }
        rc = qwen_expert(L->shared_gate, L->shared_up, L->shared_down, xt, shared.data(), threads);
        if (rc) return rc;
        float gate;
        rc = qwen_linear(shared_gate_vec, xt, &gate, threads);
        if (rc) return rc;
        float scale;
        if (gate >= 0.0f) {
            scale = 1.0f / (1.0f + std::exp(-gate));
        } else {
            const float e = std::exp(gate);
            scale = e / (1.0f + e);
        }
        scale = urbo_round_bf16(scale);
        for (size_t h = 0; h < H; ++h) {
            const float c = urbo_round_bf16(scale * shared[h]);
            out[t * H + h] = urbo_round_bf16(acc[h] + c);
            if (!finite(out[t * H + h])) return URBO_ERR_NONFINITE;
        }
    }
    return URBO_OK;
}

}  // extern "C"
