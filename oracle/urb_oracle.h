/*
 * urb_oracle.h — CPU oracle for the routed-expert (MoE) hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library restates, in plain C++17, the CPU arithmetic of
 * Urbilateria v0.2.4 (a pure-Rust runtime that cannot be compiled in this image) so that the
 * CUDA path can be checked against it.  Only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg load it.  The product library (liburb_moe.so) never links or calls it.
 *
 * Every function cites the reference file:line it follows.  Parity of this restatement is
 * pinned by the known-answer tests in tests/test_oracle_golden.py, which replay the reference's
 * own unit-test vectors (src/math/mxfp.rs, src/math/routing.rs, src/model/mlp.rs,
 * src/models/qwen3_8/moe.rs) against it.
 *
 * Status codes are shared with the product C ABI (include/urb_moe.h).
 */
#ifndef URB_ORACLE_H
#define URB_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Weight formats of WeightMatrix (src/model/weight.rs:54-61) that the MoE path uses. */
enum {
    URBO_F32 = 0,
    URBO_BF16 = 1,
    URBO_MXFP8 = 2, /* E4M3 values + E8M0 block scales (src/math/mxfp.rs:321-877) */
    URBO_MXFP4 = 3, /* packed E2M1 nibbles + E8M0 group scales (src/math/mxfp.rs:1363-1847) */
    URBO_INT8 = 4,  /* Int8Matrix: two's-complement bytes, one f32 scale per row (src/math/quant.rs:355-573) */
    URBO_INT4 = 5,  /* Int4Matrix: low-nibble-first codes (value code - 8), f32 group scales (quant.rs:28-350) */
};

enum {
    URBO_OK = 0,
    URBO_ERR_SHAPE = 1,
    URBO_ERR_INVALID_SCALE = 2,
    URBO_ERR_NONFINITE = 3,
    URBO_ERR_INVALID_GEOMETRY = 4,
    URBO_ERR_INVALID = 9,  /* DeepseekMathError::Invalid (bad hash ids, non-positive scale) */
    URBO_ERR_INVALID_GROUP = 11, /* QuantError::InvalidGroupSize (src/math/quant.rs:12) */
};

typedef struct urbo_matrix {
    int32_t format;
    size_t rows, cols;
    size_t group_size;             /* MXFP4: scale run along the input dimension */
    size_t block_rows, block_cols; /* MXFP8: scale block */
    const void *values;            /* f32 | bf16 bits (u16) | E4M3 bytes | packed nibbles */
    const uint8_t *scales;         /* E8M0 bytes (MX formats) */
    const float *fscales;          /* f32 scales (INT8: [rows]; INT4: [rows, ceil(cols/group)]) */
} urbo_matrix;

/* Codecs (src/math/mxfp.rs:44-79, 247-275). */
float urbo_decode_e8m0(uint8_t code);   /* 0xFF is not validated here */
float urbo_decode_e4m3fn(uint8_t code);
float urbo_decode_e2m1(uint8_t code);
uint8_t urbo_encode_e4m3fn(float value);
float urbo_expf(float value);           /* the libm expf the Rust reference links */

/* Constructor validation: shape, then payload (mxfp.rs:1400-1443, 394-425; quant.rs:92-131,
 * 363-396 for the INT formats). */
int urbo_validate(const urbo_matrix *m);
/* Int4Matrix::quantize_grouped (src/math/quant.rs:46-90): packed [rows, ceil(cols/2)],
 * scales [rows, ceil(cols/group)]. */
int urbo_int4_quantize_grouped(size_t rows, size_t cols, size_t group, const float *values,
                               uint8_t *packed, float *scales);
/* WeightMatrix::write_row (src/model/weight.rs:347-392): the decoded f32 weights of one row. */
int urbo_write_row(const urbo_matrix *m, size_t row, float *out);

/* WeightMatrix::matvec_rows / MxFp4Matrix::matvec_rows etc.  y has `count` entries. */
/* WeightMatrix::transpose_rows_matvec (src/model/weight.rs:332-343): y[cols] = rows
 * start..start+n of W, transposed, times x[n]; ordered f64 column sums. */
int urbo_transpose_rows_matvec(const urbo_matrix *m, size_t start, const float *x, size_t n,
                               float *y);
int urbo_matvec_rows(const urbo_matrix *m, size_t start, size_t count, const float *x, float *y,
                     int threads);
/* WeightMatrix::matmul_rows (src/model/weight.rs:106-153): x [batch, cols] -> y [batch, rows]. */
int urbo_matmul_rows(const urbo_matrix *m, const float *x, size_t batch, float *y, int threads);
/* MxFp4Matrix::matvec_rows_fp32 (src/math/mxfp.rs:1658-1723), FP32 accumulation boundary. */
int urbo_mxfp4_matvec_rows_fp32(const urbo_matrix *m, size_t start, size_t count, const float *x,
                                float *y, int threads);

/* route_noaux_tc (src/math/routing.rs:38-155).  Outputs top_k entries in selection order. */
int urbo_route_noaux_tc(const float *logits, const float *bias, size_t experts, size_t top_k,
                        size_t n_group, size_t topk_group, int normalize, float scaling,
                        int32_t *out_expert, float *out_weight, float *out_score);
/* route_softmax_top_k (src/models/qwen3_8/moe.rs:91-159). */
int urbo_route_softmax_top_k(const float *logits, size_t experts, size_t top_k,
                             int32_t *out_expert, float *out_weight);

/* silu (src/math/ops.rs:36-38) and GatedMlp::forward (src/model/mlp.rs:90-99). */
float urbo_silu(float v);
int urbo_gated_mlp_forward(const urbo_matrix *gate, const urbo_matrix *up,
                           const urbo_matrix *down, const float *x, float *y, int threads);

/* Ragged grouping: experts ascending, tokens ascending within an expert
 * (src/models/qwen3_6/runtime.rs:1083-1132).  expert_ids is [tokens, top_k] in selection
 * order.  counts/offsets have `experts` / `experts + 1` entries; perm_token / perm_slot have
 * tokens*top_k entries: the token and the selection rank of each grouped route. */
int urbo_group_routes(const int32_t *expert_ids, size_t tokens, size_t top_k, size_t experts,
                      int32_t *counts, int32_t *offsets, int32_t *perm_token, int32_t *perm_slot);

/* One GLM RuntimeMoeLayer::forward per token (src/models/glm/runtime/moe.rs:138-176):
 * BF16/any router -> route_noaux_tc -> shared GatedMlp -> routed GatedMlps in selection
 * order -> f64 combine.  x and out are [tokens, hidden]; route outputs [tokens, top_k]. */
typedef struct urbo_moe_layer {
    const urbo_matrix *router;
    const float *bias;
    size_t experts;
    const urbo_matrix *gate, *up, *down;      /* arrays of `experts` matrices */
    const urbo_matrix *shared_gate, *shared_up, *shared_down;
    size_t top_k, n_group, topk_group;
    int normalize;
    float routed_scaling_factor;
} urbo_moe_layer;

int urbo_moe_layer_forward(const urbo_moe_layer *layer, const float *x, size_t tokens,
                           float *out, int32_t *route_expert, float *route_weight,
                           float *route_score, float *router_logits, int threads);

/* Checkpoint numerics (DeepSeek-V4).  src/math/mxfp.rs:91-115 and :300-319 (E4M3 activation
 * simulation, power-of-two block scale), deepseek_v4/math.rs:90-101 (BF16 rounding) and
 * :518-549 (bounded SwiGLU), and the MoE composition of deepseek_v4/runtime.rs:2500-2700 for
 * given routes (ids / weights [tokens, top_k]; the layer's router and bias are unused). */
float urbo_power_of_two_ceiling(float value);
int urbo_simulate_e4m3_activation(float *values, size_t n, size_t block);
float urbo_round_bf16(float value);
float urbo_bounded_swiglu(float gate, float up, float limit);
/* One expert of that composition (DeepExpert::forward_with_mx_input): MX projections read mx_x
 * and round to BF16, plain ones read x; route_weight NULL for the shared expert. */
int urbo_deepseek_expert_forward(const urbo_matrix *gate, const urbo_matrix *up,
                                 const urbo_matrix *down, const float *x, const float *mx_x,
                                 const float *route_weight, float limit, float *y, int threads);
int urbo_moe_deepseek_forward(const urbo_moe_layer *layer, const float *x, size_t tokens,
                              const int32_t *route_expert, const float *route_weight,
                              float limit, float *out, int threads);
/* deepseek_v4/math.rs:451-516 route_sqrt_softplus of one row (bias, hash may be NULL), and the
 * whole DeepSeek-V4 layer forward (router + routing + the composition above). */
int urbo_route_sqrt_softplus(const float *logits, const float *bias, size_t experts,
                             const int32_t *hash, size_t top_k, float scaling, int32_t *out_expert,
                             float *out_weight, float *out_score);
int urbo_moe_deepseek_layer_forward(const urbo_moe_layer *layer, const float *x, size_t tokens,
                                    const int32_t *hash, float limit, float *out,
                                    int32_t *route_expert, float *route_weight, int threads);

/* Checkpoint numerics (Qwen3.6): src/model/bf16.rs:591-613 (FP32-lane BF16 dot),
 * src/math/mxfp.rs:122-149 (fine-grained E4M3 activation), qwen3_8/math.rs:10-26 (linear with
 * BF16 outputs), qwen3_8/expert.rs:137-200 (BF16-boundary SwiGLU) and the execute_batched_moe
 * composition of qwen3_6/runtime.rs:1067-1215 (softmax top-k, BF16 accumulation in ascending
 * expert id, sigmoid-gated shared expert).  shared_gate_vec: the [1, hidden] BF16 gate row. */
float urbo_dot_bf16_fp32_lanes(const uint16_t *row, const float *x, size_t cols);
int urbo_simulate_finegrained_e4m3(float *values, size_t n, size_t block);
int urbo_moe_qwen_layer_forward(const urbo_moe_layer *layer, const urbo_matrix *shared_gate_vec,
                                const float *x, size_t tokens, float *out, int32_t *route_expert,
                                float *route_weight, int threads);

#ifdef __cplusplus
}
#endif
#endif
