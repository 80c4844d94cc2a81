/*
 * urb_moe.h — C ABI of the B200 routed-expert (MoE) hot path.
 *
 * This is the drop-in boundary for Urbilateria's routed-expert feed-forward path.  Every entry
 * point names the reference interface it replaces (paths relative to the Urbilateria source
 * tree, v0.2.4).  The ABI is plain C: handles, host pointers, sizes and int status codes; no
 * C++ or CUDA types cross it.  A Rust `build.rs` links liburb_moe.a (built by nvcc for
 * sm_100a) and binds these symbols with `extern "C"`.
 *
 * Conventions
 *  - Weights are row-major [rows, cols]; y = W x (src/model/matrix.rs:33-38).
 *  - MXFP4: packed[row*ceil(cols/2) + col/2], even column = low nibble; one E8M0 scale per
 *    `group_size` columns: scales[row*ceil(cols/group) + col/group] (src/math/mxfp.rs:1418-1423).
 *  - MXFP8: values[row*cols + col] (E4M3FN); scales[(row/block_rows)*ceil(cols/block_cols) +
 *    col/block_cols] (src/math/mxfp.rs:434-440).
 *  - Batched inputs/outputs are token-major: x [batch, cols], y [batch, rows]
 *    (src/math/mxfp.rs:1544-1549).
 *  - Functions without a `_device` suffix take HOST pointers and return when the results are
 *    in host memory.  `_device` variants take device pointers, enqueue on the context stream
 *    and report errors through a device status word (see urb_status_*), so they can be
 *    captured in a CUDA graph.
 *  - Thread safety: a context serialises its calls with an internal mutex; use one context
 *    per host thread for concurrency.  Every call is stream-ordered on the context stream.
 *
 * Numerics: weights are decoded exactly (E2M1/E4M3 x E8M0 -> f16 with a per-row power-of-two
 * offset, BF16 kept as bf16); activations enter the tensor cores as an exact-to-2^-22 hi+lo
 * split; products are exact and accumulate in fp32.  Results match the reference's ordered-F64
 * CPU outputs to relative L2 <= 1e-3.  Router logits are computed with the reference's
 * sequential F64 order and are bit-identical; top-k indices, the token permutation and the
 * per-expert counts are bit-identical to the reference.
 */
#ifndef URB_MOE_H
#define URB_MOE_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define URB_API __attribute__((visibility("default")))
#else
#define URB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes.  1-4 mirror MxError / RouteError / MatrixError variants
 * (src/math/mxfp.rs:17-23, src/math/routing.rs:16-21, src/model/weight.rs:5-48). */
typedef enum urb_status {
    URB_OK = 0,
    URB_ERR_SHAPE = 1,             /* MxError::Shape, MatrixError::InputLength/InvalidShape */
    URB_ERR_INVALID_SCALE = 2,     /* MxError::InvalidScale (E8M0 0xFF) */
    URB_ERR_NONFINITE = 3,         /* MxError::NonFinite, RouteError::NonFinite */
    URB_ERR_INVALID_GEOMETRY = 4,  /* RouteError::InvalidGeometry */
    URB_ERR_CUDA = 5,              /* CUDA runtime failure (see urb_last_error) */
    URB_ERR_TIMEOUT = 6,           /* a bounded device wait gave up */
    URB_ERR_NCCL = 7,              /* reserved; never returned: the expert-parallel data path
                                    * runs over peer memory, and the handle exchange is the
                                    * host's (torch.distributed), whose errors it raises itself */
    URB_ERR_UNSUPPORTED = 8,       /* configuration outside what this build implements */
    URB_ERR_INVALID_ARGUMENT = 9,  /* null handle / pointer */
    URB_ERR_PEER = 10,             /* another rank of the expert-parallel group failed the forward */
    URB_ERR_INVALID_GROUP = 11,    /* QuantError::InvalidGroupSize (src/math/quant.rs:10-14) */
} urb_status;

typedef enum urb_format {
    URB_FMT_F32 = 0,   /* DenseMatrix (src/model/matrix.rs) */
    URB_FMT_BF16 = 1,  /* Bf16Matrix (src/model/bf16.rs) */
    URB_FMT_MXFP8 = 2, /* MxFp8Matrix with E8M0 scales (src/math/mxfp.rs:321) */
    URB_FMT_MXFP4 = 3, /* MxFp4Matrix (src/math/mxfp.rs:1363) */
    URB_FMT_INT8 = 4,  /* Int8Matrix: two's-complement bytes, f32 scale per row (src/math/quant.rs:355) */
    URB_FMT_INT4 = 5,  /* Int4Matrix: low-nibble-first codes (code - 8), f32 group scales (quant.rs:33) */
} urb_format;

typedef struct urb_ctx urb_ctx;
typedef struct urb_mat urb_mat;
typedef struct urb_layer urb_layer;

/* ---- context ---------------------------------------------------------------------------- */

/* Creates a context on CUDA `device` with its own stream.  Replaces the process-wide Rayon
 * pool set-up `configure_threads` (src/execution.rs:59). */
URB_API int urb_ctx_create(int device, urb_ctx **out);
URB_API int urb_ctx_destroy(urb_ctx *ctx);
/* Use the caller's cudaStream_t (passed as void*) instead of the context stream. */
URB_API int urb_ctx_set_stream(urb_ctx *ctx, void *cuda_stream);
URB_API void *urb_ctx_stream(urb_ctx *ctx);
/* Copies the last error message (NUL-terminated) into buf; returns the status it belongs to. */
URB_API int urb_last_error(urb_ctx *ctx, char *buf, size_t len);
/* Waits for all work on the context stream. */
URB_API int urb_ctx_synchronize(urb_ctx *ctx);

/* ---- weight matrices (resident in HBM) --------------------------------------------------- */

/* MxFp4Matrix::from_packed (src/math/mxfp.rs:1371-1443): validates shape (Shape) and every
 * scale (InvalidScale for 0xFF), then keeps the matrix resident on the device.  `packed` and
 * `scales` may be host or device pointers. */
URB_API int urb_mxfp4_upload(urb_ctx *ctx, size_t rows, size_t cols, size_t group_size,
                     const uint8_t *packed, size_t packed_len, const uint8_t *scales,
                     size_t scales_len, urb_mat **out);
/* MxFp8Matrix::from_packed (src/math/mxfp.rs:331-425): E4M3 NaN codes -> NonFinite,
 * 0xFF scales -> InvalidScale. */
URB_API int urb_mxfp8_upload(urb_ctx *ctx, size_t rows, size_t cols, size_t block_rows,
                     size_t block_cols, const uint8_t *values, size_t values_len,
                     const uint8_t *scales, size_t scales_len, urb_mat **out);
/* Bf16Matrix::from_le_bytes-style constructor (src/model/bf16.rs): bits as little-endian u16. */
URB_API int urb_bf16_upload(urb_ctx *ctx, size_t rows, size_t cols, const uint16_t *values,
                    size_t values_len, urb_mat **out);
/* DenseMatrix::new (src/model/matrix.rs). */
URB_API int urb_f32_upload(urb_ctx *ctx, size_t rows, size_t cols, const float *values,
                   size_t values_len, urb_mat **out);
/* Int8Matrix::from_packed (src/math/quant.rs:363-396): bytes [rows, cols], one f32 scale per
 * row.  Shape (zero dimensions, payload or scale counts), then NonFinite for a scale that is not
 * finite and positive.  Host or device pointers.  WeightMatrix::Int8PerRow (weight.rs:57). */
URB_API int urb_int8_upload(urb_ctx *ctx, size_t rows, size_t cols, const uint8_t *bytes,
                            size_t bytes_len, const float *scales, size_t scales_len, urb_mat **out);
/* Int4Matrix::from_packed (src/math/quant.rs:92-131): packed [rows, ceil(cols/2)] low nibble
 * first, f32 scales [rows, ceil(cols/group_size)].  InvalidGroup for group_size 0, Shape, then
 * NonFinite for a scale that is not finite and positive.  WeightMatrix::Int4 (weight.rs:58). */
URB_API int urb_int4_upload(urb_ctx *ctx, size_t rows, size_t cols, size_t group_size,
                            const uint8_t *packed, size_t packed_len, const float *scales,
                            size_t scales_len, urb_mat **out);
/* Int4Matrix::quantize_grouped (src/math/quant.rs:46-90; quantize_per_row is group_size ==
 * cols): quantises f32 values [rows, cols] on the device, bit-exact with the reference, and
 * keeps the result resident.  InvalidGroup, Shape, then NonFinite for a non-finite value. */
URB_API int urb_int4_quantize_grouped(urb_ctx *ctx, size_t rows, size_t cols, size_t group_size,
                                      const float *values, size_t values_len, urb_mat **out);
/* Int4Matrix packed()/scales() (quant.rs:145-151): copies the resident payload out (host or
 * device pointers, sizes as in urb_int4_upload).  URB_ERR_UNSUPPORTED for other formats. */
URB_API int urb_int4_payload(urb_ctx *ctx, const urb_mat *mat, uint8_t *packed, float *scales);
URB_API int urb_mat_free(urb_mat *mat);
/* WeightMatrix::{rows, cols, resident_bytes} (src/model/weight.rs:69-90, 306-320).
 * resident_bytes counts the payload bytes of the reference format. */
URB_API int urb_mat_info(const urb_mat *mat, int *format, size_t *rows, size_t *cols,
                 size_t *resident_bytes);

/* ---- matrix-level products ---------------------------------------------------------------- */

/* WeightMatrix::matvec_rows (src/model/weight.rs:155-203; MxFp4Matrix::matvec_rows
 * src/math/mxfp.rs:1725-1780): y[0..count) = W[start..start+count) x.  Errors: Shape (bad row
 * range), NonFinite (non-finite input; for MXFP8 also non-finite output, mxfp.rs:712). */
URB_API int urb_matvec_rows(urb_ctx *ctx, const urb_mat *mat, size_t start, size_t count,
                    const float *x, size_t x_len, float *y);
/* WeightMatrix::matmul_rows (src/model/weight.rs:106-153): x [batch, cols] -> y [batch, rows],
 * including the reference's output-finiteness rule for its <=12-token chunks. */
URB_API int urb_matmul_rows(urb_ctx *ctx, const urb_mat *mat, const float *x, size_t batch,
                    size_t x_len, float *y);
/* WeightMatrix::matmul_row_range (src/model/weight.rs:155-203). */
URB_API int urb_matmul_row_range(urb_ctx *ctx, const urb_mat *mat, size_t start, size_t count,
                         const float *x, size_t batch, size_t x_len, float *y);
/* WeightMatrix::{matvec_fp32_accum, matmul_rows_fp32_accum} (src/model/weight.rs:205-303):
 * the FP32-accumulation boundary of DeepSeek-V4.1.  Same device arithmetic (fp32 accumulate). */
URB_API int urb_matmul_rows_fp32_accum(urb_ctx *ctx, const urb_mat *mat, const float *x, size_t batch,
                               size_t x_len, float *y);
/* Device-pointer form: d_x [batch, cols] f32 -> d_y [batch, rows] f32, stream-ordered.
 * d_status (device int32, may be NULL) receives URB_ERR_NONFINITE if an input is non-finite. */
URB_API int urb_matmul_rows_device(urb_ctx *ctx, const urb_mat *mat, const float *d_x, size_t batch,
                           float *d_y, int32_t *d_status);

/* GatedMlp::forward (src/model/mlp.rs:90-99) for `tokens` rows: down(silu(gate x) * (up x)).
 * x, out [tokens, hidden] f32 host pointers. */
URB_API int urb_gated_mlp_forward(urb_ctx *ctx, const urb_mat *gate, const urb_mat *up,
                                  const urb_mat *down, const float *x, size_t tokens, float *out);
URB_API int urb_gated_mlp_forward_device(urb_ctx *ctx, const urb_mat *gate, const urb_mat *up,
                                         const urb_mat *down, const float *d_x, size_t tokens,
                                         float *d_out, int32_t *d_status);
/* urb_gated_mlp_forward_device without any allocation (no counterpart in the reference, whose
 * CPU path allocates per call).  For callers that cannot allocate device memory while they
 * run: serving loops that reserve all free HBM up front, and per-token decode loops where a
 * cudaMalloc would synchronise the device.  Temporaries live in one static 8 MiB device
 * scratch per device; calls needing more are rejected (URB_ERR_UNSUPPORTED), roughly
 * tokens * intermediate * 4 bytes must fit.  Projections must share one tiled format (MXFP4 /
 * MXFP8 with 32-column groups, or BF16); F32, INT8 / INT4 and mixed-format MLPs are rejected
 * with URB_ERR_UNSUPPORTED (their per-projection path needs a workspace).  The first call on a
 * context resolves the scratch's device address (set-up; make it before any stream capture).
 * Calls overlapping in time on one device race on the scratch: serialise them. */
URB_API int urb_gated_mlp_forward_device_noalloc(urb_ctx *ctx, const urb_mat *gate,
                                                 const urb_mat *up, const urb_mat *down,
                                                 const float *d_x, size_t tokens, float *d_out,
                                                 int32_t *d_status);

/* ---- routing -------------------------------------------------------------------------------- */

/* MoeGeometry (src/models/glm/moe_geometry.rs:1-9). */
typedef struct urb_moe_geometry {
    uint32_t top_k;
    uint32_t n_group;
    uint32_t topk_group;
    int32_t normalize;
    float routed_scaling_factor;
} urb_moe_geometry;

/* route_noaux_tc (src/math/routing.rs:38-155) for `tokens` rows of logits [tokens, experts].
 * Outputs [tokens, top_k] in selection order: expert ids, weights, selection scores (NULL ok). */
URB_API int urb_route_noaux_tc(urb_ctx *ctx, const float *logits, const float *bias, size_t tokens,
                       size_t experts, const urb_moe_geometry *geometry, int32_t *out_expert,
                       float *out_weight, float *out_score);
/* route_softmax_top_k (src/models/qwen3_8/moe.rs:91-159). */
URB_API int urb_route_softmax_top_k(urb_ctx *ctx, const float *logits, size_t tokens, size_t experts,
                            uint32_t top_k, int32_t *out_expert, float *out_weight);
/* Ragged token->expert grouping (src/models/qwen3_6/runtime.rs:1083-1132): experts ascending,
 * tokens ascending within an expert.  expert_ids [tokens, top_k]; outputs counts [experts],
 * offsets [experts+1], perm_token / perm_slot [tokens*top_k]. */
URB_API int urb_group_routes(urb_ctx *ctx, const int32_t *expert_ids, size_t tokens, uint32_t top_k,
                     size_t experts, int32_t *counts, int32_t *offsets, int32_t *perm_token,
                     int32_t *perm_slot);

/* ---- MoE layer ------------------------------------------------------------------------------ */

/* RuntimeMoeLayer::new (src/models/glm/runtime/moe.rs:88-129): router [experts, hidden],
 * correction bias [experts], per-expert gate/up [inter, hidden] and down [hidden, inter]
 * matrices, optional shared expert (NULL for none), geometry.  The layer references the
 * matrices; they must outlive it. */
URB_API int urb_moe_layer_create(urb_ctx *ctx, const urb_mat *router, const float *bias, size_t experts,
                         const urb_mat *const *gate, const urb_mat *const *up,
                         const urb_mat *const *down, const urb_mat *shared_gate,
                         const urb_mat *shared_up, const urb_mat *shared_down,
                         const urb_moe_geometry *geometry, urb_layer **out);
URB_API int urb_moe_layer_free(urb_layer *layer);

/* RuntimeMoeLayer::forward (src/models/glm/runtime/moe.rs:138-176), batched over `tokens`
 * (one call per MoE layer, not per projection).  x, out [tokens, hidden] f32 host pointers.
 * Optional outputs (NULL to skip): route expert/weight/score [tokens, top_k] in selection
 * order, router logits [tokens, experts], counts [experts], perm_token/perm_slot
 * [tokens*top_k] (the grouped order of src/models/qwen3_6/runtime.rs:1123-1132). */
URB_API int urb_moe_forward(urb_ctx *ctx, urb_layer *layer, const float *x, size_t tokens, float *out,
                    int32_t *route_expert, float *route_weight, float *route_score,
                    float *router_logits, int32_t *counts, int32_t *perm_token,
                    int32_t *perm_slot);
/* Device-pointer form of urb_moe_forward (inputs resident in HBM, stream-ordered, no host
 * synchronisation; graph-capturable).  d_status as in urb_matmul_rows_device. */
URB_API int urb_moe_forward_device(urb_ctx *ctx, urb_layer *layer, const float *d_x, size_t tokens,
                           float *d_out, int32_t *d_route_expert, float *d_route_weight,
                           int32_t *d_status);

/* The experts half of the layer forward for routes chosen by the caller (route_softmax_top_k of
 * src/models/qwen3_8/moe.rs:91-159, DeepSeek hash routing, routes replayed from a trace): the
 * ragged grouping and grouped SwiGLU experts of execute_batched_moe
 * (src/models/qwen3_6/runtime.rs:1098-1148) with the GLM combine (f64 in the given route
 * order, shared expert ungated; src/models/glm/runtime/moe.rs:164-175).  route_expert /
 * route_weight [tokens, top_k]; ids outside [0, experts) are URB_ERR_SHAPE. */
URB_API int urb_moe_forward_routed(urb_ctx *ctx, urb_layer *layer, const float *x, size_t tokens,
                                   const int32_t *route_expert, const float *route_weight,
                                   float *out);
URB_API int urb_moe_forward_routed_device(urb_ctx *ctx, urb_layer *layer, const float *d_x,
                                          size_t tokens, const int32_t *d_route_expert,
                                          const float *d_route_weight, float *d_out,
                                          int32_t *d_status);

/* WeightMatrix::transpose_rows_matvec (src/model/weight.rs:332-343; mxfp.rs:785-858 for MXFP8,
 * :1782-1821 for MXFP4, bf16.rs:430-475, matrix.rs:276-313): y[cols] = rows start..start+n of the
 * matrix, transposed, times x[n] (host pointers), bit-exact: each column is the ordered f64 sum
 * of the exact products, rounded to f32.  URB_ERR_NONFINITE for a non-finite x (checked first),
 * URB_ERR_SHAPE when start + n exceeds the rows; MXFP8 also rejects non-finite outputs. */
URB_API int urb_transpose_rows_matvec(urb_ctx *ctx, const urb_mat *mat, size_t start,
                                      const float *x, size_t n, float *y);
/* WeightMatrix::write_row / row (src/model/weight.rs:347-392; quant.rs:163-182, 414-436,
 * mxfp.rs:860-875, 1828-1845, bf16.rs:88-113): the decoded f32 weights of rows start..start+count into out
 * [count, cols] (host pointer), every format.  Shape when the range exceeds the rows. */
URB_API int urb_mat_write_rows(urb_ctx *ctx, const urb_mat *mat, size_t start, size_t count,
                               float *out);

/* ---- checkpoint numerics ---------------------------------------------------------------------- */

/* Numerics of the routed forward.  URB_NUMERICS_GLM: the GLM composition above.
 * URB_NUMERICS_DEEPSEEK_V4: DeepExpert::forward_with_mx_input and MoeWeights::forward
 * (src/models/deepseek_v4/runtime.rs:3081-3104, :2500-2650) for MX experts: the input simulated
 * as E4M3 per 128 values (src/math/mxfp.rs:91-115), gate / up outputs rounded to BF16, bounded
 * SwiGLU with `swiglu_limit` (deepseek_v4/math.rs:518-549), the route weight applied to the
 * activation before BF16 rounding, E4M3 simulation and the down projection (none for the shared
 * expert), down outputs rounded to BF16, routed rows summed in f32 in ascending expert id, the
 * shared row added last and the sum rounded to BF16.  Route weights must be finite and
 * non-negative (URB_ERR_INVALID_ARGUMENT otherwise).
 * URB_NUMERICS_QWEN36: execute_batched_moe (src/models/qwen3_6/runtime.rs:1067-1215) over
 * Qwen36Expert / linear (src/models/qwen3_8/math.rs:10-26): BF16 experts take the FP32-lane BF16
 * dot (src/model/bf16.rs:591-613), MX experts see the input simulated as E4M3 with the exact
 * per-128 scale max|v| / 448 (src/math/mxfp.rs:122-149); every projection output rounds to BF16;
 * h = BF16(BF16(silu(gate)) * up); routed contributions BF16(BF16(w) * y) accumulate in BF16 in
 * ascending expert id; the shared expert adds BF16(BF16(sigmoid(g)) * y) with g the BF16 logit of
 * the layer's shared_expert_gate row (urb_moe_layer_set_shared_expert_gate, required).  Needs a
 * BF16 router and a shared expert; `swiglu_limit` is unused. */
#define URB_NUMERICS_GLM 0
#define URB_NUMERICS_DEEPSEEK_V4 1
#define URB_NUMERICS_QWEN36 2
typedef struct urb_moe_numerics {
    int32_t mode;
    float swiglu_limit;
} urb_moe_numerics;
URB_API int urb_moe_forward_routed_ex(urb_ctx *ctx, urb_layer *layer, const float *x,
                                      size_t tokens, const int32_t *route_expert,
                                      const float *route_weight, const urb_moe_numerics *numerics,
                                      float *out);
URB_API int urb_moe_forward_routed_ex_device(urb_ctx *ctx, urb_layer *layer, const float *d_x,
                                             size_t tokens, const int32_t *d_route_expert,
                                             const float *d_route_weight,
                                             const urb_moe_numerics *numerics, float *d_out,
                                             int32_t *d_status);
/* The whole layer forward with checkpoint numerics.  URB_NUMERICS_GLM: urb_moe_forward.
 * URB_NUMERICS_DEEPSEEK_V4: MoeWeights::forward (src/models/deepseek_v4/runtime.rs:2484-2700):
 * exact router logits, route_sqrt_softplus (deepseek_v4/math.rs:451-516) with the layer's
 * correction bias and routed_scaling_factor, or the token's fixed experts `hash_experts`
 * ([tokens, top_k], NULL for learned routing; the weights still come from the scores), then the
 * routed experts with the DeepSeek-V4 numerics above.  URB_NUMERICS_QWEN36 (execute_batched_moe,
 * src/models/qwen3_6/runtime.rs:1067-1215): BF16 router logits (FP32 lanes), route_softmax_top_k
 * with the weights rounded to BF16, then the Qwen3.6 numerics above (hash_experts must be NULL).
 * Routes out in selection order (NULL to skip). */
URB_API int urb_moe_forward_ex(urb_ctx *ctx, urb_layer *layer, const float *x, size_t tokens,
                               const urb_moe_numerics *numerics, const int32_t *hash_experts,
                               float *out, int32_t *route_expert, float *route_weight);
/* route_sqrt_softplus (src/models/deepseek_v4/math.rs:451-516) for `tokens` rows of logits:
 * score = sqrt(softplus(logit)) with libm expf / log1pf, selection = score + bias (bias NULL:
 * none), top_k by selection (lower id wins ties) or the given hash experts, weight = score /
 * sum(chosen scores) * routed_scaling_factor.  Outputs [tokens, top_k]; out_score (the
 * selection score) may be NULL. */
URB_API int urb_route_sqrt_softplus(urb_ctx *ctx, const float *logits, const float *bias,
                                    size_t tokens, size_t experts, const int32_t *hash_experts,
                                    uint32_t top_k, float routed_scaling_factor,
                                    int32_t *out_expert, float *out_weight, float *out_score);
/* simulate_e4m3_activation (src/math/mxfp.rs:82-115) of n values in blocks of `block` (host
 * pointers): each block scaled by the power of two at or above max(|v|, 1e-4) / 448 and
 * round-tripped through E4M3FN. */
URB_API int urb_simulate_e4m3_activation(urb_ctx *ctx, const float *x, size_t n, size_t block,
                                         float *out);
/* simulate_finegrained_e4m3_activation (src/math/mxfp.rs:122-149): each block scaled by exactly
 * max|v| / 448 and round-tripped through E4M3FN; all-zero blocks stay zero. */
URB_API int urb_simulate_finegrained_e4m3_activation(urb_ctx *ctx, const float *x, size_t n,
                                                     size_t block, float *out);
/* The Qwen3.6 BF16 linear (src/models/qwen3_8/math.rs:10-26 with dot_bf16_fp32_avx2_fma,
 * src/model/bf16.rs:591-613) of `tokens` rows of x [tokens, cols] by a BF16 matrix [rows, cols]:
 * out [tokens, rows] = BF16(eight FP32 FMA lanes, lanes summed in order, tail added), bit-exact.
 * URB_ERR_NONFINITE when an output is not finite. */
URB_API int urb_linear_bf16_fp32_lanes(urb_ctx *ctx, const urb_mat *m, const float *x,
                                       size_t tokens, float *out);

/* ---- expert parallelism across the GPUs of one node ------------------------------------------ */

/* The layer forward of src/models/glm/runtime/moe.rs:138-176 split by experts over `world`
 * processes, one per GPU (the reference runs every expert in one process; its Rayon workers
 * split rows, src/execution.rs:154).  Rank g holds routed experts [expert_begin,
 * expert_begin + expert_count) plus the replicated router and shared expert, and owns the
 * tokens it passes to urb_ep_forward*.  Token rows and expert outputs move between the GPUs
 * through peer memory (NVLink / NVSwitch) inside the kernels; outputs are bit-identical to
 * urb_moe_forward on one GPU. */
#define URB_EP_MAX_WORLD 8
#define URB_EP_HANDLE_BYTES 256
typedef struct urb_ep urb_ep;

/* A shard of RuntimeMoeLayer::new (src/models/glm/runtime/moe.rs:88-129): router [experts,
 * hidden] and bias [experts] for all experts; gate/up/down arrays hold the `expert_count`
 * experts starting at `expert_begin`.  Runs only through urb_ep_forward*; urb_moe_forward*
 * return URB_ERR_UNSUPPORTED for it.  Needs MX (MXFP4 / MXFP8 1x32) experts. */
/* Qwen3.6 shared_expert_gate (src/models/qwen3_6/runtime.rs:1176-1213): a [1, hidden] BF16 matrix
 * whose BF16 logit gates the shared expert under URB_NUMERICS_QWEN36.  The matrix must outlive the
 * layer; NULL detaches it. */
URB_API int urb_moe_layer_set_shared_expert_gate(urb_ctx *ctx, urb_layer *layer, const urb_mat *gate);
URB_API int urb_moe_layer_create_sharded(urb_ctx *ctx, const urb_mat *router, const float *bias,
                                         size_t experts, size_t expert_begin, size_t expert_count,
                                         const urb_mat *const *gate, const urb_mat *const *up,
                                         const urb_mat *const *down, const urb_mat *shared_gate,
                                         const urb_mat *shared_up, const urb_mat *shared_down,
                                         const urb_moe_geometry *geometry, urb_layer **out);
/* This rank's member of an expert-parallel group over `layer` (a shard, or the whole layer
 * when world == 1).  max_tokens bounds the tokens any rank passes per forward; timeout_ms (0:
 * 5000) bounds every wait of a group barrier on the device. */
URB_API int urb_ep_create(urb_ctx *ctx, urb_layer *layer, int world, int rank, size_t max_tokens,
                          uint32_t timeout_ms, urb_ep **out);
/* Writes URB_EP_HANDLE_BYTES describing this rank's exchange window (a CUDA IPC handle plus
 * the group geometry) for the caller to all-gather over its host-side process group. */
URB_API int urb_ep_export(urb_ep *ep, uint8_t *handle);
/* Maps the other ranks' windows.  handles: world * URB_EP_HANDLE_BYTES in rank order.  Checks
 * that every rank describes the same group, that the expert ranges tile [0, experts) and that
 * no two ranks share a GPU (URB_ERR_UNSUPPORTED: the group's barriers need distinct GPUs). */
URB_API int urb_ep_connect(urb_ep *ep, const uint8_t *handles);
/* One forward of this rank's `tokens` (<= max_tokens, 0 allowed) tokens; collective: every
 * rank of the group calls it for every forward, in the same order.  Host pointers; outputs
 * as urb_moe_forward (out [tokens, hidden], optional route expert / weight [tokens, top_k]).
 * A rank that fails a forward fails it on every rank (URB_ERR_PEER on the others); a rank
 * that does not call it leaves the others with URB_ERR_TIMEOUT. */
URB_API int urb_ep_forward(urb_ctx *ctx, urb_ep *ep, const float *x, size_t tokens, float *out,
                           int32_t *route_expert, float *route_weight);
/* Device-pointer form (stream-ordered, no host synchronisation).  d_status is required. */
URB_API int urb_ep_forward_device(urb_ctx *ctx, urb_ep *ep, const float *d_x, size_t tokens,
                                  float *d_out, int32_t *d_route_expert, float *d_route_weight,
                                  int32_t *d_status);
URB_API int urb_ep_free(urb_ep *ep);

/* ---- measurement -------------------------------------------------------------------------- */

/* Kernel families timed by the optional per-launch profiler (CUDA events on the launch
 * stream, around each launch; off by default).  Replaces the reference's ProfileStage spans
 * (src/profiling.rs:75-136) for the device path. */
typedef enum urb_kernel_kind {
    URB_K_ROW_SHIFT = 0,
    URB_K_ROUTER_LOGITS = 1,
    URB_K_ROUTE = 2,
    URB_K_PERMUTE = 3,
    URB_K_GATE_UP = 4,
    URB_K_DOWN = 5,
    URB_K_COMBINE = 6,
    URB_K_PRODUCT = 7,
    URB_K_PREP = 8,         /* activation residual terms of a tensor-core pass */
    URB_K_GROUP_BUILD = 9,  /* device-side group / unit tables of the tensor-core passes */
    URB_K_EXCHANGE = 10,    /* expert-parallel publish, route gather and group barriers */
    URB_K_COUNT = 11
} urb_kernel_kind;
URB_API int urb_profile_enable(urb_ctx *ctx, int on);
/* Synchronises pending events; returns the total device time and launch count of `kind`. */
URB_API int urb_profile_read(urb_ctx *ctx, int kind, double *total_ms, int64_t *launches);
URB_API int urb_profile_reset(urb_ctx *ctx);

/* Device status helpers for the `_device` forms. */
URB_API int urb_status_read(urb_ctx *ctx, const int32_t *d_status, int32_t *out);

#ifdef __cplusplus
}
#endif
#endif /* URB_MOE_H */
