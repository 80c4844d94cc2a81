// urb_tc.cuh — shared definitions of the block-scaled tensor-core (tcgen05) grouped pass.
//
// Weights stay in their MX encoding all the way into the tensor core: kind::mxf4 for MXFP4
// (E2M1 x E2M1) and kind::mxf8f6f4 for MXFP8 (E4M3 x E4M3), each with E8M0 scales per 32
// columns.  Activations are written as residual terms in the same element format (x ~= t0 +
// t1 + ..., each term with its own E8M0 scale per 32 columns): 6 E2M1 terms in 8 MMA rows per
// token for MXFP4, 4 E4M3 terms in 4 rows for MXFP8; the epilogue sums a token's terms.
// BF16 weights run kind::f16 (BF16 x BF16): their 128 x 64 tiles come straight from the
// row-major matrix through a TMA tensor map (128-byte swizzle), and an f32 activation is
// three BF16 terms (hi, mid, lo; their sum is the f32 value exactly) in 4 MMA rows.
#pragma once
#include "urb_internal.cuh"

namespace urb {

constexpr int kBsIssuers = 2;  // MMA issuing threads of the grouped kernel, one accumulator each
// MMA N of a full sub-segment: the issuers' accumulators and 8 scale slots fill 512 TMEM columns.
constexpr int kBsNmax = kBsIssuers == 2 ? 128 : 96;
// MMA rows per token, residual terms per token, tokens per sub-segment.
__host__ __device__ constexpr int bs_rows_per_tok(int fmt) { return fmt == URB_FMT_MXFP4 ? 8 : 4; }
__host__ __device__ constexpr int bs_terms(int fmt) {
    return fmt == URB_FMT_MXFP4 ? 6 : (fmt == URB_FMT_MXFP8 ? 4 : 3);
}
__host__ __device__ constexpr int bs_cap(int fmt) { return kBsNmax / bs_rows_per_tok(fmt); }

// Bytes of one 128-row x 128-byte tile of the bs layout: payload (128-byte swizzled K-major)
// followed by the scale chunks (512 B each, 4 scale columns of 128 rows).
__host__ __device__ constexpr int bs_sf_chunks(int fmt) {
    return fmt == URB_FMT_MXFP4 ? 2 : (fmt == URB_FMT_MXFP8 ? 1 : 0);
}
__host__ __device__ constexpr int bs_tile_bytes(int fmt) { return 16384 + 512 * bs_sf_chunks(fmt); }
// Input columns per K stage (one 128-byte row of payload).
__host__ __device__ constexpr int bs_stage_cols(int fmt) {
    return fmt == URB_FMT_MXFP4 ? 256 : (fmt == URB_FMT_MXFP8 ? 128 : 64);
}
// Bytes of one activation stage of n MMA rows (n <= kBsNmax): payload then scale chunks.
__host__ __device__ constexpr int bs_bstage_bytes(int fmt, int n) { return n * 128 + 512 * bs_sf_chunks(fmt); }

// One group of a bs pass: a matrix applied to one run of activation columns.  Its units are
// (128-row tile mt, sub-segment j) pairs, j fastest, so the sub-segments of a large group read
// the same weight tile back to back (the second read is served by L2).
struct TcSeg {
    const uint8_t *w;     // bs tiles of the matrix (gate/up pass: the gate projection); BF16:
                          // the matrix's tensor map (tc_src)
    const uint8_t *w2;    // gate/up pass: bs tiles (BF16: tensor map) of the up projection
    long long b_off;      // byte offset of the group's activation stages in the B buffer
    int mts, ks;          // 128-row tiles, K stages
    int rows, cols;       // real rows / input columns
    int col_begin, ntok;  // activation columns
    int nsub;             // sub-segments of bs_cap(fmt) tokens
    int unit_begin;       // prefix of mts * nsub over preceding groups
    int out_off;          // column offset of this group's outputs within an output row
    int pad;
};

// Where the MMA rows of one activation column live: its sub-segment's first stage (byte offset
// in the B buffer; stage ks at base + ks * bs_bstage_bytes(fmt, n)), its token slot, and the
// sub-segment's MMA N.
struct BsSlot {
    long long base;
    int slot, n;
};

struct TcArgs {
    const TcSeg *segs;
    const int *nsegs;
    const int *total_units;
    const int *unit_group;     // [total units] group of each work unit
    uint8_t *bbuf;             // activation stages (written by the prep kernel)
    // Prep: source rows (row-major f32), each written to the activation columns that use it.
    // Gate/up pass: src = x, row t feeds columns inv[t * top_k + k] and, with a shared expert,
    // shared_col0 + t.  Down pass (inv == nullptr): src row c = h of column c (or, with
    // swiglu, [gate | up] of column c and h = silu(gate) * up), feeding column c.
    const float *src;
    int src_stride;
    int nrows;                 // source rows
    int cols, ks;              // input columns and K stages of the pass
    int swiglu;
    const int32_t *inv;        // gate/up: inv[r * top_k + k] < 0 marks a route held elsewhere
    int top_k, shared_col0;    // shared_col0 < 0: no shared expert
    int shared_row0, shared_rows;  // source rows [shared_row0, +shared_rows) feed the shared
                                   // expert's columns shared_col0 + (r - shared_row0)
    const BsSlot *slots;       // [activation columns]
    // pair = 1 (gate/up pass): each group pairs the gate and up tiles of one expert and the
    // epilogue writes h = silu(gate) * up rows to `out` (row = activation column).
    // pair = 2 (down pass): each unit pairs neighbouring row tiles mt, mt + 1 of its matrix
    // (the group's units then count ceil(mts / 2) tiles each).
    int pair;
    // Checkpoint numerics (0: GLM f32 path).  1 (DeepSeek-V4): the prep simulates E4M3 per 128
    // columns with a power-of-two scale (sim128 = 1) before building terms; the gate/up
    // epilogue rounds gate and up to BF16, applies bounded SwiGLU (limit), multiplies by the
    // column's route weight (col_w) and rounds h to BF16; the down epilogue rounds its outputs
    // to BF16.  2 (Qwen3.6): the prep simulates E4M3 per 128 columns with the exact scale
    // max|v| / 448 (sim128 = 2); the gate/up epilogue writes h = BF16(BF16(silu(BF16(gate)))
    // * BF16(up)) with the libm expf (expf); the down epilogue rounds to BF16.  Non-finite h
    // or outputs set status.
    int variant, sim128;
    // MXFP4: 1 -> every MMA row of a token carries a residual term (8 instead of 6, about 22
    // instead of 17 bits of each activation), for numerics whose BF16 boundaries magnify
    // small differences.  MXFP8 always uses all its rows.
    int full_terms;
    float limit;
    const float *col_w;
    ExpfTable expf;
    float *out;
    int out_stride;
    int32_t *status;
    // Expert-parallel shard (all null / 0 on one GPU).  Gate/up: source row r is row
    // r % rows_per_rank of rank r / rows_per_rank's activations src_ranks[...].  Down: columns
    // [*nvalid, routed_cols) carry no route; routed column c holds route i = out_rows[c] of
    // the owning rank's tokens, written to row i % out_rank_rows of out_ranks[i / out_rank_rows]
    // (the owner's memory); the shared expert's column c goes to row c - routed_cols of `out`.
    const float *const *src_ranks;
    int rows_per_rank;
    const int32_t *nvalid;
    int routed_cols;
    const int32_t *out_rows;
    float *const *out_ranks;
    int out_rank_rows;
    int skip_prep;             // the activation stages were written by an earlier prep launch
};

// Prep (activation terms) + tensor-core pass over every group of the launch; the profiler
// records the prep as URB_K_PREP and the pass as `kind`.
int launch_tc_grouped(Ctx *ctx, int fmt, const TcArgs &a, int kind, cudaStream_t st);
// The prep (activation terms) of a pass alone.
int launch_tc_prep(Ctx *ctx, int fmt, const TcArgs &a, cudaStream_t st);
int repack_tc(Ctx *ctx, Mat *m, cudaStream_t st);

}  // namespace urb
