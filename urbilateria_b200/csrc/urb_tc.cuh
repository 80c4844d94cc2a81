// urb_tc.cuh — shared definitions of the tensor-core (tcgen05) grouped pass.
#pragma once
#include "urb_internal.cuh"

namespace urb {

// Bytes of one 128x64 tile of the tc layout (payload + 256 B of scales).
__host__ __device__ constexpr int tc_tile_bytes(int fmt) {
    return fmt == URB_FMT_MXFP4 ? 128 * 32 + 256 : 128 * 64 + 256;
}

// One segment of a tensor-core pass: a matrix (or gate/up pair) applied to a run of
// activation columns; its work units are its 128-row tiles.
struct TcSeg {
    const uint8_t *a;     // tc tiles of the (gate) matrix
    const uint8_t *b;     // tc tiles of the up matrix (pairs) or nullptr
    const int8_t *ra;     // row exponent offsets of a (>= mts*128 entries)
    const int8_t *rb;
    long long b_off;      // byte offset of this segment's activation tiles in the B buffer
    int mts, ks;          // 128-row tiles, 64-column stages
    int rows, cols;       // real rows / input columns
    int col_begin, ntok;  // activation columns
    int npad, rowsper;    // MMA N (multiple of 16) and activation rows per token (1 or 2)
    int unit_begin;       // prefix of mts over preceding segments
    int pad;
};

struct TcArgs {
    const TcSeg *segs;
    const int *nsegs;
    const int *total_units;
    int nmax;                  // largest npad of the launch (shared-memory sizing)
    int stages_a;              // weight ring depth (set by the launcher)
    uint8_t *bbuf;             // activation tiles (written by the prep kernel)
    const float *src;          // activation rows f32
    int src_stride;
    const int32_t *col_src;    // activation column -> src row (nullptr: identity)
    const int32_t *src_shift;  // explicit power-of-two shift per src row, or
    const int32_t *src_maxexp; // ilogb(max|row|) per src row (-1000: zero row)
    float *out;
    int out_stride;
    int32_t *out_maxexp;
    int32_t *status;
};

// Prep (activation tiles) + tensor-core pass.
int launch_tc_grouped(Ctx *ctx, int fmt, bool pair, const TcArgs &a, int max_segs, int max_ks,
                      cudaStream_t st);
int repack_tc(Ctx *ctx, Mat *m, cudaStream_t st);

}  // namespace urb
