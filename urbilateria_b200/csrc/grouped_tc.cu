// grouped_tc.cu — tensor-core (tcgen05 / TMEM) grouped pass for MX weights.
//
// One persistent CTA per SM walks work units (segment, 128-row tile).  Per 64-column K stage:
//   * warp 0 (producer): bulk-copies (TMA engine, 1-D) the raw MX tile(s) of the stage and the
//     segment's activation tile (pre-swizzled f16, 128-byte canonical K-major layout) into a
//     shared-memory ring;
//   * warps 4..11 (decoders): each thread owns one weight row (its TMEM lane); it decodes
//     32 E2M1 or E4M3 values with cvt.rn.f16x2.{e2m1x2,e4m3x2}, applies the E8M0 scale with one
//     HMUL2 per pair (exact: powers of two within the row's f16 window) and stores the 16
//     f16x2 words into TMEM with tcgen05.st;
//   * warp 1 (one thread): tcgen05.mma kind::f16, A from TMEM, B from the shared-memory
//     descriptor, f32 accumulators in TMEM; tcgen05.commit releases the stage.
// After the last stage the decoders read the accumulators back (tcgen05.ld), undo the
// power-of-two scalings, fuse SwiGLU for gate/up pairs, and store token-major rows.
//
// Tile layout of a resident MX matrix ("tc layout"): tiles of 128 rows x 64 columns, tile
// (mt, ks) at ((mt * KS + ks) * TB); inside a tile, payload [chunk][row 0..127][16 B] then
// scales [row][2] (E8M0 of columns 0-31 and 32-63).  MXFP4: 2 chunks (TB = 4352 B),
// MXFP8: 4 chunks (TB = 8448 B).
#include "tc_common.cuh"
#include "urb_internal.cuh"
#include "urb_tc.cuh"

namespace urb {
namespace {

// Rings: raw weight tiles (deep: the HBM stream), activation tiles, TMEM A stages.
constexpr int kStagesAMax = 12;  // weight ring depth (runtime: as many as shared memory holds)
constexpr int kStagesB = 4;
constexpr int kStagesT = 4;
constexpr int kDecWarps = 16;    // two teams of 8 warps alternate K stages
constexpr int kThreadsTc = 32 * (4 + kDecWarps);  // w0: A producer, w1: MMA, w2: B producer, w3: idle

__device__ __forceinline__ uint32_t pow2_h2(int k) {
    k = max(-24, min(15, k));
    uint32_t h = k >= -14 ? uint32_t(k + 15) << 10 : 1u << (k + 24);
    return h | (h << 16);
}
__device__ __forceinline__ uint32_t hmul2_bits(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ void e2m1x8_to_f16(uint32_t w, uint32_t *d) {
    asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
        "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
        "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
        "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
        "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
        "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(w));
}
__device__ __forceinline__ void e4m3x4_to_f16(uint32_t w, uint32_t *d) {
    asm("{\n\t.reg .b16 h0, h1;\n\t"
        "mov.b32 {h0, h1}, %2;\n\t"
        "cvt.rn.f16x2.e4m3x2 %0, h0;\n\t"
        "cvt.rn.f16x2.e4m3x2 %1, h1;\n\t}"
        : "=r"(d[0]), "=r"(d[1])
        : "r"(w));
}

__device__ __forceinline__ void set_status(int32_t *status, int code) {
    if (status) atomicCAS(status, 0, int32_t(code));
}

// Segment of a work unit (segments ordered by unit_begin).
__device__ __forceinline__ int find_seg(const TcSeg *segs, int nsegs, int u) {
    int lo = 0, hi = nsegs - 1;
    while (lo < hi) {
        int mid = (lo + hi + 1) >> 1;
        if (segs[mid].unit_begin <= u) lo = mid; else hi = mid - 1;
    }
    return lo;
}

__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + expf(-v)); }

// Decodes this thread's 32 weights (one row, one K half) of one matrix of a staged tile into
// 16 f16x2 words scaled by 2^(scale-127-e0).
template <int FMT>
__device__ __forceinline__ void decode_row_half(const uint8_t *t, int row, int hlf, int e0,
                                                uint32_t *v) {
    constexpr int TB = tc_tile_bytes(FMT);
    const int scale = t[TB - 256 + 2 * row + hlf];
    const uint32_t mul = pow2_h2(scale - 127 - e0);
    if (FMT == URB_FMT_MXFP4) {
        const uint4 w = *reinterpret_cast<const uint4 *>(t + hlf * 2048 + row * 16);
        e2m1x8_to_f16(w.x, v + 0);
        e2m1x8_to_f16(w.y, v + 4);
        e2m1x8_to_f16(w.z, v + 8);
        e2m1x8_to_f16(w.w, v + 12);
    } else {
        const uint4 w0 = *reinterpret_cast<const uint4 *>(t + (2 * hlf) * 2048 + row * 16);
        const uint4 w1 = *reinterpret_cast<const uint4 *>(t + (2 * hlf + 1) * 2048 + row * 16);
        e4m3x4_to_f16(w0.x, v + 0);
        e4m3x4_to_f16(w0.y, v + 2);
        e4m3x4_to_f16(w0.z, v + 4);
        e4m3x4_to_f16(w0.w, v + 6);
        e4m3x4_to_f16(w1.x, v + 8);
        e4m3x4_to_f16(w1.y, v + 10);
        e4m3x4_to_f16(w1.z, v + 12);
        e4m3x4_to_f16(w1.w, v + 14);
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = hmul2_bits(v[i], mul);
}

template <int FMT, bool PAIR>
__global__ void __launch_bounds__(kThreadsTc, 1) k_tc_grouped(TcArgs a) {
    constexpr int MATS = PAIR ? 2 : 1;
    constexpr int TB = tc_tile_bytes(FMT);
    constexpr int TBA = (MATS * TB + 1023) / 1024 * 1024;  // raw A region per stage (aligned)
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int kStagesA = a.stages_a;
    uint8_t *ring_a = smem;                                  // kStagesA x TBA
    uint8_t *ring_b = smem + size_t(kStagesA) * TBA;         // kStagesB x nmax*128 (1024-aligned)
    const int bstage = a.nmax * 128;
    __shared__ __align__(8) uint64_t a_full[kStagesAMax], a_empty[kStagesAMax];
    __shared__ __align__(8) uint64_t b_full[kStagesB], b_empty[kStagesB];
    __shared__ __align__(8) uint64_t t_full[kStagesT], t_empty[kStagesT];
    __shared__ __align__(8) uint64_t acc_full, acc_empty;
    __shared__ uint32_t tmem_base;
    __shared__ int abort_flag, skip;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nsegs = *a.nsegs;
    const int total_units = *a.total_units;
    // A failed earlier stage (status set) means no work; one thread decides for the whole CTA.
    if (threadIdx.x == 0) skip = (total_units <= 0 || nsegs <= 0 || (a.status && *a.status)) ? 1 : 0;
    __syncthreads();
    if (skip) return;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStagesA; ++s) { tc::mbar_init(&a_full[s], 1); tc::mbar_init(&a_empty[s], 8); }
        for (int s = 0; s < kStagesB; ++s) { tc::mbar_init(&b_full[s], 1); tc::mbar_init(&b_empty[s], 1); }
        for (int s = 0; s < kStagesT; ++s) { tc::mbar_init(&t_full[s], 8); tc::mbar_init(&t_empty[s], 1); }
        tc::mbar_init(&acc_full, 1);
        tc::mbar_init(&acc_empty, kDecWarps);
        tc::mbar_fence_init();
        abort_flag = 0;
    }
    if (warp == 1) {
        tc::tmem_alloc(&tmem_base, 512);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tbase = tmem_base;
    // TMEM columns: accumulators (pair: gate [0,128) up [128,256); single [0,256)), then the A
    // stages (32 columns = 64 f16 per matrix per stage).
    const uint32_t acc_col[2] = {0u, PAIR ? 128u : 0u};
    auto a_col = [&](int t, int m) -> uint32_t { return 256u + uint32_t((t * MATS + m) * 32); };
    auto fail = [&]() {
        abort_flag = 1;
        set_status(a.status, URB_ERR_TIMEOUT);
    };

    if (warp == 0 && lane == 0) {
        // ---------------- weight producer ----------------
        uint32_t g = 0;
        for (int u = blockIdx.x; u < total_units && !abort_flag; u += gridDim.x) {
            const TcSeg S = a.segs[find_seg(a.segs, nsegs, u)];
            const size_t tile0 = size_t(u - S.unit_begin) * S.ks;
            for (int ks = 0; ks < S.ks; ++ks, ++g) {
                const int s = int(g % kStagesA);
                if (!tc::mbar_wait(&a_empty[s], ((g / kStagesA) & 1) ^ 1, &abort_flag)) { fail(); break; }
                uint8_t *st = ring_a + size_t(s) * TBA;
                tc::mbar_arrive_expect_tx(&a_full[s], uint32_t(MATS * TB));
                tc::bulk_g2s(st, S.a + (tile0 + ks) * TB, TB, &a_full[s]);
                if (PAIR) tc::bulk_g2s(st + TB, S.b + (tile0 + ks) * TB, TB, &a_full[s]);
            }
        }
    } else if (warp == 2 && lane == 0) {
        // ---------------- activation producer ----------------
        uint32_t g = 0;
        for (int u = blockIdx.x; u < total_units && !abort_flag; u += gridDim.x) {
            const TcSeg S = a.segs[find_seg(a.segs, nsegs, u)];
            const uint32_t bbytes = uint32_t(S.npad) * 128;
            for (int ks = 0; ks < S.ks; ++ks, ++g) {
                const int s = int(g % kStagesB);
                if (!tc::mbar_wait(&b_empty[s], ((g / kStagesB) & 1) ^ 1, &abort_flag)) { fail(); break; }
                tc::mbar_arrive_expect_tx(&b_full[s], bbytes);
                tc::bulk_g2s(ring_b + size_t(s) * bstage, a.bbuf + S.b_off + size_t(ks) * bbytes, bbytes,
                             &b_full[s]);
            }
        }
    } else if (warp == 1 && lane == 0) {
        // ---------------- MMA issuer ----------------
        uint32_t g = 0, j = 0;
        for (int u = blockIdx.x; u < total_units && !abort_flag; u += gridDim.x, ++j) {
            const TcSeg S = a.segs[find_seg(a.segs, nsegs, u)];
            const uint32_t idesc = tc::idesc_f16(S.npad, FMT == URB_FMT_BF16);
            if (j > 0 && !tc::mbar_wait(&acc_empty, (j - 1) & 1, &abort_flag)) { fail(); break; }
            tc::fence_after_sync();
            bool ok = true;
            for (int ks = 0; ks < S.ks; ++ks, ++g) {
                const int sb = int(g % kStagesB), st = int(g % kStagesT);
                if (!tc::mbar_wait(&t_full[st], (g / kStagesT) & 1, &abort_flag) ||
                    !tc::mbar_wait(&b_full[sb], (g / kStagesB) & 1, &abort_flag)) {
                    ok = false;
                    break;
                }
                tc::fence_after_sync();
                const uint64_t bdesc = tc::sdesc_sw128(tc::smem_u32(ring_b + size_t(sb) * bstage));
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
                    for (int m = 0; m < MATS; ++m)
                        tc::mma_ts(tbase + acc_col[m], tbase + a_col(st, m) + 8 * kk,
                                   bdesc + uint64_t(2 * kk), idesc, ks > 0 || kk > 0);
                }
                tc::mma_commit(&t_empty[st]);
                tc::mma_commit(&b_empty[sb]);
                if (ks == S.ks - 1) tc::mma_commit(&acc_full);
            }
            if (!ok) { fail(); break; }
        }
    } else if (warp >= 4) {
        // ---------------- decoders (two teams) + epilogue ----------------
        const int dw = warp - 4;
        const int team = dw >> 3;         // stages g with g % 2 == team
        const int q = warp & 3;           // TMEM lane quarter
        const int hlf = (dw >> 2) & 1;    // K half of the stage
        const int gid = dw >> 2;          // epilogue column group 0..3
        const int row = 32 * q + lane;    // row within the 128-row tile
        const uint32_t lane_base = uint32_t(32 * q) << 16;
        uint32_t g = 0, j = 0;
        for (int u = blockIdx.x; u < total_units && !abort_flag; u += gridDim.x, ++j) {
            const TcSeg S = a.segs[find_seg(a.segs, nsegs, u)];
            const int grow = (u - S.unit_begin) * 128 + row;  // row within the matrix
            int e0[2];
            e0[0] = S.ra[grow];
            e0[1] = PAIR ? S.rb[grow] : 0;
            bool ok = true;
            for (int ks = 0; ks < S.ks; ++ks, ++g) {
                if (int(g & 1) != team) continue;
                const int sa = int(g % kStagesA), st = int(g % kStagesT);
                if (!tc::mbar_wait(&a_full[sa], (g / kStagesA) & 1, &abort_flag)) { ok = false; break; }
                const uint8_t *t = ring_a + size_t(sa) * TBA;
                uint32_t v[MATS][16];
#pragma unroll
                for (int m = 0; m < MATS; ++m) decode_row_half<FMT>(t + m * TB, row, hlf, e0[m], v[m]);
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&a_empty[sa]);  // raw tile consumed
                if (!tc::mbar_wait(&t_empty[st], ((g / kStagesT) & 1) ^ 1, &abort_flag)) { ok = false; break; }
                tc::fence_after_sync();
#pragma unroll
                for (int m = 0; m < MATS; ++m)
                    tc::tmem_st16(tbase + lane_base + a_col(st, m) + 16 * hlf, v[m]);
                tc::wait_st();
                tc::fence_before_sync();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&t_full[st]);
            }
            if (!ok) break;
            // Epilogue of this tile: 16 warps, column chunks round-robin over 4 groups.
            if (!tc::mbar_wait(&acc_full, j & 1, &abort_flag)) break;
            tc::fence_after_sync();
            const bool row_ok = grow < S.rows;
            const int chunks = S.npad / 16;
            const int per = S.rowsper;
            for (int c = gid; c < chunks; c += 4) {
                uint32_t d[2][16];
#pragma unroll
                for (int m = 0; m < MATS; ++m) tc::tmem_ld16(tbase + lane_base + acc_col[m] + 16 * c, d[m]);
                tc::wait_ld();
                // Column n = 16c + i of the accumulator is activation row n of the segment.
#pragma unroll
                for (int i = 0; i < 16; i += 2) {
#pragma unroll
                    for (int t2 = 0; t2 < 2; ++t2) {
                        if (per == 2 && t2 == 1) break;
                        const int n = 16 * c + i + (per == 2 ? 0 : t2);
                        const int tok = n / per;
                        const bool tok_ok = tok < S.ntok;
                        const int col = S.col_begin + (tok_ok ? tok : 0);
                        const int srow = a.col_src ? a.col_src[col] : col;
                        const int shift = tok_ok ? (a.src_shift ? a.src_shift[srow]
                                                    : (a.src_maxexp[srow] > -1000 ? 14 - a.src_maxexp[srow] : 0))
                                                 : 0;
                        float vv[2];
#pragma unroll
                        for (int m = 0; m < MATS; ++m) {
                            const float x0 = __uint_as_float(d[m][i + (per == 2 ? 0 : t2)]);
                            const float x1 = per == 2 ? __uint_as_float(d[m][i + 1]) : 0.0f;
                            vv[m] = ldexpf(x0 + x1, e0[m] - shift);
                        }
                        float o = vv[0];
                        if (PAIR) o = silu_f(vv[0]) * vv[MATS - 1];
                        if (tok_ok && row_ok) a.out[size_t(col) * a.out_stride + grow] = o;
                        if (PAIR && a.out_maxexp) {
                            int me = (tok_ok && row_ok && o != 0.0f && isfinite(o)) ? ilogbf(o) : -1000;
#pragma unroll
                            for (int off = 16; off > 0; off >>= 1)
                                me = max(me, __shfl_xor_sync(0xffffffffu, me, off));
                            if (lane == 0 && me > -1000) atomicMax(a.out_maxexp + col, me);
                        }
                    }
                }
            }
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&acc_empty);
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tbase, 512);
    }
}

// Activation tiles of every segment: rows (token hi [, lo]) x 64 columns per K stage, f16,
// 128-byte swizzled canonical K-major layout, padded to S.npad rows.  One warp per
// (segment, stage, 8 rows); grid-stride over all of them.
__global__ void k_prep_b(TcArgs a, int max_ks) {
    const int nsegs = *a.nsegs;
    if (a.status && *a.status) return;
    const long long total = (long long)nsegs * max_ks * 32;  // (seg, ks, 8-row group) items
    const int lane = threadIdx.x & 31;
    for (long long it = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5; it < total;
         it += (gridDim.x * (long long)blockDim.x) >> 5) {
        const int rg = int(it % 32), ks = int((it / 32) % max_ks), si = int(it / 32 / max_ks);
        const TcSeg S = a.segs[si];
        if (ks >= S.ks || rg * 8 >= S.npad) continue;
        uint8_t *dst = a.bbuf + S.b_off + size_t(ks) * S.npad * 128;
        // 32 lanes: 8 rows x 4 lanes, each lane two 16-byte chunks.
        const int r = rg * 8 + (lane >> 2);
        for (int jc = (lane & 3); jc < 8; jc += 4) {
            const int tok = r / S.rowsper, part = r % S.rowsper;
            uint4 out = make_uint4(0, 0, 0, 0);
            if (tok < S.ntok) {
                const int col = S.col_begin + tok;
                const int srow = a.col_src ? a.col_src[col] : col;
                const int shift = a.src_shift ? a.src_shift[srow]
                                              : (a.src_maxexp[srow] > -1000 ? 14 - a.src_maxexp[srow] : 0);
                const float *p = a.src + size_t(srow) * a.src_stride;
                const int k0 = ks * 64 + jc * 8;
                uint32_t h[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float x = k0 + i < S.cols ? ldexpf(p[k0 + i], shift) : 0.0f;
                    __half hi = __float2half_rn(x);
                    __half v = part ? __float2half_rn(x - __half2float(hi)) : hi;
                    h[i] = __half_as_ushort(v);
                }
                out = make_uint4(h[0] | (h[1] << 16), h[2] | (h[3] << 16), h[4] | (h[5] << 16),
                                 h[6] | (h[7] << 16));
            }
            *reinterpret_cast<uint4 *>(dst + r * 128 + ((jc ^ (r & 7)) << 4)) = out;
        }
    }
}

// Repack of the reference layout into the tc layout (one thread per (tile, row)).
template <int FMT>
__global__ void k_repack_tc(const uint8_t *values, const uint8_t *scales, size_t rows,
                            size_t cols, size_t scale_cols, size_t block_rows,
                            size_t block_cols, int mts, int ks_n, uint8_t *out) {
    const size_t id = blockIdx.x * size_t(blockDim.x) + threadIdx.x;
    if (id >= size_t(mts) * ks_n * 128) return;
    const int r = int(id & 127);
    const size_t tile = id >> 7;
    const int ks = int(tile % ks_n);
    const size_t mt = tile / ks_n;
    const size_t row = mt * 128 + r;
    constexpr int TB = tc_tile_bytes(FMT);
    uint8_t *t = out + tile * TB;
    const size_t c0 = size_t(ks) * 64;
    if (FMT == URB_FMT_MXFP4) {
        const size_t row_bytes = (cols + 1) / 2;
        for (int ch = 0; ch < 2; ++ch)
            for (int b = 0; b < 16; ++b) {
                const size_t c = c0 + ch * 32 + 2 * b;
                uint8_t lo = 0, hi = 0;
                if (row < rows && c < cols) lo = values[row * row_bytes + c / 2] & 0x0f;
                if (row < rows && c + 1 < cols) hi = values[row * row_bytes + c / 2] >> 4;
                t[ch * 2048 + r * 16 + b] = uint8_t(lo | (hi << 4));
            }
        for (int h = 0; h < 2; ++h) {
            const size_t c = c0 + 32 * h;
            t[TB - 256 + 2 * r + h] = (row < rows && c < cols) ? scales[row * scale_cols + c / 32] : 127;
        }
    } else {
        for (int ch = 0; ch < 4; ++ch)
            for (int b = 0; b < 16; ++b) {
                const size_t c = c0 + ch * 16 + b;
                t[ch * 2048 + r * 16 + b] = (row < rows && c < cols) ? values[row * cols + c] : 0;
            }
        for (int h = 0; h < 2; ++h) {
            const size_t c = c0 + 32 * h;
            t[TB - 256 + 2 * r + h] =
                (row < rows && c < cols) ? scales[(row / block_rows) * scale_cols + c / block_cols] : 127;
        }
    }
}

template <int FMT, bool PAIR>
int launch_tc_t(Ctx *ctx, const TcArgs &a, cudaStream_t st) {
    constexpr int MATS = PAIR ? 2 : 1;
    const size_t tba = (size_t(MATS) * tc_tile_bytes(FMT) + 1023) / 1024 * 1024;
    const size_t budget = 220 * 1024, bring = kStagesB * size_t(a.nmax) * 128 + 1024;
    if (bring + 3 * tba > budget) return set_error(ctx, URB_ERR_UNSUPPORTED, "tc pass: shared memory");
    TcArgs args = a;
    args.stages_a = int(std::min<size_t>(kStagesAMax, (budget - bring) / tba));
    // At least 116 KB so that exactly one CTA (and one 512-column TMEM allocation) fits per SM.
    const size_t smem = std::max<size_t>(116 * 1024, bring + args.stages_a * tba);
    auto k = k_tc_grouped<FMT, PAIR>;
    URB_CUDA(ctx, cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
    k<<<ctx->num_sms, kThreadsTc, smem, st>>>(args);
    URB_CUDA(ctx, cudaGetLastError());
    return URB_OK;
}

}  // namespace

int launch_tc_grouped(Ctx *ctx, int fmt, bool pair, const TcArgs &a, int max_segs, int max_ks,
                      cudaStream_t st) {
    if (a.nmax > (pair ? 128 : 256) || a.nmax % 16)
        return set_error(ctx, URB_ERR_UNSUPPORTED, "tc pass: N out of range");
    (void)max_segs;
    k_prep_b<<<ctx->num_sms * 8, 256, 0, st>>>(a, max_ks);
    URB_CUDA(ctx, cudaGetLastError());
    if (fmt == URB_FMT_MXFP4) return pair ? launch_tc_t<URB_FMT_MXFP4, true>(ctx, a, st)
                                          : launch_tc_t<URB_FMT_MXFP4, false>(ctx, a, st);
    if (fmt == URB_FMT_MXFP8) return pair ? launch_tc_t<URB_FMT_MXFP8, true>(ctx, a, st)
                                          : launch_tc_t<URB_FMT_MXFP8, false>(ctx, a, st);
    return set_error(ctx, URB_ERR_UNSUPPORTED, "tc pass: format");
}

int repack_tc(Ctx *ctx, Mat *m, cudaStream_t st) {
    if (m->format != URB_FMT_MXFP4 && m->format != URB_FMT_MXFP8) return URB_OK;
    m->tc_mts = int((m->rows + 127) / 128);
    m->tc_ks = int((m->cols + 63) / 64);
    const int TB = tc_tile_bytes(m->format);
    URB_CUDA(ctx, cudaMallocAsync((void **)&m->tc_tiles, size_t(m->tc_mts) * m->tc_ks * TB, st));
    const size_t threads = size_t(m->tc_mts) * m->tc_ks * 128;
    const unsigned blocks = unsigned((threads + 255) / 256);
    const uint8_t *v = static_cast<const uint8_t *>(m->raw_values);
    if (m->format == URB_FMT_MXFP4) {
        const size_t sc = (m->cols + m->group_size - 1) / m->group_size;
        k_repack_tc<URB_FMT_MXFP4><<<blocks, 256, 0, st>>>(v, m->raw_scales, m->rows, m->cols, sc,
                                                          1, 32, m->tc_mts, m->tc_ks, m->tc_tiles);
    } else {
        const size_t sc = (m->cols + m->block_cols - 1) / m->block_cols;
        k_repack_tc<URB_FMT_MXFP8><<<blocks, 256, 0, st>>>(v, m->raw_scales, m->rows, m->cols, sc,
                                                          m->block_rows, m->block_cols, m->tc_mts,
                                                          m->tc_ks, m->tc_tiles);
    }
    URB_CUDA(ctx, cudaGetLastError());
    return URB_OK;
}

}  // namespace urb
