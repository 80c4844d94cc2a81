// matvec_tc.cu — single-token MX matvec (MxFp4Matrix::matvec_rows, src/math/mxfp.rs:1725-1780;
// MxFp8Matrix::matvec_rows, mxfp.rs:660-714) on the block-scaled tensor cores, reading the same
// resident 128-row tiles as the grouped passes (no second copy of the weights).
//
// A decode product streams every weight byte once, so the kernel is shaped around HBM:
//   * k_mv_tc splits every 128-row tile's K stages over a cluster of `ksplit` CTAs (one per
//     SM).  Each CTA requests its weight tiles first (one bulk copy per lane, up to 8 in
//     flight, then a ring), before it waits for the kernel ahead of it (programmatic dependent
//     launch), so the weight stream starts at once and overlaps the previous kernel's tail.
//   * Meanwhile its warps write its own K range of x straight into shared memory as exact
//     fixed-point digit terms (the 24-bit significand relative to each 32-column block's
//     largest exponent, one redux.sync per block): 12 base-4 digits as E2M1 codes 0..3 for
//     MXFP4, 6 base-16 digits as E4M3 integers for MXFP8, each term with its E8M0 scale, in
//     the activation-stage layout of the grouped passes (16 MMA rows per K stage).
//   * Four issuing threads take turns over the stages, each into its own TMEM accumulator
//     (N = 16); the epilogue
//     warps sum each row's term columns; ranks >= 1 push their partial sums into rank 0's
//     shared memory, which adds them in rank order, so the result is deterministic.  No
//     global scratch is used.
// Every wait is bounded (URB_ERR_TIMEOUT); every copy in flight lands before a CTA exits.
#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>

#include "bs_terms.cuh"
#include "tc_common.cuh"
#include "urb_internal.cuh"
#include "urb_tc.cuh"

namespace urb {
namespace {

constexpr int kMvMaxStages = 8;             // K stages per CTA: all its tiles resident at once
constexpr int kMvN = 16;                    // MMA N: activation rows per stage
constexpr int kMvThreads = 512;
constexpr int kMvWSlot = 17408;             // bytes of a weight slot (largest bs tile)
constexpr int kMvBSlot = 3072;              // bytes of an activation slot (largest stage)
constexpr int kMvIssuers = 4;               // MMA issuing threads, one accumulator each
constexpr uint32_t kMvAccCols = 16;         // accumulator columns per issuer
constexpr uint32_t kMvSfCol0 = kMvIssuers * kMvAccCols;  // TMEM scale slot s at kMvSfCol0 + 16 s
static_assert(bs_tile_bytes(URB_FMT_MXFP4) <= kMvWSlot && bs_tile_bytes(URB_FMT_MXFP8) <= kMvWSlot, "slot");
static_assert(bs_bstage_bytes(URB_FMT_MXFP4, kMvN) <= kMvBSlot, "slot");

// Dynamic shared memory of a CTA holding S stages (weights, then activation terms) and the TMEM
// columns it allocates (a power of two >= 32).
__host__ __device__ constexpr int mv_smem(int S) { return S * (kMvWSlot + kMvBSlot) + 1024; }
__host__ __device__ constexpr uint32_t mv_tmem_cols(int S) { return kMvSfCol0 + 16 * S <= 128 ? 128 : 256; }
static_assert(mv_smem(kMvMaxStages) <= 227 * 1024, "shared memory");
static_assert(kMvSfCol0 + 16 * kMvMaxStages <= 256, "tmem");

// Activation terms per token: x as fixed-point digits of its 24-bit significand relative to
// its 32-column block's largest exponent, 2 bits per E2M1 term (12 terms) or 4 bits per E4M3
// term (6 terms); every one of them within the 16 MMA rows.
template <int FMT>
constexpr int mv_digit_bits() { return FMT == URB_FMT_MXFP4 ? 2 : 4; }
template <int FMT>
constexpr int mv_terms() { return 24 / mv_digit_bits<FMT>(); }

__device__ __forceinline__ void set_status(int32_t *status, int code) {
    if (status) atomicCAS(status, 0, int32_t(code));
}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// The value x of this lane as X * 2^(emax - 150) (X < 2^24, rounded to nearest even), emax the
// biased exponent of the largest |x| of the warp's 32 values (at least 1, so subnormals share
// the smallest normal binade's units); emax = -1 for an all-zero block.  One warp reduction:
// non-negative floats order like their bit patterns.
__device__ __forceinline__ void block_fixed_point(float x, uint32_t &X, uint32_t &neg, int &emax) {
    const uint32_t bx = __float_as_uint(x), ab = bx & 0x7fffffffu;
    const uint32_t bm = __reduce_max_sync(0xffffffffu, ab);
    neg = bx >> 31;
    int ex = int(ab >> 23), em = int(bm >> 23);
    const uint32_t M = (ab & 0x7fffffu) | (ex ? 0x800000u : 0u);
    ex = max(ex, 1);
    em = max(em, 1);
    const int sh = em - ex;
    X = sh == 0 ? M : (sh >= 25 ? 0u : (M + (1u << (sh - 1)) - 1u + ((M >> sh) & 1u)) >> sh);
    emax = bm ? em : -1;
}

// Digit term j of a block: its element code (E2M1: digit d in 0..3 is the value d / 2, codes
// 0..3; E4M3: the integer d in 0..15, whose codes come from a 16-byte table) with the sign, and
// its E8M0 scale byte, so that code * 2^(byte - 127) = d * 2^(bits * j) * 2^(emax - 150).
// A scale below E8M0's range (|max| < 2^-104) drops the digit.
// The twelve base-4 digits of X (< 2^24) as E2M1 codes 0..3 in the nibbles of a 48-bit word
// (digit j in nibble j), the sign bit set on the non-zero ones, digits below E8M0's scale range
// (scale byte emax - 22 + 2j < 0) dropped.
__device__ __forceinline__ uint64_t e2m1_digit_nibbles(uint32_t X, uint32_t neg, int emax) {
    uint64_t v = uint64_t(X & 0xfffu) | (uint64_t(X & 0xfff000u) << 12);        // 12-bit halves
    v = (v & 0x00003f00003full) | ((v & 0x000fc0000fc0ull) << 6);                // 6-bit quarters
    v = (v & 0x003003003003ull) | ((v & 0x00c00c00c00cull) << 2) | ((v & 0x030030030030ull) << 4);
    const uint64_t nz = (v | (v >> 1)) & 0x111111111111ull;
    v |= neg ? nz << 3 : 0ull;
    // Digits whose scale byte emax - 22 + 2j would be negative: j < (22 - emax) / 2.
    const int drop = emax < 22 ? (23 - emax) >> 1 : 0;
    if (emax < 0 || drop >= 12) return 0;
    if (drop > 0) v &= ~((uint64_t(1) << (4 * drop)) - 1);
    return v;
}

// Transposes an 8 x 8 matrix of nibbles held by 8 consecutive lanes (lane i holds column i,
// nibble k = row k) so that lane i holds row i (nibble k = column k): three butterfly stages.
__device__ __forceinline__ uint32_t transpose_nibbles8(uint32_t a, int lane) {
    uint32_t b = __shfl_xor_sync(0xffffffffu, a, 1);
    a = (lane & 1) ? ((b >> 4) & 0x0f0f0f0fu) | (a & 0xf0f0f0f0u) : (a & 0x0f0f0f0fu) | ((b << 4) & 0xf0f0f0f0u);
    b = __shfl_xor_sync(0xffffffffu, a, 2);
    a = (lane & 2) ? ((b >> 8) & 0x00ff00ffu) | (a & 0xff00ff00u) : (a & 0x00ff00ffu) | ((b << 8) & 0xff00ff00u);
    b = __shfl_xor_sync(0xffffffffu, a, 4);
    a = (lane & 4) ? ((b >> 16) & 0x0000ffffu) | (a & 0xffff0000u) : (a & 0x0000ffffu) | ((b << 16) & 0xffff0000u);
    return a;
}

// The same for a 4 x 4 matrix of bytes held by 4 consecutive lanes.
__device__ __forceinline__ uint32_t transpose_bytes4(uint32_t a, int lane) {
    uint32_t b = __shfl_xor_sync(0xffffffffu, a, 1);
    a = (lane & 1) ? ((b >> 8) & 0x00ff00ffu) | (a & 0xff00ff00u) : (a & 0x00ff00ffu) | ((b << 8) & 0xff00ff00u);
    b = __shfl_xor_sync(0xffffffffu, a, 2);
    a = (lane & 2) ? ((b >> 16) & 0x0000ffffu) | (a & 0xffff0000u) : (a & 0x0000ffffu) | ((b << 16) & 0xffff0000u);
    return a;
}

template <int FMT>
__device__ __forceinline__ uint32_t digit_code(uint32_t X, uint32_t neg, int j, int emax, int &byte) {
    constexpr int B = mv_digit_bits<FMT>();
    const uint32_t d = (X >> (B * j)) & ((1u << B) - 1);
    byte = FMT == URB_FMT_MXFP4 ? emax - 22 + 2 * j : emax - 23 + 4 * j;
    if (emax < 0 || byte < 0) {
        byte = 0;
        return 0;
    }
    uint32_t code;
    if (FMT == URB_FMT_MXFP4) {
        code = d;
        if (d && neg) code |= 8u;
    } else {
        // E4M3 codes of the integers 0 .. 15 (1 = 0x38, 2 = 0x40, ..., 15 = 0x57).
        const uint32_t lo = d < 8 ? 0x44403800u : 0x53525150u, hi = d < 8 ? 0x4E4C4A48u : 0x57565554u;
        code = __byte_perm(lo, hi, d & 7) & 0xffu;
        if (d && neg) code |= 0x80u;
    }
    return code;
}

struct MvArgs {
    const uint8_t *tiles;  // bs tiles, tile (mt, ks) at (ks * mts + mt) * TB
    int mts, ks;
    int mt_lo;             // first row tile of the launch (grid y offset)
    int spc;               // K stages per CTA of a cluster (<= kMvMaxStages)
    int rows, cols;        // real rows / input columns of the matrix
    long long row_start, row_count;  // output rows [row_start, row_start + row_count) -> y[0..)
    const float *x;
    float *y;
    int32_t *status;
};

// Waits (acquire at cluster scope) for the phase with the given parity; bounded.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t *bar, uint32_t parity, uint32_t limit) {
    for (uint32_t i = 0; i < limit; ++i) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok) : "r"(tc::smem_u32(bar)), "r"(parity) : "memory");
        if (ok) return true;
    }
    return false;
}

template <int FMT, int NT>
__global__ void __launch_bounds__(kMvThreads, 1) k_mv_tc(MvArgs a) {
    constexpr int TB = bs_tile_bytes(FMT);
    constexpr int CH = bs_sf_chunks(FMT);
    constexpr int KBS = FMT == URB_FMT_MXFP4 ? 8 : 4;  // 32-column blocks per stage
    constexpr int KIND_FMT = FMT == URB_FMT_MXFP4 ? 1 : 0;
    constexpr int WARPS = kMvThreads / 32;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ __align__(8) uint64_t a_full[kMvMaxStages], sf_full[kMvMaxStages];
    __shared__ __align__(8) uint64_t acc_full[kMvIssuers], mma_done[kMvIssuers], red_full;
    __shared__ uint32_t tmem_base;
    __shared__ int abort_flag, never;
    __shared__ float red[8][128];  // rank 0: the cluster's partial sums by rank

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kq = blockIdx.x;  // rank in the cluster (cluster dims (ksplit, 1, 1))
    const int nq = gridDim.x;
    const int mt = a.mt_lo + blockIdx.y;
    const int s0 = kq * a.spc;
    const int S = max(0, min(a.ks, s0 + a.spc) - s0);
    uint8_t *wslots = smem;                                   // [spc][kMvWSlot]
    uint8_t *bstages = smem + size_t(a.spc) * kMvWSlot;       // [spc][kMvBSlot]
    const uint32_t tcols = mv_tmem_cols(a.spc);
    const uint8_t *wsrc = a.tiles + (size_t(s0) * a.mts + mt) * TB;
    const size_t wstride = size_t(a.mts) * TB;  // next K stage of the same row tile

    // x may be the output of the kernel before this one.  Its loads go out first (warp 0 first
    // requests the weights): they share the SM's memory path with the weight stream, so every
    // value of a warp is requested at once.
    constexpr int MAXB = kMvMaxStages * KBS / WARPS;  // 32-column blocks per warp at most
    const int nb = S * KBS;
    float xv[MAXB];
    auto load_x = [&]() {
        pdl_wait();
#pragma unroll
        for (int u = 0; u < MAXB; ++u) {
            const int lb = warp + u * WARPS;
            const int c = (s0 * KBS + lb) * 32 + lane;
            xv[u] = lb < nb && c < a.cols ? __ldg(a.x + c) : 0.0f;
        }
    };
    if (warp != 0) load_x();
    if (warp == 0) {
        // The weight stream needs nothing from earlier kernels: the barriers are initialised
        // and every tile of the CTA requested (one lane per tile) before anything else.
        if (lane == 0) {
            for (int s = 0; s < kMvMaxStages; ++s) {
                tc::mbar_init(&a_full[s], 1);
                tc::mbar_init(&sf_full[s], 4);  // one arrival per scale warp of the stage's group
            }
            for (int i = 0; i < kMvIssuers; ++i) {
                tc::mbar_init(&acc_full[i], 1);
                tc::mbar_init(&mma_done[i], 1);
            }
            tc::mbar_init(&red_full, 1);
            tc::mbar_fence_init();
            abort_flag = 0;
            never = 0;
        }
        __syncwarp();
        if (lane < S) {
            // Weights are read once per product: they leave L2 first.
            tc::mbar_arrive_expect_tx(&a_full[lane], uint32_t(TB));
            tc::bulk_g2s_hint(wslots + size_t(lane) * kMvWSlot, wsrc + size_t(lane) * wstride, TB,
                              &a_full[lane], tc::l2_evict_first_policy());
        }
        // Rank 0 expects the other ranks' partial sums (128 floats each) on red_full.
        if (lane == 0 && kq == 0 && nq > 1) tc::mbar_arrive_expect_tx(&red_full, uint32_t(512 * (nq - 1)));
        load_x();
    } else if (warp == 1) {
        tc::tmem_alloc(&tmem_base, tcols);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    // Rank 0's reduction barrier is initialised before any CTA of the cluster uses it.
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
    pdl_launch_dependents();
    const uint32_t tbase = tmem_base;
    volatile int *abortp = &abort_flag;
    auto fail = [&]() {
        *abortp = 1;
        set_status(a.status, URB_ERR_TIMEOUT);
    };

    // ---- x -> digit terms of this CTA's K stages, straight into shared memory -------------
    // A warp per 32-column block (one value per lane, loaded above), encoded in lockstep,
    // blocks past the CTA's range on zeros with their stores skipped.  Terms in MMA rows 0 .. NT-1; rows NT .. 15 are never written:
    // they only feed accumulator columns the epilogue does not read.
    {
#pragma unroll
        for (int u = 0; u < MAXB; ++u) {
            const int lb = warp + u * WARPS;
            const bool live = lb < nb;  // warp-uniform
            float v = xv[u];
            if (!isfinite(v)) {
                set_status(a.status, URB_ERR_NONFINITE);
                v = 0.0f;
            }
            uint32_t X, neg;
            int emax;
            block_fixed_point(v, X, neg, emax);
            const int kbs = lb % KBS;
            uint8_t *stage = bstages + size_t(lb / KBS) * kMvBSlot;
            // Rows are assembled as whole 32-bit words by transposes across lanes (byte stores
            // from several lanes into one word would serialise); row R's chunk c sits at
            // (c ^ (R & 7)) * 16 of the row (128-byte swizzle).
            if (FMT == URB_FMT_MXFP4) {
                // Lane 8w + i ends up with row i (and row 8 + i) of columns 8w .. 8w + 7; column
                // 2b in the low nibble of byte b of the block's chunk kbs.
                const uint64_t nib = e2m1_digit_nibbles(X, neg, emax);
                const uint32_t lo = transpose_nibbles8(uint32_t(nib), lane);
                const uint32_t hi = transpose_nibbles8(uint32_t(nib >> 32), lane);
                if (live) {
                    const int i = lane & 7, w = lane >> 3;
                    *reinterpret_cast<uint32_t *>(stage + (i >> 3) * 1024 + (i & 7) * 128 +
                                                  ((kbs ^ (i & 7)) << 4) + 4 * w) = lo;
                    if (i < NT - 8) {
                        const int R = 8 + i;
                        *reinterpret_cast<uint32_t *>(stage + (R >> 3) * 1024 + (R & 7) * 128 +
                                                      ((kbs ^ (R & 7)) << 4) + 4 * w) = hi;
                    }
                }
            } else {
                // Lane 4w + i ends up with row i (and row 4 + i) of columns 4w .. 4w + 3.
                uint32_t q0 = 0, q1 = 0;
#pragma unroll
                for (int R = 0; R < NT; ++R) {
                    int byte;
                    const uint32_t code = digit_code<FMT>(X, neg, R, emax, byte);
                    if (R < 4) q0 |= code << (8 * R);
                    else q1 |= code << (8 * (R - 4));
                }
                q0 = transpose_bytes4(q0, lane);
                q1 = transpose_bytes4(q1, lane);
                if (live) {
                    const int i = lane & 3, w = lane >> 2;
                    const int ch = 2 * kbs + (w >> 2);
                    *reinterpret_cast<uint32_t *>(stage + (i & 7) * 128 + ((ch ^ (i & 7)) << 4) + 4 * (w & 3)) = q0;
                    if (i < NT - 4) {
                        const int R = 4 + i;
                        *reinterpret_cast<uint32_t *>(stage + (R & 7) * 128 + ((ch ^ (R & 7)) << 4) + 4 * (w & 3)) = q1;
                    }
                }
            }
            // Scale bytes: lane R writes term R's.
            if (live && lane < NT) {
                const int byte = FMT == URB_FMT_MXFP4 ? emax - 22 + 2 * lane : emax - 23 + 4 * lane;
                stage[kMvN * 128 + 512 * (kbs >> 2) + 16 * lane + (kbs & 3)] =
                    uint8_t(emax < 0 || byte < 0 ? 0 : byte);
            }
        }
    }
    // The tensor cores (async proxy) read what the threads just wrote.
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");

    if ((warp == 1 || warp == 2 || warp == 3 || warp == 8) && lane == 0) {
        // ---------------- MMA issuers (one per scheduler): stages j = me, me + 4, ... -------
        const int me = warp == 8 ? 3 : warp - 1;
        const uint32_t acc = tbase + uint32_t(me) * kMvAccCols;
        bool any = false, ok = true;
        for (int j = me; j < S; j += kMvIssuers) {
            if (!tc::mbar_wait(&sf_full[j], 0, abortp)) { ok = false; break; }
            tc::fence_after_sync();
            const uint64_t adesc = tc::sdesc_sw128(tc::smem_u32(wslots + size_t(j) * kMvWSlot));
            const uint64_t bdesc = tc::sdesc_sw128(tc::smem_u32(bstages + size_t(j) * kMvBSlot));
            const uint32_t sfa = tbase + kMvSfCol0 + 16u * j, sfb = sfa + 8;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const bool accum = any || kk > 0;
                if (FMT == URB_FMT_MXFP4) {
                    const uint32_t id = 2u * (kk & 1), col = 4u * (kk >> 1);
                    tc::mma_mxf4(acc, adesc + 2 * kk, bdesc + 2 * kk, tc::idesc_bs(KIND_FMT, kMvN, id, id),
                                 (sfa + col) | (id << 30), (sfb + col) | (id << 30), accum);
                } else {
                    const uint32_t id = uint32_t(kk);
                    tc::mma_mxf8(acc, adesc + 2 * kk, bdesc + 2 * kk, tc::idesc_bs(KIND_FMT, kMvN, id, id),
                                 sfa | (id << 30), sfb | (id << 30), accum);
                }
            }
            any = true;
        }
        if (!ok) fail();
        if (any) tc::mma_commit(&acc_full[me]);
        // Every MMA of this thread completes before TMEM is released.
        tc::mma_commit(&mma_done[me]);
        tc::mbar_wait(&mma_done[me], 0, &never);
    } else if ((warp >= 4 && warp < 8) || warp >= 12) {
        // ---------------- scale warps (warps 4-7: even stages, 12-15: odd), then the
        // epilogue (warps 4-7) ----------------
        const int qtr = warp & 3;  // TMEM lane quarter of this warp
        const uint32_t lane_base = uint32_t(32 * qtr) << 16;
        const int grp = warp >= 12 ? 1 : 0;
        bool ok = true;
        // Stage j's scales (A's chunks at +0 / +4, B's at +8 / +12 of TMEM slot j; lane l of
        // every quarter holds bytes 16 l .. 16 l + 15 of each 512-byte chunk) go out as soon
        // as its tile has landed; tiles that have already landed are staged together behind
        // one wait for the stores.
        int done = grp;
        while (done < S && ok) {
            int j = done;
            if (!tc::mbar_wait(&a_full[j], 0, abortp)) { ok = false; break; }
            do {
                const uint8_t *sfa = wslots + size_t(j) * kMvWSlot + 16384 + 16 * lane;
                const uint8_t *sfb = bstages + size_t(j) * kMvBSlot + kMvN * 128 + 16 * lane;
                uint32_t v[16];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    uint4 qa = make_uint4(0, 0, 0, 0), qb = make_uint4(0, 0, 0, 0);
                    if (h < CH) {
                        qa = *reinterpret_cast<const uint4 *>(sfa + 512 * h);
                        qb = *reinterpret_cast<const uint4 *>(sfb + 512 * h);
                    }
                    v[4 * h] = qa.x; v[4 * h + 1] = qa.y; v[4 * h + 2] = qa.z; v[4 * h + 3] = qa.w;
                    v[8 + 4 * h] = qb.x; v[9 + 4 * h] = qb.y; v[10 + 4 * h] = qb.z; v[11 + 4 * h] = qb.w;
                }
                tc::tmem_st16(tbase + lane_base + kMvSfCol0 + 16u * j, v);
                j += 2;
            } while (j < S && tc::mbar_try_wait(&a_full[j], 0));
            tc::wait_st();
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0)
                for (int i = done; i < j; i += 2) tc::mbar_arrive(&sf_full[i]);
            done = j;
        }
        if (!ok) fail();
        if (grp) goto role_done;
        // Epilogue: row 32 qtr + lane of the tile; the issuers' accumulators summed over the
        // token's term columns.
        float part = 0.0f;
        const int used = min(S, kMvIssuers);  // issuers that ran a stage
        for (int i = 0; i < used && ok; ++i)
            if (!tc::mbar_wait(&acc_full[i], 0, abortp)) { fail(); ok = false; }
        if (ok && used > 0) {
            tc::fence_after_sync();
            uint32_t v[kMvIssuers][16];
#pragma unroll
            for (int i = 0; i < kMvIssuers; ++i)
                if (i < used) tc::tmem_ld16(tbase + lane_base + uint32_t(i) * kMvAccCols, v[i]);
            tc::wait_ld();
#pragma unroll
            for (int i = 0; i < kMvIssuers; ++i) {
                if (i >= used) break;
                float s = 0.0f;
#pragma unroll
                for (int t = 0; t < NT; ++t) s += __uint_as_float(v[i][t]);
                part += s;
            }
        }
        const int row = 32 * qtr + lane;
        if (kq != 0) {
            // Ranks >= 1 store their partial sums into rank 0's shared memory; each store
            // completes its bytes on rank 0's barrier.  Every thread stores on every path, so
            // rank 0's wait always completes.
            uint32_t dst, bar;
            asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(dst) : "r"(tc::smem_u32(&red[kq][row])));
            asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(bar) : "r"(tc::smem_u32(&red_full)));
            asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.f32 [%0], %1, [%2];"
                         ::"r"(dst), "f"(part), "r"(bar) : "memory");
        } else {
            // Rank 0 stays until every partial has arrived (a far longer bound than any wait of
            // the other ranks, which always store), adds them in rank order and stores y.
            if (nq > 1 && !mbar_wait_cluster(&red_full, 0, 1u << 26)) fail();
            float v = part;
            for (int q = 1; q < nq; ++q) v += red[q][row];
            const long long grow = (long long)mt * 128 + row;
            if (grow < a.rows && grow >= a.row_start && grow < a.row_start + a.row_count)
                a.y[grow - a.row_start] = v;
        }
    }
role_done:
    __syncwarp();
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tbase, tcols);
    }
}

// Clusters of `ksplit` CTAs of this kernel that can be resident at once on the current device.
template <typename K>
int query_resident_clusters(K kern, int ksplit, int spc) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ksplit, 1, 1);
    cfg.blockDim = dim3(kMvThreads);
    cfg.dynamicSmemBytes = mv_smem(spc);
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = ksplit;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

// Per-device set-up of a format's kernel, cached (host work on every launch otherwise): its
// shared-memory size and the resident clusters per K split.
constexpr int kMvMaxDevices = 64;
std::atomic<int> g_resident[kMvMaxDevices][2][9][kMvMaxStages + 1];
std::atomic<bool> g_attrs_set[kMvMaxDevices][2];

// Launch attributes (URB_MV_LAUNCH=plain drops programmatic dependent launch; for timing).
bool mv_pdl() {
    static const bool on = [] {
        const char *v = std::getenv("URB_MV_LAUNCH");
        return !(v && std::strcmp(v, "plain") == 0);
    }();
    return on;
}

template <int FMT>
int launch_t(Ctx *ctx, const Mat *m, size_t start, size_t count, const float *d_x, float *d_y,
             int32_t *d_status, cudaStream_t st) {
    constexpr int NT = mv_terms<FMT>();
    auto kern = k_mv_tc<FMT, NT>;
    const int f = FMT == URB_FMT_MXFP4 ? 0 : 1;
    const int dev = ctx->device;
    const bool cached = dev >= 0 && dev < kMvMaxDevices;
    if (!cached || !g_attrs_set[dev][f].load()) {
        URB_CUDA(ctx, cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           mv_smem(kMvMaxStages)));
        if (cached) g_attrs_set[dev][f].store(true);
    }
    auto resident = [&](int ksp, int spc) {
        if (!cached) return query_resident_clusters(kern, ksp, spc);
        int v = g_resident[dev][f][ksp][spc].load(std::memory_order_relaxed);
        if (v <= 0) {
            v = query_resident_clusters(kern, ksp, spc);
            g_resident[dev][f][ksp][spc].store(v, std::memory_order_relaxed);
        }
        return v;
    };
    const int mt_lo = int(start / 128), mt_hi = int((start + count + 127) / 128);
    const int nmt = mt_hi - mt_lo;
    // K split: about one CTA per SM (measured faster than two smaller ones per SM: each CTA's
    // fixed set-up, encoding and tail cost the same whatever its share of the weights), at
    // most 8 per row tile (one portable cluster), every cluster of the launch resident at
    // once, and at most kMvMaxStages stages per CTA (longer K: the CUDA-core kernel takes the
    // product).
    const int need = (m->tc_ks + kMvMaxStages - 1) / kMvMaxStages;
    if (need > 8) return URB_ERR_UNSUPPORTED;
    int ksplit = std::max(need, std::min(std::min(8, ctx->num_sms / std::max(1, nmt)), m->tc_ks));
    auto spc_of = [&](int k) { return (m->tc_ks + k - 1) / k; };
    while (ksplit > need && resident(ksplit, spc_of(ksplit)) < nmt) --ksplit;
    const int spc = spc_of(ksplit);

    MvArgs a{};
    a.tiles = m->tc_tiles;
    a.mts = m->tc_mts;
    a.ks = m->tc_ks;
    a.mt_lo = mt_lo;
    a.spc = spc;
    a.rows = int(m->rows);
    a.cols = int(m->cols);
    a.row_start = (long long)start;
    a.row_count = (long long)count;
    a.x = d_x;
    a.y = d_y;
    a.status = d_status;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = ksplit;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cm = {};
    cm.gridDim = dim3(unsigned(ksplit), unsigned(nmt), 1);
    cm.blockDim = dim3(kMvThreads);
    cm.dynamicSmemBytes = mv_smem(spc);
    cm.stream = st;
    cm.attrs = at;
    cm.numAttrs = mv_pdl() ? 2 : 1;
    URB_CUDA(ctx, cudaLaunchKernelEx(&cm, kern, a));
    return URB_OK;
}

}  // namespace

bool matvec_tc_applies(const Mat *m) {
    return m->tc_tiles && (m->format == URB_FMT_MXFP4 || m->format == URB_FMT_MXFP8);
}

int launch_matvec_tc(Ctx *ctx, const Mat *m, size_t start, size_t count, const float *d_x,
                     float *d_y, int32_t *d_status, cudaStream_t st) {
    if (count == 0) return URB_OK;
    if (!matvec_tc_applies(m)) return URB_ERR_UNSUPPORTED;
    return m->format == URB_FMT_MXFP4
               ? launch_t<URB_FMT_MXFP4>(ctx, m, start, count, d_x, d_y, d_status, st)
               : launch_t<URB_FMT_MXFP8>(ctx, m, start, count, d_x, d_y, d_status, st);
}

}  // namespace urb
