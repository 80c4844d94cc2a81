// skinny.cu — grouped "skinny" products for the routed-expert path: decode matvecs, small
// token batches and ragged per-expert groups (N <= 16 activation columns per pass).
//
// Design (B200): the pass is HBM-bound, so the kernel is organised around streaming the weight
// bytes exactly once at full bandwidth and spending as few instructions per weight as possible.
//  * Work space: the concatenated rows of all segments; CTA i of a 148-CTA grid (one per SM)
//    owns rows [i*R/G, (i+1)*R/G), so every SM streams the same number of weight bytes.
//  * Weights arrive through a per-warp cp.async ring (16 B per lane per copy, masked rows are
//    zero-filled without touching HBM) in the tiled layout, so one warp reads one contiguous
//    1-4 KB tile per 16x128 block.
//  * Each lane decodes its own 32-column group of two rows straight into mma.sync A fragments:
//    MXFP4 via cvt.rn.f16x2.e2m1x2, MXFP8 via cvt.rn.f16x2.e4m3x2, one HMUL2 per two weights for
//    the E8M0 scale (exact: powers of two inside the f16 range by construction); BF16 needs no
//    decode.  The tensor core is used as a register-sourced dot-product engine; decoded weights
//    never round-trip through shared memory.
//  * Activations (<= 16 columns: tokens, or token hi/lo halves) are converted once per segment
//    into shared memory in fragment order (conflict-free 8-byte loads).
//  * Epilogue: exact power-of-two rescale, optional SwiGLU of a gate/up pair, store.
#include "numerics.cuh"
#include "urb_internal.cuh"

namespace urb {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

__device__ __forceinline__ uint32_t pow2_h2(int k) {
    // f16 bits of 2^k replicated in both halves; k clamped to the f16 range.  Out-of-range k
    // only occurs for zero-padded groups, whose weights are zero.
    k = max(-24, min(15, k));
    uint32_t h = k >= -14 ? uint32_t(k + 15) << 10 : 1u << (k + 24);
    return h | (h << 16);
}

__device__ __forceinline__ uint32_t hmul2_bits(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

// 4 bytes (8 E2M1 nibbles, low nibble first) -> 4 f16x2 (element 2i in the low half).
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

// 4 bytes (4 E4M3FN values) -> 2 f16x2.
__device__ __forceinline__ void e4m3x4_to_f16(uint32_t w, uint32_t *d) {
    asm("{\n\t.reg .b16 h0, h1;\n\t"
        "mov.b32 {h0, h1}, %2;\n\t"
        "cvt.rn.f16x2.e4m3x2 %0, h0;\n\t"
        "cvt.rn.f16x2.e4m3x2 %1, h1;\n\t}"
        : "=r"(d[0]), "=r"(d[1])
        : "r"(w));
}

template <bool BF16>
__device__ __forceinline__ void mma16816(float *c, const uint32_t *a, uint32_t b0, uint32_t b1) {
    if (BF16) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
            "{%8,%9}, {%0,%1,%2,%3};"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    } else {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
            "{%8,%9}, {%0,%1,%2,%3};"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
}

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem, bool valid) {
    uint32_t s = uint32_t(__cvta_generic_to_shared(smem));
    int n = valid ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(n));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N)); }

// Copies this lane's slice of one tile (own rows only; masked rows are zero-filled).
template <int FMT>
__device__ __forceinline__ void copy_tile(uint8_t *dst, const uint8_t *src, int lane, bool vg,
                                          bool vg8) {
    constexpr int half = tile_payload_bytes(FMT) / 64;  // bytes per row per lane
    constexpr int chunks = half / 16;
#pragma unroll
    for (int c = 0; c < chunks; ++c) {
        cp_async16(dst + lane * 2 * half + c * 16, src + lane * 2 * half + c * 16, vg);
        cp_async16(dst + lane * 2 * half + half + c * 16, src + lane * 2 * half + half + c * 16, vg8);
    }
    if (FMT != URB_FMT_BF16 && lane < 4)
        cp_async16(dst + tile_payload_bytes(FMT) + lane * 16,
                   src + tile_payload_bytes(FMT) + lane * 16, true);
}

// Decodes this lane's two rows of a staged tile into f16/bf16 pairs: A0 (row g), A1 (row g+8),
// 16 registers each, element pair j = columns (2j, 2j+1) of the lane's 32-column group.
template <int FMT>
__device__ __forceinline__ void decode_tile(const uint8_t *t, int lane, int e0g, int e0g8,
                                            uint32_t *A0, uint32_t *A1) {
    if (FMT == URB_FMT_MXFP4) {
        uint4 w0 = *reinterpret_cast<const uint4 *>(t + lane * 32);
        uint4 w1 = *reinterpret_cast<const uint4 *>(t + lane * 32 + 16);
        uint32_t sc = *reinterpret_cast<const uint16_t *>(t + 1024 + 2 * lane);
        uint32_t m0 = pow2_h2(int(sc & 0xff) - 127 - e0g);
        uint32_t m1 = pow2_h2(int(sc >> 8) - 127 - e0g8);
        e2m1x8_to_f16(w0.x, A0 + 0); e2m1x8_to_f16(w0.y, A0 + 4);
        e2m1x8_to_f16(w0.z, A0 + 8); e2m1x8_to_f16(w0.w, A0 + 12);
        e2m1x8_to_f16(w1.x, A1 + 0); e2m1x8_to_f16(w1.y, A1 + 4);
        e2m1x8_to_f16(w1.z, A1 + 8); e2m1x8_to_f16(w1.w, A1 + 12);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            A0[j] = hmul2_bits(A0[j], m0);
            A1[j] = hmul2_bits(A1[j], m1);
        }
    } else if (FMT == URB_FMT_MXFP8) {
        const uint4 *p = reinterpret_cast<const uint4 *>(t + lane * 64);
        uint4 a = p[0], b = p[1], c = p[2], d = p[3];
        uint32_t sc = *reinterpret_cast<const uint16_t *>(t + 2048 + 2 * lane);
        uint32_t m0 = pow2_h2(int(sc & 0xff) - 127 - e0g);
        uint32_t m1 = pow2_h2(int(sc >> 8) - 127 - e0g8);
        e4m3x4_to_f16(a.x, A0 + 0); e4m3x4_to_f16(a.y, A0 + 2);
        e4m3x4_to_f16(a.z, A0 + 4); e4m3x4_to_f16(a.w, A0 + 6);
        e4m3x4_to_f16(b.x, A0 + 8); e4m3x4_to_f16(b.y, A0 + 10);
        e4m3x4_to_f16(b.z, A0 + 12); e4m3x4_to_f16(b.w, A0 + 14);
        e4m3x4_to_f16(c.x, A1 + 0); e4m3x4_to_f16(c.y, A1 + 2);
        e4m3x4_to_f16(c.z, A1 + 4); e4m3x4_to_f16(c.w, A1 + 6);
        e4m3x4_to_f16(d.x, A1 + 8); e4m3x4_to_f16(d.y, A1 + 10);
        e4m3x4_to_f16(d.z, A1 + 12); e4m3x4_to_f16(d.w, A1 + 14);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            A0[j] = hmul2_bits(A0[j], m0);
            A1[j] = hmul2_bits(A1[j], m1);
        }
    } else {
        const uint4 *p = reinterpret_cast<const uint4 *>(t + lane * 128);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            uint4 v = p[i];
            A0[4 * i + 0] = v.x; A0[4 * i + 1] = v.y; A0[4 * i + 2] = v.z; A0[4 * i + 3] = v.w;
            uint4 u = p[4 + i];
            A1[4 * i + 0] = u.x; A1[4 * i + 1] = u.y; A1[4 * i + 2] = u.z; A1[4 * i + 3] = u.w;
        }
    }
}

// 8 mma k-steps of one 128-column slice: A pairs (2b, 2b+1) against B fragments from smem.
template <int FMT, int NB>
__device__ __forceinline__ void mma_slice(float (*acc)[4], const uint32_t *A0, const uint32_t *A1,
                                          const uint2 *bfrag, int slice_stride) {
#pragma unroll
    for (int b = 0; b < 8; ++b) {
        uint32_t a[4] = {A0[2 * b], A1[2 * b], A0[2 * b + 1], A1[2 * b + 1]};
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) {
            uint2 f = bfrag[nb * slice_stride + b * 32];
            mma16816<FMT == URB_FMT_BF16>(acc[nb], a, f.x, f.y);
        }
    }
}

__device__ __forceinline__ uint32_t pack_f16(float v, int part) {
    __half h = __float2half_rn(v);
    if (part) h = __float2half_rn(v - __half2float(h));
    return __half_as_ushort(h);
}
__device__ __forceinline__ uint32_t pack_bf16(float v, int part) {
    __nv_bfloat16 h = __float2bfloat16_rn(v);
    if (part) h = __float2bfloat16_rn(v - __bfloat162float(h));
    return __bfloat16_as_ushort(h);
}

// Power-of-two shift of an activation row: explicit (src_shift) or derived from the row's
// ilogb(max|v|) recorded by a SwiGLU epilogue (src_maxexp), so that max|v| * 2^shift < 2^15.
__device__ __forceinline__ int src_shift_of(const GroupArgs &a, int srow) {
    if (a.src_shift) return a.src_shift[srow];
    int e = a.src_maxexp[srow];
    return e > -1000 ? 14 - e : 0;
}

template <int FMT, int NB>
__device__ void fill_b(uint2 *bsm, const Seg &S, const GroupArgs &a, const int hilo) {
    const int entries = NB * S.kslices * 256;
    for (int idx = threadIdx.x; idx < entries; idx += kThreads) {
        int le = idx & 31, b = (idx >> 5) & 7;
        int s = (idx >> 8) % S.kslices, nb = (idx >> 8) / S.kslices;
        int col = nb * 8 + (le >> 2);
        int k0 = s * 128 + (le & 3) * 32 + b * 4;
        int tok = hilo ? col >> 1 : col, part = hilo ? (col & 1) : 0;
        uint2 v = make_uint2(0, 0);
        if (tok < S.ntok) {
            int c = S.col_begin + tok;
            int srow = a.col_src ? a.col_src[c] : c;
            int shift = src_shift_of(a, srow);
            const float *p = a.src + size_t(srow) * a.src_stride;
            uint32_t h[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                float x = (k0 + i < S.cols) ? ldexpf(p[k0 + i], shift) : 0.0f;
                h[i] = FMT == URB_FMT_BF16 ? pack_bf16(x, part) : pack_f16(x, part);
            }
            v.x = h[0] | (h[1] << 16);
            v.y = h[2] | (h[3] << 16);
        }
        bsm[idx] = v;
    }
}

__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + expf(-v)); }

template <int FMT, bool PAIR, int KSPLIT, int NB, int DEPTH>
__global__ void __launch_bounds__(kThreads, 1) k_grouped(GroupArgs a, int kslices_max) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int MATS = PAIR ? 2 : 1;
    constexpr int TB = tile_bytes(FMT);
    constexpr int RB_PER_ROUND = kWarps / KSPLIT;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, q = lane & 3;

    const int total_rows = *a.total_rows;
    const int nsegs = *a.nsegs;
    const int hilo = (a.lofree && *a.lofree) ? 0 : a.hilo;
    if (total_rows <= 0 || nsegs <= 0) return;
    const long r0 = long(total_rows) * blockIdx.x / gridDim.x;
    const long r1 = long(total_rows) * (blockIdx.x + 1) / gridDim.x;
    if (r0 >= r1) return;

    // Shared memory carve-up: [B fragments][per-warp rings][k-split reduction].
    uint2 *bsm = reinterpret_cast<uint2 *>(smem);
    uint8_t *ring = smem + size_t(NB) * kslices_max * 2048;
    uint8_t *my_ring = ring + size_t(warp) * DEPTH * MATS * TB;
    float *red = reinterpret_cast<float *>(ring + size_t(kWarps) * DEPTH * MATS * TB);

    // First segment touching r0 (segments are ordered by row_begin).
    int lo_i = 0, hi_i = nsegs - 1;
    while (lo_i < hi_i) {
        int mid = (lo_i + hi_i + 1) >> 1;
        if (a.segs[mid].row_begin <= r0) lo_i = mid; else hi_i = mid - 1;
    }
    int loaded = -1;
    for (int si = lo_i; si < nsegs; ++si) {
        const Seg S = a.segs[si];
        const long seg_lo = S.row_begin, seg_hi = S.row_begin + 16L * S.rbs;
        if (seg_lo >= r1) break;
        const long lo = max(r0, seg_lo), hi = min(r1, seg_hi);
        if (lo >= hi) continue;
        if (loaded != si) {
            __syncthreads();
            fill_b<FMT, NB>(bsm, S, a, hilo);
            __syncthreads();
            loaded = si;
        }
        const int rb_lo = int((lo - seg_lo) >> 4), rb_hi = int((hi - seg_lo + 15) >> 4);
        for (int rbase = rb_lo; rbase < rb_hi; rbase += RB_PER_ROUND) {
            const int rb = rbase + warp / KSPLIT, kpart = warp % KSPLIT;
            const bool active = rb < rb_hi;
            float acc[MATS][NB][4];
#pragma unroll
            for (int m = 0; m < MATS; ++m)
#pragma unroll
                for (int nb = 0; nb < NB; ++nb)
#pragma unroll
                    for (int i = 0; i < 4; ++i) acc[m][nb][i] = 0.0f;
            const long wrow_g = seg_lo + 16L * rb + g;  // work-space row of lane row g
            const bool vg = active && wrow_g >= lo && wrow_g < hi && 16 * rb + g < S.rows;
            const bool vg8 = active && wrow_g + 8 >= lo && wrow_g + 8 < hi && 16 * rb + g + 8 < S.rows;
            int e0[MATS][2];
            if (active) {
                const int nmine = (S.kslices - kpart + KSPLIT - 1) / KSPLIT;
                const uint8_t *src[MATS];
                src[0] = S.tiles_a + (size_t(rb) * S.kslices) * TB;
                e0[0][0] = S.rexp_a[16 * rb + g];
                e0[0][1] = S.rexp_a[16 * rb + g + 8];
                if (PAIR) {
                    src[MATS - 1] = S.tiles_b + (size_t(rb) * S.kslices) * TB;
                    e0[MATS - 1][0] = S.rexp_b[16 * rb + g];
                    e0[MATS - 1][1] = S.rexp_b[16 * rb + g + 8];
                }
                // Prologue: DEPTH-1 stages in flight.
#pragma unroll
                for (int st = 0; st < DEPTH - 1; ++st) {
                    if (st < nmine) {
                        const int s = kpart + st * KSPLIT;
#pragma unroll
                        for (int m = 0; m < MATS; ++m)
                            copy_tile<FMT>(my_ring + (st * MATS + m) * TB, src[m] + size_t(s) * TB,
                                           lane, vg, vg8);
                    }
                    cp_async_commit();
                }
                for (int j = 0; j < nmine; ++j) {
                    cp_async_wait<DEPTH - 2>();
                    __syncwarp();
                    const int stage = j % DEPTH;
                    const int s = kpart + j * KSPLIT;
                    const uint2 *bfrag = bsm + size_t(s) * 256 + lane;
#pragma unroll
                    for (int m = 0; m < MATS; ++m) {
                        uint32_t A0[16], A1[16];
                        decode_tile<FMT>(my_ring + (stage * MATS + m) * TB, lane, e0[m][0],
                                         e0[m][1], A0, A1);
                        mma_slice<FMT, NB>(acc[m], A0, A1, bfrag, S.kslices * 256);
                    }
                    __syncwarp();
                    const int jn = j + DEPTH - 1;
                    if (jn < nmine) {
                        const int sn = kpart + jn * KSPLIT, stn = jn % DEPTH;
#pragma unroll
                        for (int m = 0; m < MATS; ++m)
                            copy_tile<FMT>(my_ring + (stn * MATS + m) * TB,
                                           src[m] + size_t(sn) * TB, lane, vg, vg8);
                    }
                    cp_async_commit();
                }
                cp_async_wait<0>();
            }
            if (KSPLIT > 1) {
                float *mine = red + size_t(warp) * MATS * NB * 128;
                if (active) {
#pragma unroll
                    for (int m = 0; m < MATS; ++m)
#pragma unroll
                        for (int nb = 0; nb < NB; ++nb)
#pragma unroll
                            for (int i = 0; i < 4; ++i)
                                mine[((m * NB + nb) * 4 + i) * 32 + lane] = acc[m][nb][i];
                }
                __syncthreads();
                if (active && kpart == 0) {
#pragma unroll
                    for (int m = 0; m < MATS; ++m)
#pragma unroll
                        for (int nb = 0; nb < NB; ++nb)
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                float s = 0.0f;
                                for (int kp = 0; kp < KSPLIT; ++kp)
                                    s += red[size_t(warp + kp) * MATS * NB * 128 +
                                             ((m * NB + nb) * 4 + i) * 32 + lane];
                                acc[m][nb][i] = s;
                            }
                }
                __syncthreads();
            }
            if (!active || kpart != 0) continue;
            // Epilogue.  acc[m][nb] = {D[g][2q], D[g][2q+1], D[g+8][2q], D[g+8][2q+1]} of
            // n-block nb; column n = nb*8 + 2q + (0|1).  hilo: column pair = one token.
            const int row_g = 16 * rb + g;
#pragma unroll
            for (int nb = 0; nb < NB; ++nb) {
#pragma unroll
                for (int t2 = 0; t2 < 2; ++t2) {
                    if (hilo && t2 == 1) break;  // warp-uniform
                    const int tok = hilo ? nb * 4 + q : nb * 8 + 2 * q + t2;
                    const bool tok_ok = tok < S.ntok;
                    const int c = S.col_begin + (tok_ok ? tok : 0);
                    int shift = 0;
                    if (tok_ok) shift = src_shift_of(a, a.col_src ? a.col_src[c] : c);
                    float v[MATS][2];
#pragma unroll
                    for (int m = 0; m < MATS; ++m) {
                        const float d0 = t2 ? acc[m][nb][1] : acc[m][nb][0];
                        const float d2 = t2 ? acc[m][nb][3] : acc[m][nb][2];
                        const float lo_r = hilo ? acc[m][nb][0] + acc[m][nb][1] : d0;
                        const float hi_r = hilo ? acc[m][nb][2] + acc[m][nb][3] : d2;
                        v[m][0] = ldexpf(lo_r, e0[m][0] - shift);
                        v[m][1] = ldexpf(hi_r, e0[m][1] - shift);
                    }
                    float *orow = a.out + size_t(c) * a.out_stride;
                    int mexp = -1000;
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const bool valid = tok_ok && (h ? vg8 : vg);
                        float o = v[0][h];
                        if (PAIR && a.variant == 2) {  // Qwen3.6 BF16 boundaries
                            const float act = num_round_bf16(num_silu_libm(num_round_bf16(v[0][h]), a.expf));
                            o = num_round_bf16(__fmul_rn(act, num_round_bf16(v[MATS - 1][h])));
                        } else if (PAIR) {
                            o = silu_f(v[0][h]) * v[MATS - 1][h];
                        } else if (a.variant != 0) {
                            o = num_round_bf16(o);
                        }
                        if (valid && a.variant != 0 && !isfinite(o) && a.status)
                            atomicCAS(a.status, 0, int32_t(URB_ERR_NONFINITE));
                        if (valid) {
                            orow[row_g + 8 * h] = o;
                            if (PAIR && o != 0.0f && isfinite(o)) mexp = max(mexp, ilogbf(o));
                        }
                    }
                    if (PAIR && a.out_maxexp) {
                        // Max over the 8 lanes that share this column (same q).
#pragma unroll
                        for (int off = 4; off < 32; off <<= 1)
                            mexp = max(mexp, __shfl_xor_sync(0xffffffffu, mexp, off));
                        if (g == 0 && mexp > -1000) atomicMax(a.out_maxexp + c, mexp);
                    }
                }
            }
        }
    }
}

template <int FMT, bool PAIR, int KSPLIT, int NB>
int launch_t(const GroupArgs &a, int kslices_max, int grid, cudaStream_t st) {
    constexpr int DEPTH = FMT == URB_FMT_BF16 ? (PAIR ? 2 : 3) : (FMT == URB_FMT_MXFP8 ? 3 : 4);
    constexpr int MATS = PAIR ? 2 : 1;
    size_t smem = size_t(NB) * kslices_max * 2048 + size_t(kWarps) * DEPTH * MATS * tile_bytes(FMT) +
                  (KSPLIT > 1 ? size_t(kWarps) * MATS * NB * 128 * 4 : 0);
    if (smem > 227 * 1024) return URB_ERR_UNSUPPORTED;
    auto kern = k_grouped<FMT, PAIR, KSPLIT, NB, DEPTH>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return URB_ERR_CUDA;
    kern<<<grid, kThreads, smem, st>>>(a, kslices_max);
    return cudaGetLastError() == cudaSuccess ? URB_OK : URB_ERR_CUDA;
}

template <int FMT, bool PAIR>
int launch_ks(const GroupArgs &a, int ksplit, int nb, int kslices_max, int grid, cudaStream_t st) {
    if (nb == 1) {
        switch (ksplit) {
        case 1: return launch_t<FMT, PAIR, 1, 1>(a, kslices_max, grid, st);
        case 2: return launch_t<FMT, PAIR, 2, 1>(a, kslices_max, grid, st);
        default: return launch_t<FMT, PAIR, 8, 1>(a, kslices_max, grid, st);
        }
    }
    switch (ksplit) {
    case 1: return launch_t<FMT, PAIR, 1, 2>(a, kslices_max, grid, st);
    case 2: return launch_t<FMT, PAIR, 2, 2>(a, kslices_max, grid, st);
    default: return launch_t<FMT, PAIR, 8, 2>(a, kslices_max, grid, st);
    }
}

}  // namespace

// ksplit_hint: 1, 2 or 8 warps cooperating on one 16-row block (8 for matvec-like passes with
// few rows per SM).  max_cols: activation columns per segment (8 -> one n-block, 16 -> two).
int launch_grouped_ex(Ctx *ctx, int fmt, bool pair, int ksplit, const GroupArgs &args,
                      int max_cols, int kslices_max, cudaStream_t st) {
    int nb = max_cols > 8 ? 2 : 1;
    int grid = ctx->num_sms;
    int rc;
    switch (fmt) {
    case URB_FMT_MXFP4:
        rc = pair ? launch_ks<URB_FMT_MXFP4, true>(args, ksplit, nb, kslices_max, grid, st)
                  : launch_ks<URB_FMT_MXFP4, false>(args, ksplit, nb, kslices_max, grid, st);
        break;
    case URB_FMT_MXFP8:
        rc = pair ? launch_ks<URB_FMT_MXFP8, true>(args, ksplit, nb, kslices_max, grid, st)
                  : launch_ks<URB_FMT_MXFP8, false>(args, ksplit, nb, kslices_max, grid, st);
        break;
    case URB_FMT_BF16:
        rc = pair ? launch_ks<URB_FMT_BF16, true>(args, ksplit, nb, kslices_max, grid, st)
                  : launch_ks<URB_FMT_BF16, false>(args, ksplit, nb, kslices_max, grid, st);
        break;
    default:
        rc = URB_ERR_UNSUPPORTED;
    }
    if (rc == URB_ERR_CUDA) return cuda_fail(ctx, cudaGetLastError(), "grouped skinny launch");
    if (rc == URB_ERR_UNSUPPORTED)
        return set_error(ctx, rc, "grouped pass: shared memory or format out of range");
    return rc;
}

}  // namespace urb
