// matvec.cu — single-token MX matvec (MxFp4Matrix::matvec, src/math/mxfp.rs:1463,1725-1780;
// MxFp8Matrix::matvec, mxfp.rs:660-714) on CUDA cores, for the decode-shaped product
// y[rows] = W[rows, cols] . x[cols].
//
// A single token leaves nothing for a tensor-core tile to amortise; the product is one pass
// over the packed weights, so the kernel is built to keep HBM busy and the SMs out of dependent
// chains: one CTA per 16-row block of the mma tile layout, its warps taking the block's
// 128-column slices in turn, each warp keeping its next batch of 16-byte loads in flight while
// it reduces the current one.  A lane owns rows g and g+8 of one 32-column group per slice (the
// tile's fragment order); it decodes E2M1 / E4M3 with cvt.rn.f16x2.{e2m1x2,e4m3x2} (exact),
// accumulates the group in four f32 chains against x from shared memory, and applies the
// group's E8M0 scale (an exact power of two) to the group sum.  Lane and
// warp partial sums are added in a fixed order, so results are deterministic.
#include "urb_internal.cuh"

namespace urb {
namespace {

// Slices a warp holds in registers at once (E4M3 tiles carry twice the bytes per lane).
template <int FMT>
constexpr int mv_batch() { return FMT == URB_FMT_MXFP4 ? 8 : 4; }

__device__ __forceinline__ float pow2_e8m0(uint32_t s) {
    // 2^(s-127): normal for s >= 1, the subnormal 2^-127 for s == 0 (s == 0xFF is rejected at
    // upload).
    return s ? __uint_as_float(s << 23) : __uint_as_float(1u << 22);
}

__device__ __forceinline__ float2 h2f(uint32_t h) {
    return __half22float2(*reinterpret_cast<const __half2 *>(&h));
}

// Dot of 32 E2M1 values (16 bytes, low nibble first) with x[0..31]: four accumulation chains
// (word i feeds chain i), added in a fixed order.
__device__ __forceinline__ float dot32_e2m1(uint4 w, const float4 *x4) {
    const uint32_t words[4] = {w.x, w.y, w.z, w.w};
    float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        uint32_t h[4];
        asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
            "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
            "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
            "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
            "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
            "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
            : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
            : "r"(words[i]));
        const float4 xa = x4[2 * i], xb = x4[2 * i + 1];
        const float2 a = h2f(h[0]), b = h2f(h[1]), c = h2f(h[2]), d = h2f(h[3]);
        s[i] = fmaf(a.x, xa.x, s[i]);
        s[i] = fmaf(a.y, xa.y, s[i]);
        s[i] = fmaf(b.x, xa.z, s[i]);
        s[i] = fmaf(b.y, xa.w, s[i]);
        s[i] = fmaf(c.x, xb.x, s[i]);
        s[i] = fmaf(c.y, xb.y, s[i]);
        s[i] = fmaf(d.x, xb.z, s[i]);
        s[i] = fmaf(d.y, xb.w, s[i]);
    }
    return (s[0] + s[1]) + (s[2] + s[3]);
}

// Dot of 32 E4M3 values (32 bytes) with x[0..31]: four accumulation chains (words 2i, 2i + 1
// feed chain i), added in a fixed order.
__device__ __forceinline__ float dot32_e4m3(uint4 w0, uint4 w1, const float4 *x4) {
    const uint32_t words[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        uint32_t h[2];
        asm("{\n\t.reg .b16 s0, s1;\n\t"
            "mov.b32 {s0, s1}, %2;\n\t"
            "cvt.rn.f16x2.e4m3x2 %0, s0;\n\t"
            "cvt.rn.f16x2.e4m3x2 %1, s1;\n\t}"
            : "=r"(h[0]), "=r"(h[1])
            : "r"(words[i]));
        const float4 xa = x4[i];
        const float2 a = h2f(h[0]), b = h2f(h[1]);
        float &t = s[i >> 1];
        t = fmaf(a.x, xa.x, t);
        t = fmaf(a.y, xa.y, t);
        t = fmaf(b.x, xa.z, t);
        t = fmaf(b.y, xa.w, t);
    }
    return (s[0] + s[1]) + (s[2] + s[3]);
}

template <int FMT, int WARPS>
__global__ void __launch_bounds__(32 * WARPS) k_matvec1(const uint8_t *tiles, int rb_lo, int kslices,
                                                        const float *x, int cols, float *y,
                                                        size_t row_start, size_t row_count) {
    constexpr int TB = tile_bytes(FMT);
    constexpr int PAY = tile_payload_bytes(FMT);
    constexpr int LANE_BYTES = PAY / 32;  // rows g and g+8 of one 32-column group
    constexpr int V = LANE_BYTES / 16;     // uint4 per lane per slice (2: E2M1, 4: E4M3)
    extern __shared__ __align__(16) float xs[];  // [kslices * 128], zero past cols
    __shared__ float red[WARPS][16];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, q = lane & 3;
    const int rb = rb_lo + blockIdx.x;
    const uint8_t *base = tiles + size_t(rb) * kslices * TB;

    // Warp w takes slices w, w + WARPS, ... of the row block in batches of B, double-buffered:
    // the next batch's 16-byte loads are in flight while the current batch is reduced.
    constexpr int B = mv_batch<FMT>() / 2;
    const int nmine = kslices > warp ? (kslices - warp + WARPS - 1) / WARPS : 0;
    float acc0 = 0.0f, acc1 = 0.0f;  // rows g and g+8
    uint4 wc[B][V], wn[B][V];
    uint32_t scc[B], scn[B];
    auto load = [&](uint4 (&w)[B][V], uint32_t (&sc)[B], int j0) {
#pragma unroll
        for (int i = 0; i < B; ++i) {
            if (j0 + i < nmine) {
                const uint8_t *t = base + size_t(warp + WARPS * (j0 + i)) * TB;
#pragma unroll
                for (int v = 0; v < V; ++v)
                    w[i][v] = __ldg(reinterpret_cast<const uint4 *>(t + lane * LANE_BYTES) + v);
                sc[i] = __ldg(reinterpret_cast<const uint16_t *>(t + PAY) + lane);
            }
        }
    };
    load(wc, scc, 0);
    {
        // x into shared memory once (its latency overlaps the weight loads in flight): all of a
        // thread's 16-byte loads are issued before any is stored.
        constexpr int XV = 8;  // float4 per thread per round
        const int n4 = kslices * 32;  // float4 of the padded x
        const bool vec = (cols & 3) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
        for (int i0 = threadIdx.x; i0 < n4; i0 += 32 * WARPS * XV) {
            float4 v[XV];
#pragma unroll
            for (int j = 0; j < XV; ++j) {
                const int i = i0 + j * 32 * WARPS;
                v[j] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                if (i < n4 && 4 * i < cols) {
                    if (vec) {
                        v[j] = __ldg(reinterpret_cast<const float4 *>(x) + i);
                    } else {
                        float e[4];
                        for (int k = 0; k < 4; ++k) e[k] = 4 * i + k < cols ? x[4 * i + k] : 0.0f;
                        v[j] = make_float4(e[0], e[1], e[2], e[3]);
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < XV; ++j) {
                const int i = i0 + j * 32 * WARPS;
                if (i < n4) reinterpret_cast<float4 *>(xs)[i] = v[j];
            }
        }
        __syncthreads();
    }
    for (int j0 = 0; j0 < nmine; j0 += B) {
        if (j0 + B < nmine) load(wn, scn, j0 + B);
#pragma unroll
        for (int i = 0; i < B; ++i) {
            if (j0 + i >= nmine) break;
            const int s = warp + WARPS * (j0 + i);
            const float4 *x4 = reinterpret_cast<const float4 *>(xs + s * 128 + q * 32);
            float p0, p1;
            if (FMT == URB_FMT_MXFP4) {
                p0 = dot32_e2m1(wc[i][0], x4);
                p1 = dot32_e2m1(wc[i][V - 1], x4);
            } else {
                p0 = dot32_e4m3(wc[i][0], wc[i][1], x4);
                p1 = dot32_e4m3(wc[i][V - 2], wc[i][V - 1], x4);
            }
            acc0 = fmaf(p0, pow2_e8m0(scc[i] & 0xff), acc0);
            acc1 = fmaf(p1, pow2_e8m0(scc[i] >> 8), acc1);
        }
#pragma unroll
        for (int i = 0; i < B; ++i) {
            scc[i] = scn[i];
#pragma unroll
            for (int v = 0; v < V; ++v) wc[i][v] = wn[i][v];
        }
    }
    // Column groups of a row sit in lanes 4g .. 4g+3.
    acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
    acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
    acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
    acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
    if (q == 0) {
        red[warp][g] = acc0;
        red[warp][g + 8] = acc1;
    }
    __syncthreads();
    if (threadIdx.x < 16) {
        float v = 0.0f;
#pragma unroll
        for (int i = 0; i < WARPS; ++i) v += red[i][threadIdx.x];
        const size_t row = size_t(rb) * 16 + threadIdx.x;
        if (row >= row_start && row < row_start + row_count) y[row - row_start] = v;
    }
}

}  // namespace

// Rows [start, start + count) of a tiled MX matrix times one x vector (device pointers).
int launch_matvec1(Ctx *ctx, const Mat *m, size_t start, size_t count, const float *d_x,
                   float *d_y, cudaStream_t st) {
    if (count == 0) return URB_OK;
    const int rb_lo = int(start / 16), rb_hi = int((start + count + 15) / 16);
    const size_t smem = size_t(m->kslices) * 128 * sizeof(float);
    if (smem > 200 * 1024) return URB_ERR_UNSUPPORTED;
    if (m->format == URB_FMT_MXFP4) {
        auto k = k_matvec1<URB_FMT_MXFP4, 8>;
        URB_CUDA(ctx, cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
        k<<<rb_hi - rb_lo, 256, smem, st>>>(m->tiles, rb_lo, m->kslices, d_x, int(m->cols), d_y,
                                            start, count);
    } else if (m->format == URB_FMT_MXFP8) {
        auto k = k_matvec1<URB_FMT_MXFP8, 16>;
        URB_CUDA(ctx, cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
        k<<<rb_hi - rb_lo, 512, smem, st>>>(m->tiles, rb_lo, m->kslices, d_x, int(m->cols), d_y,
                                            start, count);
    } else {
        return URB_ERR_UNSUPPORTED;
    }
    URB_CUDA(ctx, cudaGetLastError());
    return URB_OK;
}

}  // namespace urb
