// gemv_bf16.cu — BF16 products for a few tokens (decode steps and short prefill chunks) on
// CUDA cores: Bf16Matrix::matvec_rows / matmul_rows (src/model/bf16.rs:121-216) and
// GatedMlp::forward (src/model/mlp.rs:90-99) with BF16 projections.
//
// With at most a few dozen tokens every weight byte is used a few dozen times at most, so the
// product is a single streaming pass over the row-major BF16 weights: a warp takes R rows, its
// lanes walk the columns 8 at a time with 16-byte loads (a bf16 widens to f32 by a shift), the
// CTA's token tile of x sits in shared memory and each x read serves R rows, and the warp sum
// of each (row, token) goes to the output.  The SwiGLU form reads the gate and up rows of the
// same index together and writes h = silu(gate . x) * (up . x).  Sums are in f32 (each lane's
// columns, then the warp tree), a fixed order, so results are deterministic.
#include "urb_internal.cuh"

namespace urb {
namespace {

constexpr int kGvWarps = 4;

__device__ __forceinline__ void widen8(uint4 q, float *w) {
    const uint32_t v[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        w[2 * i] = __uint_as_float(v[i] << 16);
        w[2 * i + 1] = __uint_as_float(v[i] & 0xffff0000u);
    }
}

// Rows [row0 + (blockIdx.x * kGvWarps + warp) * R, + R) of `w` (and of `w2` for SwiGLU) times
// tokens [blockIdx.y * TT, + TT) of x (row-major [tokens, cols]); output row t at
// y + t * y_stride, column = row - row0.  Non-finite x sets status.
template <int TT, int R, int NCH, bool SWIGLU>
__global__ void __launch_bounds__(32 * kGvWarps) k_gemv_bf16(const uint16_t *w, const uint16_t *w2,
                                                             int row0, int nrows, int cols,
                                                             const float *x, int tokens, float *y,
                                                             int y_stride, int32_t *status) {
    constexpr int M = SWIGLU ? 2 : 1;
    extern __shared__ __align__(16) float xs[];  // [TT][colsp], zero past cols and tokens
    const int colsp = (cols + 7) & ~7;
    const int t0 = blockIdx.y * TT;
    const int nt = min(TT, tokens - t0);
    // The token tile of x into shared memory, eight 16-byte loads in flight per thread.
    bool bad = false;
    const bool xvec = (cols & 3) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
    const int n4 = TT * colsp / 4;
    for (int i0 = threadIdx.x; i0 < n4; i0 += 8 * blockDim.x) {
        float4 v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int i = i0 + j * blockDim.x;
            const int t = 4 * i / colsp, c = 4 * i - t * colsp;
            v[j] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (i < n4 && t < nt) {
                const float *src = x + size_t(t0 + t) * cols + c;
                if (xvec && c + 4 <= cols) {
                    v[j] = __ldg(reinterpret_cast<const float4 *>(src));
                } else {
                    float e[4];
#pragma unroll
                    for (int k = 0; k < 4; ++k) e[k] = c + k < cols ? src[k] : 0.0f;
                    v[j] = make_float4(e[0], e[1], e[2], e[3]);
                }
            }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int i = i0 + j * blockDim.x;
            if (i < n4) {
                bad |= !isfinite(v[j].x) || !isfinite(v[j].y) || !isfinite(v[j].z) || !isfinite(v[j].w);
                reinterpret_cast<float4 *>(xs)[i] = v[j];
            }
        }
    }
    if (bad && status) atomicCAS(status, 0, int32_t(URB_ERR_NONFINITE));
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rl = (blockIdx.x * kGvWarps + warp) * R;  // first row of this warp, relative
    if (rl >= nrows) return;
    float acc[M][R][TT];
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int t = 0; t < TT; ++t) acc[m][r][t] = 0.0f;
    // Rows past the matrix read its last row (their sums are never stored).
    int rowc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) rowc[r] = row0 + min(rl + r, nrows - 1);
    auto fma8 = [&](const float (&wv)[8], int m, int r, int c) {
#pragma unroll
        for (int t = 0; t < TT; ++t) {
            if (t >= nt) break;
            const float4 xa = *reinterpret_cast<const float4 *>(xs + t * colsp + c);
            const float4 xb = *reinterpret_cast<const float4 *>(xs + t * colsp + c + 4);
            const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[m][r][t] = fmaf(wv[i], xv[i], acc[m][r][t]);
        }
    };
    if ((cols & 7) == 0) {
        // NCH column chunks of 8 per lane in flight: every 16-byte load of the batch is issued
        // (unconditionally, at a clamped address) before any is used.
        for (int c0 = lane * 8; c0 < cols; c0 += 256 * NCH) {
            uint4 q[NCH][M][R];
#pragma unroll
            for (int j = 0; j < NCH; ++j) {
                const int cc = min(c0 + 256 * j, cols - 8);
#pragma unroll
                for (int m = 0; m < M; ++m)
#pragma unroll
                    for (int r = 0; r < R; ++r)
                        q[j][m][r] = __ldg(reinterpret_cast<const uint4 *>((m ? w2 : w) + size_t(rowc[r]) * cols + cc));
            }
#pragma unroll
            for (int j = 0; j < NCH; ++j) {
                const int c = c0 + 256 * j;
                if (c >= cols) break;
#pragma unroll
                for (int m = 0; m < M; ++m)
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        float wv[8];
                        widen8(q[j][m][r], wv);
                        fma8(wv, m, r, c);
                    }
            }
        }
    } else {
        for (int c = lane * 8; c < colsp; c += 256) {
#pragma unroll
            for (int m = 0; m < M; ++m)
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    const uint16_t *wr = (m ? w2 : w) + size_t(rowc[r]) * cols;
                    float wv[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        wv[i] = c + i < cols ? __uint_as_float(uint32_t(wr[c + i]) << 16) : 0.0f;
                    fma8(wv, m, r, c);
                }
        }
    }
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int t = 0; t < TT; ++t)
#pragma unroll
                for (int o = 16; o > 0; o >>= 1)
                    acc[m][r][t] += __shfl_xor_sync(0xffffffffu, acc[m][r][t], o);
    if (lane != 0) return;
#pragma unroll
    for (int r = 0; r < R; ++r) {
        if (rl + r >= nrows) break;
#pragma unroll
        for (int t = 0; t < TT; ++t) {
            if (t >= nt) break;
            float v = acc[0][r][t];
            if (SWIGLU) {
                const float gv = acc[0][r][t];
                v = gv / (1.0f + expf(-gv)) * acc[M - 1][r][t];
            }
            y[size_t(t0 + t) * y_stride + rl + r] = v;
        }
    }
}

template <int TT, int R, int NCH, bool SWIGLU>
int launch_t(Ctx *ctx, const uint16_t *w, const uint16_t *w2, int row0, int nrows, int cols,
             const float *x, int tokens, float *y, int y_stride, int32_t *status, cudaStream_t st) {
    const size_t smem = size_t(TT) * ((cols + 7) & ~7) * sizeof(float);
    if (smem > 200 * 1024) return URB_ERR_UNSUPPORTED;
    auto k = k_gemv_bf16<TT, R, NCH, SWIGLU>;
    // The attribute is per function and device; set it on every launch that needs more than
    // the default (contexts on one device may run concurrently, so no cached "granted" value).
    if (smem > 48 * 1024)
        URB_CUDA(ctx, cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
    const dim3 grid(unsigned((nrows + kGvWarps * R - 1) / (kGvWarps * R)), unsigned((tokens + TT - 1) / TT));
    k<<<grid, 32 * kGvWarps, smem, st>>>(w, w2, row0, nrows, cols, x, tokens, y, y_stride, status);
    URB_CUDA(ctx, cudaGetLastError());
    return URB_OK;
}

// One token: a row per warp (many CTAs), 8 chunks in flight; more: a tile of 4 or 8 tokens,
// 2 rows per warp, 4 (4 tokens) or 2 (8 tokens) chunks in flight.
template <bool SWIGLU>
int launch(Ctx *ctx, const uint16_t *w, const uint16_t *w2, int row0, int nrows, int cols,
           const float *x, int tokens, float *y, int y_stride, int32_t *status, cudaStream_t st) {
    if (tokens == 1)
        return launch_t<1, 1, 8, SWIGLU>(ctx, w, w2, row0, nrows, cols, x, tokens, y, y_stride, status, st);
    if (tokens <= 4 || size_t(8) * ((cols + 7) & ~7) * 4 > 200 * 1024)
        return launch_t<4, 2, 4, SWIGLU>(ctx, w, w2, row0, nrows, cols, x, tokens, y, y_stride, status, st);
    return launch_t<8, 2, 2, SWIGLU>(ctx, w, w2, row0, nrows, cols, x, tokens, y, y_stride, status, st);
}

}  // namespace

bool bf16_gemv_applies(const Mat *m, size_t tokens) {
    return m->format == URB_FMT_BF16 && m->raw_values && tokens >= 1 && tokens <= kBf16GemvMaxTokens &&
           m->cols <= 12 * 1024;
}

int launch_bf16_gemv(Ctx *ctx, const Mat *m, size_t start, size_t count, const float *d_x,
                     size_t tokens, float *d_y, int32_t *d_status, cudaStream_t st) {
    return launch<false>(ctx, static_cast<const uint16_t *>(m->raw_values), nullptr, int(start),
                         int(count), int(m->cols), d_x, int(tokens), d_y, int(count), d_status, st);
}

int launch_bf16_swiglu(Ctx *ctx, const Mat *g, const Mat *u, const Mat *d, const float *d_x,
                       int tokens, float *d_h, float *d_out, int32_t *d_status, cudaStream_t st) {
    const int H = int(g->cols), I = int(g->rows);
    prof_begin(ctx, URB_K_GATE_UP, st);
    int rc = launch<true>(ctx, static_cast<const uint16_t *>(g->raw_values),
                          static_cast<const uint16_t *>(u->raw_values), 0, I, H, d_x, tokens, d_h, I,
                          d_status, st);
    prof_end(ctx, st);
    if (rc) return rc;
    prof_begin(ctx, URB_K_DOWN, st);
    rc = launch<false>(ctx, static_cast<const uint16_t *>(d->raw_values), nullptr, 0, H, I, d_h, tokens,
                       d_out, H, nullptr, st);
    prof_end(ctx, st);
    return rc;
}

}  // namespace urb
