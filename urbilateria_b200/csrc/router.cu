// router.cu — bit-exact expert routing.
//
//  * Router logits: the reference evaluates each logit as a sequential F64 sum, in column
//    order, of exact f64 products bf16(w) * x, starting from -0.0, rounded once to f32
//    (src/model/bf16.rs:494-525 via glm/runtime/moe.rs:154).  A product of a bf16 and an f32
//    is exact in f64, so fma(w, x, acc) equals the reference's multiply-then-add.  The chains
//    run on the FP64 tensor path: mma.sync m8n8k4 f64 advances an 8 x 8 block of chains by four
//    columns as four fused multiply-adds in column order (checked bit for bit against
//    sequential FMA chains on B200), so the logits are bit-identical at a fraction of the
//    latency of dependent DFMAs.
//  * route_noaux_tc (src/math/routing.rs:38-155) and route_softmax_top_k
//    (src/models/qwen3_8/moe.rs:91-159): one warp per token, IEEE f32 arithmetic in the
//    reference's order, libm-exact expf, total_cmp ranking with the lower id winning ties.
#include "expf_glibc.cuh"
#include "urb_internal.cuh"

namespace urb {
namespace {

constexpr int kRouterKc = 64;   // columns staged per tile
constexpr int kRouterWarps = 4;
constexpr int kRouterTpt = 2;   // token chains per thread
constexpr int kRouterTok = kRouterWarps * kRouterTpt;  // tokens per CTA

template <bool BF16>
__device__ __forceinline__ double widen(const void *w, size_t idx) {
    return BF16 ? double(__uint_as_float(uint32_t(static_cast<const uint16_t *>(w)[idx]) << 16))
                : double(static_cast<const float *>(w)[idx]);
}

// CTA = 32 experts x 8 tokens; thread (lane = expert, warp = token pair) owns two chains and
// performs, for each of them, exactly the reference's additions in column order.  The chains
// are latency-bound (one f64 FMA after another), so a thread interleaves two of them and the
// operands come from shared memory without bank conflicts: the experts' weights are staged
// column-major (lane-contiguous), the token pair's x values as one broadcast 16-byte load.
// Column tiles are double-buffered; the next tile is fetched into registers while the current
// one is consumed.
// Sigmoid gate and biased selection score of one logit (routing.rs:101-105), libm-exact.
__device__ __forceinline__ void gate_of(float l, float b, const ExpfTable &tab, float *gate,
                                        float *sel, int32_t *status) {
    if (!isfinite(l) || !isfinite(b)) atomicCAS(status, 0, int32_t(URB_ERR_NONFINITE));
    const float gv = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf_libm(-l, tab)));
    *gate = gv;
    *sel = __fadd_rn(gv, b);
}

// Optional epilogue of the logits kernel: the route_noaux_tc gates and selection scores of
// every (token, expert), so that the routing kernel only ranks.
struct GateOut {
    const float *bias;
    float *gate, *sel;
    int32_t *status;
    ExpfTable tab;
};

template <bool BF16>
__global__ void __launch_bounds__(32 * kRouterWarps) k_router_logits(const void *w, int experts,
                                                                     int cols, const float *x,
                                                                     int tokens, float *logits,
                                                                     GateOut go) {
    constexpr int KC = kRouterKc, NT = 32 * kRouterWarps;
    constexpr int WPT = 32 * KC / NT;          // weights fetched per thread per tile (16)
    constexpr int XPT = kRouterTok * KC / NT;  // x values fetched per thread per tile (4)
    __shared__ __align__(16) double ws[2][KC][32];
    __shared__ __align__(16) double xs[2][KC][kRouterTok];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int e0 = blockIdx.x * 32, t0 = blockIdx.y * kRouterTok;
    const int ntiles = (cols + KC - 1) / KC;
    // Fetch geometry: weights row wr_r, columns wr_c .. +WPT; x row xr_r, columns xr_c .. +XPT.
    const int wr_r = threadIdx.x / (KC / WPT), wr_c = (threadIdx.x % (KC / WPT)) * WPT;
    const int xr_r = threadIdx.x / (KC / XPT), xr_c = (threadIdx.x % (KC / XPT)) * XPT;
    double wr[WPT], xr[XPT];
    auto fetch = [&](int tile) {
        const int c0 = tile * KC;
        const bool wrow = e0 + wr_r < experts, xrow = t0 + xr_r < tokens;
#pragma unroll
        for (int j = 0; j < WPT; ++j) {
            const int c = c0 + wr_c + j;
            wr[j] = (wrow && c < cols) ? widen<BF16>(w, size_t(e0 + wr_r) * cols + c) : 0.0;
        }
#pragma unroll
        for (int j = 0; j < XPT; ++j) {
            const int c = c0 + xr_c + j;
            xr[j] = (xrow && c < cols) ? double(x[size_t(t0 + xr_r) * cols + c]) : 0.0;
        }
    };
    auto stash = [&](int buf) {
#pragma unroll
        for (int j = 0; j < WPT; ++j) ws[buf][wr_c + j][wr_r] = wr[j];
#pragma unroll
        for (int j = 0; j < XPT; ++j) xs[buf][xr_c + j][xr_r] = xr[j];
    };
    fetch(0);
    stash(0);
    __syncthreads();
    // Iterator::sum over f64 starts from -0.0 (bf16.rs:500).
    double acc0 = -0.0, acc1 = -0.0;
    for (int tile = 0; tile < ntiles; ++tile) {
        const int buf = tile & 1;
        if (tile + 1 < ntiles) fetch(tile + 1);
        const int kc = min(KC, cols - tile * KC);
        // Exactly the reference's additions: columns in order, one rounding each.
        if (kc == KC) {
#pragma unroll 16
            for (int c = 0; c < KC; ++c) {
                const double wv = ws[buf][c][lane];
                const double2 xv = *reinterpret_cast<const double2 *>(&xs[buf][c][kRouterTpt * warp]);
                acc0 = fma(wv, xv.x, acc0);
                acc1 = fma(wv, xv.y, acc1);
            }
        } else {
            for (int c = 0; c < kc; ++c) {
                const double wv = ws[buf][c][lane];
                const double2 xv = *reinterpret_cast<const double2 *>(&xs[buf][c][kRouterTpt * warp]);
                acc0 = fma(wv, xv.x, acc0);
                acc1 = fma(wv, xv.y, acc1);
            }
        }
        if (tile + 1 < ntiles) stash(buf ^ 1);
        __syncthreads();
    }
    const int e = e0 + lane, t = t0 + kRouterTpt * warp;
    if (e < experts) {
        const float l0 = float(acc0), l1 = float(acc1);
        if (t < tokens) logits[size_t(t) * experts + e] = l0;
        if (t + 1 < tokens) logits[size_t(t + 1) * experts + e] = l1;
        if (go.gate) {
            const float b = go.bias[e];
            const size_t i0 = size_t(t) * experts + e, i1 = i0 + experts;
            if (t < tokens) gate_of(l0, b, go.tab, go.gate + i0, go.sel + i0, go.status);
            if (t + 1 < tokens) gate_of(l1, b, go.tab, go.gate + i1, go.sel + i1, go.status);
        }
    }
}

// Widens a bf16 (BF16) or f32 matrix to f64 (exact), grid-stride.
template <bool BF16>
__global__ void k_to_f64(const void *src, size_t n, double *dst) {
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n;
         i += size_t(gridDim.x) * blockDim.x)
        dst[i] = widen<BF16>(src, i);
}

__device__ __forceinline__ void dmma_8x8x4(double &d0, double &d1, double a, double b) {
    asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0,%1}, {%2}, {%3}, {%0,%1};"
                 : "+d"(d0), "+d"(d1)
                 : "d"(a), "d"(b));
}

// One warp per 8 tokens x 8 experts, one warp per CTA so that the 512 blocks of a 128-token,
// 256-expert forward spread over every SM (the FP64 path is throughput-bound per SM: CTAs of
// four warps measured 1.9x slower).  A = x (row: token, k: column), B = router (k:
// column, n: expert); lane q holds A[q/4][q%4], B[q%4][q/4] and D[q/4][2(q%4) .. +1].  The
// columns past the last multiple of four are added by each lane with scalar FMAs, in order.
constexpr int kDmmaWarps = 1;
__global__ void __launch_bounds__(32 * kDmmaWarps) k_router_dmma(const double *x64,
                                                                 const double *w64, int tokens,
                                                                 int experts, int cols,
                                                                 float *logits, GateOut go) {
    const int lane = threadIdx.x & 31;
    const int eblk = (experts + 7) / 8;
    const int blk = blockIdx.x * kDmmaWarps + (threadIdx.x >> 5);
    if (blk >= eblk * ((tokens + 7) / 8)) return;
    const int tb = blk / eblk, eb = blk % eblk;
    const int ar = tb * 8 + (lane >> 2), bc = eb * 8 + (lane >> 2), kq = lane & 3;
    const bool arow = ar < tokens, bcol = bc < experts;
    const double *xa = x64 + size_t(arow ? ar : 0) * cols + kq;
    const double *wb = w64 + size_t(bcol ? bc : 0) * cols + kq;
    double d0 = -0.0, d1 = -0.0;  // Iterator::sum over f64 starts from -0.0 (bf16.rs:500)
    const int k4 = cols & ~3;
#pragma unroll 8
    for (int k = 0; k < k4; k += 4) {
        const double a = arow ? xa[k] : 0.0, b = bcol ? wb[k] : 0.0;
        dmma_8x8x4(d0, d1, a, b);
    }
    const int t = tb * 8 + (lane >> 2), e0 = eb * 8 + 2 * (lane & 3);
    if (k4 < cols && t < tokens) {
        const double *xr = x64 + size_t(t) * cols;
        for (int k = k4; k < cols; ++k) {
            if (e0 < experts) d0 = fma(w64[size_t(e0) * cols + k], xr[k], d0);
            if (e0 + 1 < experts) d1 = fma(w64[size_t(e0 + 1) * cols + k], xr[k], d1);
        }
    }
    if (t >= tokens) return;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int e = e0 + i;
        if (e >= experts) continue;
        const float l = float(i ? d1 : d0);
        const size_t o = size_t(t) * experts + e;
        logits[o] = l;
        if (go.gate) gate_of(l, go.bias[e], go.tab, go.gate + o, go.sel + o, go.status);
    }
}

__device__ __forceinline__ bool better(int32_t ka, int ia, int32_t kb, int ib) {
    return ka > kb || (ka == kb && ia < ib);
}

// Warp argmax over (key desc, id asc).
__device__ __forceinline__ void warp_best(int32_t &key, int &id) {
    for (int o = 16; o > 0; o >>= 1) {
        int32_t k2 = __shfl_xor_sync(0xffffffffu, key, o);
        int i2 = __shfl_xor_sync(0xffffffffu, id, o);
        if (better(k2, i2, key, id)) { key = k2; id = i2; }
    }
}

__device__ __forceinline__ void set_status(int32_t *status, int code) {
    if (status) atomicCAS(status, 0, int32_t(code));
}

// One warp per token.  Shared memory per warp (warp_bytes): gate[E], sel[E], group score
// [n_group] floats, then one flag byte per expert (1 allowed, 2 taken, 0 masked).  PRE: the
// gates and selection scores come precomputed (logits kernel epilogue, which also reported
// non-finite logits or biases) in `logits` / `bias` as [tokens, E] arrays.
template <bool PRE>
__global__ void k_route_noaux(const float *logits, const float *bias, int tokens, int E,
                              int top_k, int n_group, int topk_group, int normalize,
                              float scaling, ExpfTable tab, int32_t *out_e, float *out_w,
                              float *out_s, int32_t *status, int warp_bytes) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * (blockDim.x >> 5) + warp;
    if (t >= tokens) return;
    float *gate = reinterpret_cast<float *>(smem + size_t(warp) * warp_bytes);
    float *sel = gate + E;
    float *gscore = sel + E;
    uint8_t *flags = reinterpret_cast<uint8_t *>(gscore + n_group);
    const float *lg = logits + size_t(t) * E;
    bool bad = false;
    if (PRE) {
        const float *sg = bias + size_t(t) * E;
        for (int i = lane; i < E; i += 32) {
            gate[i] = lg[i];
            sel[i] = sg[i];
            flags[i] = 1;
        }
    }
    // routing.rs:103: gate = 1 / (1 + exp(-logit)).  Eight experts per lane at a time, with all
    // of their exception-table loads issued before any is used (independent, in flight together).
    constexpr int kB = 8;
    for (int i0 = 0; !PRE && i0 < E; i0 += 32 * kB) {
        float l[kB], b[kB];
        uint32_t lo[kB], hi[kB];
#pragma unroll
        for (int j = 0; j < kB; ++j) {
            const int i = i0 + 32 * j + lane;
            l[j] = i < E ? lg[i] : 0.0f;
            b[j] = i < E ? bias[i] : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < kB; ++j) {
            const uint32_t bucket = __float_as_uint(-l[j]) >> 12;
            lo[j] = tab.index ? tab.index[bucket] : 0;
            hi[j] = tab.index ? tab.index[bucket + 1] : 0;
        }
#pragma unroll
        for (int j = 0; j < kB; ++j) {
            const int i = i0 + 32 * j + lane;
            if (i >= E) continue;
            bad |= !isfinite(l[j]) || !isfinite(b[j]);
            const float ex = expf_libm_range(-l[j], tab, lo[j], hi[j]);
            const float gv = __fdiv_rn(1.0f, __fadd_rn(1.0f, ex));
            gate[i] = gv;
            sel[i] = __fadd_rn(gv, b[j]);
            flags[i] = 1;
        }
    }
    if (__any_sync(0xffffffffu, bad)) {
        // Rejected token: report, and leave distinct valid ids with zero weight so that the
        // rest of a device pipeline stays in bounds (it short-circuits on the status anyway).
        if (lane == 0) set_status(status, URB_ERR_NONFINITE);
        for (int r = lane; r < top_k; r += 32) {
            out_e[size_t(t) * top_k + r] = r;
            out_w[size_t(t) * top_k + r] = 0.0f;
            if (out_s) out_s[size_t(t) * top_k + r] = 0.0f;
        }
        return;
    }
    __syncwarp();
    if (n_group > 1) {
        // routing.rs:112-129: group score = sum of the two largest selections (total order).
        const int gs = E / n_group;
        for (int grp = lane; grp < n_group; grp += 32) {
            int32_t k1 = INT32_MIN, k2 = INT32_MIN;
            float v1 = 0.0f, v2 = 0.0f;
            for (int i = grp * gs; i < (grp + 1) * gs; ++i) {
                int32_t k = total_key(sel[i]);
                if (k > k1) { k2 = k1; v2 = v1; k1 = k; v1 = sel[i]; }
                else if (k > k2) { k2 = k; v2 = sel[i]; }
            }
            gscore[grp] = __fadd_rn(v1, v2);
        }
        __syncwarp();
        // Groups ranked by score desc, lower group id first; the best topk_group stay allowed.
        for (int grp = lane; grp < n_group; grp += 32) {
            const int32_t kg = total_key(gscore[grp]);
            int rank = 0;
            for (int o = 0; o < n_group; ++o)
                if (better(total_key(gscore[o]), o, kg, grp)) ++rank;
            const uint8_t allowed = rank < topk_group ? 1 : 0;
            for (int i = grp * gs; i < (grp + 1) * gs; ++i) flags[i] = allowed;
        }
        __syncwarp();
    }
    // routing.rs:131-141: top_k by selection desc, lower id wins ties.  The chosen ids go
    // straight to the output row; lane 0 accumulates the f32 denominator in ranking order.
    int32_t *oe = out_e + size_t(t) * top_k;
    float den = -0.0f;
    for (int r = 0; r < top_k; ++r) {
        int32_t key = INT32_MIN;
        int id = INT32_MAX;
        for (int i = lane; i < E; i += 32) {
            if (flags[i] == 1) {
                int32_t k = total_key(sel[i]);
                if (better(k, i, key, id)) { key = k; id = i; }
            }
        }
        warp_best(key, id);
        if (id == INT32_MAX) {  // fewer allowed experts than top_k
            if (lane == 0) set_status(status, URB_ERR_INVALID_GEOMETRY);
            for (int r2 = lane; r2 < top_k; r2 += 32) {
                out_e[size_t(t) * top_k + r2] = r2;
                out_w[size_t(t) * top_k + r2] = 0.0f;
            }
            return;
        }
        if (lane == (id & 31)) flags[id] = 2;
        if (lane == 0) {
            oe[r] = id;
            den = __fadd_rn(den, gate[id]);
        }
        __syncwarp();
    }
    if (lane == 0) {
        den = __fadd_rn(den, 1e-20f);  // routing.rs:143-146
        if (normalize && !isfinite(den)) {
            set_status(status, URB_ERR_NONFINITE);
            return;
        }
    }
    den = __shfl_sync(0xffffffffu, den, 0);
    for (int r = lane; r < top_k; r += 32) {
        const int id = oe[r];
        const float w = normalize ? __fdiv_rn(gate[id], den) : gate[id];
        out_w[size_t(t) * top_k + r] = __fmul_rn(w, scaling);
        if (out_s) out_s[size_t(t) * top_k + r] = sel[id];
    }
}

// route_softmax_top_k (src/models/qwen3_8/moe.rs:108-158).  One warp per token.
__global__ void k_route_softmax(const float *logits, int tokens, int E, int top_k,
                                ExpfTable tab, int32_t *out_e, float *out_w, int32_t *status) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * (blockDim.x >> 5) + warp;
    if (t >= tokens) return;
    float *p = reinterpret_cast<float *>(smem) + size_t(warp) * E;
    uint8_t *taken = smem + size_t(blockDim.x >> 5) * E * 4 + size_t(warp) * E;
    const float *lg = logits + size_t(t) * E;
    float mx = -INFINITY;
    bool bad = false;
    for (int i = lane; i < E; i += 32) {
        float l = lg[i];
        bad |= !isfinite(l);
        mx = fmaxf(mx, l);
        taken[i] = 0;
    }
    if (__any_sync(0xffffffffu, bad)) {
        if (lane == 0) set_status(status, URB_ERR_NONFINITE);
        return;
    }
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    for (int i = lane; i < E; i += 32) p[i] = expf_libm(__fsub_rn(lg[i], mx), tab);
    __syncwarp();
    float den = 0.0f;
    if (lane == 0)
        for (int i = 0; i < E; ++i) den = __fadd_rn(den, p[i]);
    den = __shfl_sync(0xffffffffu, den, 0);
    if (!isfinite(den) || den <= 0.0f) {
        if (lane == 0) set_status(status, URB_ERR_NONFINITE);
        return;
    }
    for (int i = lane; i < E; i += 32) p[i] = __fdiv_rn(p[i], den);
    __syncwarp();
    int32_t *oe = out_e + size_t(t) * top_k;
    float selected = 0.0f;
    for (int r = 0; r < top_k; ++r) {
        int32_t key = INT32_MIN;
        int id = INT32_MAX;
        for (int i = lane; i < E; i += 32)
            if (!taken[i]) {
                int32_t k = total_key(p[i]);
                if (better(k, i, key, id)) { key = k; id = i; }
            }
        warp_best(key, id);
        if (lane == (id & 31)) taken[id] = 1;
        if (lane == 0) {
            oe[r] = id;
            selected = __fadd_rn(selected, p[id]);
        }
        __syncwarp();
    }
    selected = __shfl_sync(0xffffffffu, selected, 0);
    if (!isfinite(selected) || selected <= 0.0f) {
        if (lane == 0) set_status(status, URB_ERR_NONFINITE);
        return;
    }
    for (int r = lane; r < top_k; r += 32) {
        const float w = __fdiv_rn(p[oe[r]], selected);
        if (!isfinite(w)) set_status(status, URB_ERR_NONFINITE);
        out_w[size_t(t) * top_k + r] = w;
    }
}

}  // namespace

namespace {

ExpfTable table_of(const Ctx *ctx) { return ExpfTable{ctx->expf_keys, ctx->expf_vals, ctx->expf_index}; }

}  // namespace

int launch_router_logits(const Mat *router, const float *d_x, int tokens, float *d_logits,
                         cudaStream_t st, const RouterGates *rg) {
    if (tokens <= 0) return URB_OK;
    GateOut go{};
    if (rg) go = GateOut{rg->bias, rg->gate, rg->sel, rg->status, table_of(rg->ctx)};
    dim3 grid(unsigned((router->rows + 31) / 32), unsigned((tokens + kRouterTok - 1) / kRouterTok));
    constexpr int nt = 32 * kRouterWarps;
    if (router->format == URB_FMT_BF16)
        k_router_logits<true><<<grid, nt, 0, st>>>(router->raw_values, int(router->rows),
                                                   int(router->cols), d_x, tokens, d_logits, go);
    else if (router->format == URB_FMT_F32)
        k_router_logits<false><<<grid, nt, 0, st>>>(router->raw_values, int(router->rows),
                                                    int(router->cols), d_x, tokens, d_logits, go);
    else
        return URB_ERR_UNSUPPORTED;
    return cudaGetLastError() == cudaSuccess ? URB_OK : URB_ERR_CUDA;
}

int widen_router_f64(const Mat *router, double *dst, cudaStream_t st) {
    const size_t n = router->rows * router->cols;
    if (router->format == URB_FMT_BF16)
        k_to_f64<true><<<1024, 256, 0, st>>>(router->raw_values, n, dst);
    else if (router->format == URB_FMT_F32)
        k_to_f64<false><<<1024, 256, 0, st>>>(router->raw_values, n, dst);
    else
        return URB_ERR_UNSUPPORTED;
    return cudaGetLastError() == cudaSuccess ? URB_OK : URB_ERR_CUDA;
}

int launch_router_logits_f64(const double *w64, int experts, const float *d_x, int tokens,
                             int cols, double *x64, float *d_logits, cudaStream_t st,
                             const RouterGates *rg) {
    if (tokens <= 0) return URB_OK;
    GateOut go{};
    if (rg) go = GateOut{rg->bias, rg->gate, rg->sel, rg->status, table_of(rg->ctx)};
    k_to_f64<false><<<512, 256, 0, st>>>(d_x, size_t(tokens) * cols, x64);
    const int blocks = ((tokens + 7) / 8) * ((experts + 7) / 8);
    k_router_dmma<<<(blocks + kDmmaWarps - 1) / kDmmaWarps, 32 * kDmmaWarps, 0, st>>>(
        x64, w64, tokens, experts, cols, d_logits, go);
    return cudaGetLastError() == cudaSuccess ? URB_OK : URB_ERR_CUDA;
}

int launch_route_noaux(Ctx *ctx, const float *d_logits, const float *d_bias, int tokens,
                       int experts, const urb_moe_geometry &g, int32_t *d_expert,
                       float *d_weight, float *d_score, int32_t *d_status, cudaStream_t st,
                       const RouterGates *pre) {
    if (tokens <= 0) return URB_OK;
    int warps = 4;
    int warp_bytes = int(((2 * size_t(experts) + g.n_group) * 4 + experts + 15) & ~size_t(15));
    size_t smem = size_t(warps) * warp_bytes;
    auto k = pre ? k_route_noaux<true> : k_route_noaux<false>;
    k<<<(tokens + warps - 1) / warps, warps * 32, smem, st>>>(
        pre ? pre->gate : d_logits, pre ? pre->sel : d_bias, tokens, experts, int(g.top_k),
        int(g.n_group), int(g.topk_group), g.normalize, g.routed_scaling_factor, table_of(ctx),
        d_expert, d_weight, d_score, d_status, warp_bytes);
    URB_CUDA(ctx, cudaGetLastError());
    return URB_OK;
}

int launch_route_softmax(Ctx *ctx, const float *d_logits, int tokens, int experts, int top_k,
                         int32_t *d_expert, float *d_weight, int32_t *d_status,
                         cudaStream_t st) {
    if (tokens <= 0) return URB_OK;
    int warps = 4;
    size_t smem = size_t(warps) * experts * 5;
    k_route_softmax<<<(tokens + warps - 1) / warps, warps * 32, smem, st>>>(
        d_logits, tokens, experts, top_k, table_of(ctx), d_expert, d_weight, d_status);
    URB_CUDA(ctx, cudaGetLastError());
    return URB_OK;
}

}  // namespace urb
