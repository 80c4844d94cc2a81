// router.cu — bit-exact expert routing.
//
//  * Router logits: the reference evaluates each logit as a sequential F64 sum, in column
//    order, of exact f64 products bf16(w) * x, starting from -0.0, rounded once to f32
//    (src/model/bf16.rs:494-525 via glm/runtime/moe.rs:154).  A product of a bf16 and an f32
//    is exact in f64, so fma(w, x, acc) equals the reference's multiply-then-add.  The chains
//    run on the FP64 tensor path: mma.sync m8n8k4 f64 advances an 8 x 8 block of chains by four
//    columns as four fused multiply-adds in column order (checked bit for bit against
//    sequential FMA chains on B200), so the logits are bit-identical.  A chain is 1,792
//    dependent MMAs for the C2 hidden size; its operands are staged through shared memory by
//    TMA bulk copies several stages ahead, so the chain runs at the MMA latency instead of
//    waiting on L2 for every step.
//  * route_noaux_tc (src/math/routing.rs:38-155) and route_softmax_top_k
//    (src/models/qwen3_8/moe.rs:91-159): one warp per token, IEEE f32 arithmetic in the
//    reference's order, libm-exact expf, total_cmp ranking with the lower id winning ties.
#include "expf_glibc.cuh"
#include "numerics.cuh"
#include "route_noaux.cuh"
#include "tc_common.cuh"
#include "urb_internal.cuh"

namespace urb {
namespace {

// Sigmoid gate and biased selection score of one logit (routing.rs:101-105), libm-exact.
__device__ __forceinline__ void gate_of(float l, float b, const ExpfTable &tab, float *gate,
                                        float *sel, int32_t *status) {
    if ((!isfinite(l) || !isfinite(b)) && status) atomicCAS(status, 0, int32_t(URB_ERR_NONFINITE));
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
__device__ __forceinline__ double widen(const void *w, size_t idx) {
    return BF16 ? double(__uint_as_float(uint32_t(static_cast<const uint16_t *>(w)[idx]) << 16))
                : double(static_cast<const float *>(w)[idx]);
}

__device__ __forceinline__ double lds_f64(uint32_t addr) {
    double v;
    asm volatile("ld.shared.f64 %0, [%1];" : "=d"(v) : "r"(addr));
    return v;
}

__device__ __forceinline__ void dmma_8x8x4(double &d0, double &d1, double a, double b) {
    asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0,%1}, {%2}, {%3}, {%0,%1};"
                 : "+d"(d0), "+d"(d1)
                 : "d"(a), "d"(b));
}

// Widens a bf16 (BF16) or f32 row-major [rows, cols] matrix to f64 in the router's blocked
// layout (exact): blocks of 8 rows, each cut into chunks of kRc columns stored as one
// contiguous [8][kRrow] tile (rows padded to kRrow doubles), chunk-major within the block.
// Rows past `rows`, columns past `cols` and the padding are zero.  One thread per element.
template <bool BF16>
__global__ void k_to_f64_blocked(const void *src, int rows, int cols, double *dst) {
    grid_dep_wait();  // programmatic dependent launch: the kernel ahead has completed
    grid_dep_trigger();
    const int nch = router_chunks(cols);
    const size_t n = size_t((rows + 7) / 8) * nch * 8 * kRrow;
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n;
         i += size_t(gridDim.x) * blockDim.x) {
        const int c = int(i % kRrow);
        const size_t rest = i / kRrow;
        const int r = int(rest % 8);
        const size_t tile = rest / 8;
        const int ch = int(tile % nch), rb = int(tile / nch);
        const int row = rb * 8 + r, col = ch * kRc + c;
        dst[i] = (c < kRc && row < rows && col < cols) ? widen<BF16>(src, size_t(row) * cols + col) : 0.0;
    }
}

// One chain warp per 8 tokens x 8 experts (a block), one block per CTA, so the 512 blocks of a
// 128-token, 256-expert forward spread over every SM.  A = x (row: token, k: column), B =
// router (k: column, n: expert); lane q holds A[q/4][q%4], B[q%4][q/4] and D[q/4][2(q%4) .. +1].
// Each chain is one dependent MMA per four columns, so the kernel is bound by the MMA latency
// as long as its operands are already in shared memory: the block's x tile and router tile of
// each kRc-column chunk arrive by two 1-D TMA bulk copies, NB chunks ahead, each stage
// completing on its own mbarrier.  A second warp issues the copies and refills a stage once
// the chain warp has released it, so the chain warp's instruction stream holds nothing but
// the waits, the operand loads and the MMAs.  The padded rows make a lane's 8-byte reads
// conflict-free (lanes 0-15 and 16-31 each cover the 32 banks once).  In the last, partial
// chunk the columns past the last multiple of four are added with scalar FMAs, in order.
template <int NB>
__global__ void __launch_bounds__(64) k_router_dmma(const double *x64b, const double *w64b,
                                                    int tokens, int experts, int cols,
                                                    float *logits, GateOut go, int32_t *status) {
    grid_dep_wait();  // programmatic dependent launch: the kernel ahead has completed
    grid_dep_trigger();
    extern __shared__ __align__(16) double rs[];
    uint64_t *full = reinterpret_cast<uint64_t *>(rs + NB * kRstage);
    uint64_t *empty = full + NB;  // the chain warp has read the stage
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int eblk = (experts + 7) / 8;
    const int blk = blockIdx.x;
    if (blk >= eblk * ((tokens + 7) / 8)) return;
    const int tb = blk / eblk, eb = blk % eblk;
    const int nch = router_chunks(cols);
    constexpr uint32_t kTile = 8 * kRrow * 8;  // bytes of one operand's tile
    const double *xsrc = x64b + size_t(tb) * nch * 8 * kRrow;
    const double *wsrc = w64b + size_t(eb) * nch * 8 * kRrow;
    // x rows of the block's real tokens only (a prefix of the tile; the rows past them feed
    // only outputs that are not stored).
    const uint32_t xbytes = uint32_t(min(8, tokens - tb * 8)) * kRrow * 8;
    if (threadIdx.x == 0) {
        for (int s = 0; s < NB; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], 1);
        }
        tc::mbar_fence_init();
    }
    __syncthreads();
    volatile int never = 0;
    if (warp == 1) {
        // Copy warp (one lane): stage ch once the chain warp has read chunk ch - NB from it.
        if (lane == 0) {
            int ch = 0;
            for (; ch < nch; ++ch) {
                if (ch >= NB && !tc::mbar_wait(&empty[ch % NB], uint32_t(ch / NB - 1) & 1u, &never)) break;
                double *dst = rs + (ch % NB) * kRstage;
                uint64_t *bar = &full[ch % NB];
                tc::mbar_arrive_expect_tx(bar, xbytes + kTile);
                tc::bulk_g2s(dst, xsrc + size_t(ch) * 8 * kRrow, xbytes, bar);
                tc::bulk_g2s(dst + 8 * kRrow, wsrc + size_t(ch) * 8 * kRrow, kTile, bar);
            }
            // Every copy this CTA issued lands before it can exit.
            for (int c = ch > NB ? ch - NB : 0; c < ch; ++c)
                tc::mbar_wait(&full[c % NB], uint32_t(c / NB) & 1u, &never);
        }
        return;
    }
    // Chain warp: nothing but the waits, the operand loads and the MMAs.
    const int r = lane >> 2, kq = lane & 3;
    double d0 = -0.0, d1 = -0.0;  // Iterator::sum over f64 starts from -0.0 (bf16.rs:500)
    int ch = 0;
    for (; ch < nch; ++ch) {
        if (!tc::mbar_wait(&full[ch % NB], uint32_t(ch / NB) & 1u, &never)) break;
        const double *b = rs + (ch % NB) * kRstage;
        const int kc = min(kRc, cols - ch * kRc);
        if (kc == kRc) {
            // Shared-space loads (ld.shared; generic loads of the stage measured a long
            // scoreboard stall per step), kept after the stage's wait by being volatile.
            const uint32_t xa = tc::smem_u32(b + r * kRrow + kq), wa = tc::smem_u32(b + (8 + r) * kRrow + kq);
            double a[kRc / 4], w[kRc / 4];
#pragma unroll
            for (int i = 0; i < kRc / 4; ++i) {
                a[i] = lds_f64(xa + 32u * i);
                w[i] = lds_f64(wa + 32u * i);
            }
#pragma unroll
            for (int i = 0; i < kRc / 4; ++i) dmma_8x8x4(d0, d1, a[i], w[i]);
        } else {
            const int k4 = kc & ~3;
            for (int k = 0; k < k4; k += 4)
                dmma_8x8x4(d0, d1, b[r * kRrow + k + kq], b[(8 + r) * kRrow + k + kq]);
            for (int k = k4; k < kc; ++k) {  // lane: token r, experts 2kq, 2kq + 1
                const double xv = b[r * kRrow + k];
                d0 = fma(b[(8 + 2 * kq) * kRrow + k], xv, d0);
                d1 = fma(b[(9 + 2 * kq) * kRrow + k], xv, d1);
            }
        }
        // Every lane's reads of the stage have been consumed by issued MMAs.
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&empty[ch % NB]);
    }
    if (ch < nch) {
        // A stage never completed: report and leave without writing logits (the copy warp
        // lets the copies still in flight land).
        if (lane == 0 && status) atomicCAS(status, 0, int32_t(URB_ERR_TIMEOUT));
        return;
    }
    const int t = tb * 8 + r, e0 = eb * 8 + 2 * kq;
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

// One warp per token (route_noaux_token).
template <bool PRE>
__global__ void k_route_noaux(RouteNoauxArgs ra) {
    grid_dep_wait();  // programmatic dependent launch: the kernel ahead has completed
    grid_dep_trigger();
    extern __shared__ __align__(16) uint8_t smem[];
    const int warp = threadIdx.x >> 5;
    const int t = blockIdx.x * (blockDim.x >> 5) + warp;
    if (t >= ra.tokens) return;
    route_noaux_token<PRE>(ra, t, smem + size_t(warp) * ra.warp_bytes);
}

// route_softmax_top_k (src/models/qwen3_8/moe.rs:108-158).  One warp per token.
__global__ void k_route_softmax(const float *logits, int tokens, int E, int top_k,
                                ExpfTable tab, int32_t *out_e, float *out_w, int32_t *status,
                                int bf16_weights) {
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
        float w = __fdiv_rn(p[oe[r]], selected);
        if (bf16_weights) w = num_round_bf16(w);
        if (!isfinite(w)) set_status(status, URB_ERR_NONFINITE);
        out_w[size_t(t) * top_k + r] = w;
    }
}

// BF16 linear of the Qwen3.6 router and shared-expert gate (qwen3_8/math.rs:10-26 over
// dot_bf16_fp32_avx2_fma, src/model/bf16.rs:591-613).  Per output: eight FMA lanes from +0.0,
// column c in lane c % 8 over the largest multiple of eight columns; the lanes summed in order
// from -0.0; the remaining columns added as separately rounded products; the sum rounded to
// BF16.  One thread per (row, 4 tokens) keeps all 32 chains in registers; row `rows` is the
// gate row.  VEC: 16-byte weight and activation loads (cols % 8 == 0, aligned bases).
template <bool VEC>
__global__ void __launch_bounds__(128) k_router_bf16_lanes(const uint16_t *w, int rows,
                                                           const uint16_t *gate_row,
                                                           const float *x, int tokens, int cols,
                                                           float *logits, float *gate_logit,
                                                           int32_t *status) {
    constexpr int TT = 4;
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows + (gate_row ? 1 : 0)) return;
    const int t0 = blockIdx.y * TT;
    const uint16_t *wr = r < rows ? w + size_t(r) * cols : gate_row;
    const float *xr[TT];
#pragma unroll
    for (int i = 0; i < TT; ++i) xr[i] = x + size_t(min(t0 + i, tokens - 1)) * cols;
    const int complete = cols / 8 * 8;
    float acc[TT][8];
#pragma unroll
    for (int i = 0; i < TT; ++i)
#pragma unroll
        for (int l = 0; l < 8; ++l) acc[i][l] = 0.0f;
    for (int c = 0; c < complete; c += 8) {
        float wv[8];
        if (VEC) {
            const uint4 q = *reinterpret_cast<const uint4 *>(wr + c);
            const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                wv[2 * j] = __uint_as_float(qw[j] << 16);
                wv[2 * j + 1] = __uint_as_float(qw[j] & 0xffff0000u);
            }
        } else {
#pragma unroll
            for (int l = 0; l < 8; ++l) wv[l] = __uint_as_float(uint32_t(wr[c + l]) << 16);
        }
#pragma unroll
        for (int i = 0; i < TT; ++i) {
            float xv[8];
            if (VEC) {
                const float4 a = *reinterpret_cast<const float4 *>(xr[i] + c);
                const float4 b = *reinterpret_cast<const float4 *>(xr[i] + c + 4);
                xv[0] = a.x; xv[1] = a.y; xv[2] = a.z; xv[3] = a.w;
                xv[4] = b.x; xv[5] = b.y; xv[6] = b.z; xv[7] = b.w;
            } else {
#pragma unroll
                for (int l = 0; l < 8; ++l) xv[l] = xr[i][c + l];
            }
#pragma unroll
            for (int l = 0; l < 8; ++l) acc[i][l] = fmaf(wv[l], xv[l], acc[i][l]);
        }
    }
#pragma unroll
    for (int i = 0; i < TT; ++i) {
        if (t0 + i >= tokens) break;
        float s = -0.0f;
#pragma unroll
        for (int l = 0; l < 8; ++l) s = __fadd_rn(s, acc[i][l]);
        for (int c = complete; c < cols; ++c)
            s = __fadd_rn(s, __fmul_rn(__uint_as_float(uint32_t(wr[c]) << 16), xr[i][c]));
        s = num_round_bf16(s);
        if (!isfinite(s)) set_status(status, URB_ERR_NONFINITE);
        if (r < rows)
            logits[size_t(t0 + i) * rows + r] = s;
        else
            gate_logit[t0 + i] = s;
    }
}

}  // namespace

namespace {

ExpfTable table_of(const Ctx *ctx) { return ExpfTable{ctx->expf_keys, ctx->expf_vals, ctx->expf_index}; }

}  // namespace

int widen_router_f64(const Mat *router, double *dst, cudaStream_t st) {
    const int rows = int(router->rows), cols = int(router->cols);
    if (router->format == URB_FMT_BF16)
        k_to_f64_blocked<true><<<1024, 256, 0, st>>>(router->raw_values, rows, cols, dst);
    else if (router->format == URB_FMT_F32)
        k_to_f64_blocked<false><<<1024, 256, 0, st>>>(router->raw_values, rows, cols, dst);
    else
        return URB_ERR_UNSUPPORTED;
    return cudaGetLastError() == cudaSuccess ? URB_OK : URB_ERR_CUDA;
}

int launch_router_logits_f64(const double *w64b, int experts, const float *d_x, int tokens,
                             int cols, double *x64b, float *d_logits, cudaStream_t st,
                             const RouterGates *rg) {
    if (tokens <= 0) return URB_OK;
    GateOut go{};
    if (rg) go = GateOut{rg->bias, rg->gate, rg->sel, rg->status, table_of(rg->ctx)};
    auto widen = k_to_f64_blocked<false>;
    URB_LAUNCH_DEP(widen, 592, 256, 0, st, d_x, tokens, cols, x64b);
    // Stages in flight: 3 when the blocks fill the SMs several times over (four CTAs of 51 KB
    // per SM), 8 for the few blocks of a decode step (one CTA of 135 KB per SM).
    const int blocks = ((tokens + 7) / 8) * ((experts + 7) / 8);
    const bool deep = blocks <= 256;
    auto k = deep ? k_router_dmma<8> : k_router_dmma<kRnb>;
    const int smem = router_smem(deep ? 8 : kRnb);
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return URB_ERR_CUDA;
    URB_LAUNCH_DEP(k, blocks, 64, smem, st, x64b, w64b, tokens, experts, cols, d_logits, go,
                   rg ? rg->status : nullptr);
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
    const RouteNoauxArgs ra = route_noaux_args(ctx, d_logits, d_bias, tokens, experts, g, d_expert, d_weight,
                                               d_score, d_status, pre);
    URB_LAUNCH_DEP(k, (tokens + warps - 1) / warps, warps * 32, smem, st, ra);
    URB_CUDA(ctx, cudaGetLastError());
    return URB_OK;
}

namespace {

ExpfTable log1p_table_of(const Ctx *ctx) {
    return ExpfTable{ctx->log1pf_keys, ctx->log1pf_vals, ctx->log1pf_index};
}

// softplus of deepseek_v4/math.rs:604-610 with libm expf / log1pf, then the square root.
__device__ __forceinline__ float sqrt_softplus(float v, const ExpfTable &ex, const ExpfTable &lp) {
    const float sp = v > 0.0f ? __fadd_rn(v, log1pf_libm(expf_libm(-v, ex), lp))
                              : log1pf_libm(expf_libm(v, ex), lp);
    return __fsqrt_rn(sp);
}

// route_sqrt_softplus (deepseek_v4/math.rs:451-516), one warp per token: score = sqrt(
// softplus(logit)), selection = score + bias; top_k by selection desc with the lower id winning
// ties (total order), or the token's hash experts as given; the denominator sums the chosen
// scores in order (f32); weight = score / denominator * scale.  Shared memory per warp:
// score[E], sel[E] floats and a taken flag per expert.
__global__ void k_route_sqrt_softplus(const float *logits, const float *bias,
                                      const int32_t *hash, int tokens, int E, int top_k,
                                      float scaling, ExpfTable ex, ExpfTable lp, int32_t *out_e,
                                      float *out_w, float *out_s, int32_t *status,
                                      int warp_bytes) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * (blockDim.x >> 5) + warp;
    if (t >= tokens) return;
    float *score = reinterpret_cast<float *>(smem + size_t(warp) * warp_bytes);
    float *sel = score + E;
    uint8_t *taken = reinterpret_cast<uint8_t *>(sel + E);
    const float *lg = logits + size_t(t) * E;
    bool bad = false;
    for (int i = lane; i < E; i += 32) {
        const float l = lg[i], b = bias ? bias[i] : 0.0f;
        bad |= !isfinite(l) || !isfinite(b);
        const float sc = sqrt_softplus(l, ex, lp);
        score[i] = sc;
        sel[i] = bias ? __fadd_rn(sc, b) : sc;
        taken[i] = 0;
    }
    int32_t *oe = out_e + size_t(t) * top_k;
    float *ow = out_w + size_t(t) * top_k;
    auto reject = [&](int code) {
        if (lane == 0) set_status(status, code);
        for (int r = lane; r < top_k; r += 32) {
            oe[r] = r;
            ow[r] = 0.0f;
            if (out_s) out_s[size_t(t) * top_k + r] = 0.0f;
        }
    };
    if (__any_sync(0xffffffffu, bad)) { reject(URB_ERR_NONFINITE); return; }
    if (hash) {
        bool oob = false;
        for (int r = lane; r < top_k; r += 32) {
            const int32_t e = hash[size_t(t) * top_k + r];
            oob |= e < 0 || e >= E;
        }
        if (__any_sync(0xffffffffu, oob)) { reject(URB_ERR_SHAPE); return; }
    }
    __syncwarp();
    float den = -0.0f;  // Iterator::sum over f32
    for (int r = 0; r < top_k; ++r) {
        int id;
        if (hash) {
            id = hash[size_t(t) * top_k + r];
        } else {
            int32_t key = INT32_MIN;
            id = INT32_MAX;
            for (int i = lane; i < E; i += 32)
                if (!taken[i]) {
                    const int32_t k = total_key(sel[i]);
                    if (better(k, i, key, id)) { key = k; id = i; }
                }
            warp_best(key, id);
            if (lane == (id & 31)) taken[id] = 1;
        }
        if (lane == 0) {
            oe[r] = id;
            den = __fadd_rn(den, score[id]);
        }
        __syncwarp();
    }
    den = __shfl_sync(0xffffffffu, den, 0);
    if (!isfinite(den) || den <= 0.0f) { reject(URB_ERR_NONFINITE); return; }
    for (int r = lane; r < top_k; r += 32) {
        const int id = oe[r];
        ow[r] = __fmul_rn(__fdiv_rn(score[id], den), scaling);
        if (out_s) out_s[size_t(t) * top_k + r] = sel[id];
    }
}

}  // namespace

int launch_route_sqrt_softplus(Ctx *ctx, const float *d_logits, const float *d_bias,
                               const int32_t *d_hash, int tokens, int experts, int top_k,
                               float scaling, int32_t *d_expert, float *d_weight, float *d_score,
                               int32_t *d_status, cudaStream_t st) {
    if (tokens <= 0) return URB_OK;
    const int warps = 4;
    const int warp_bytes = (experts * 9 + 15) & ~15;
    k_route_sqrt_softplus<<<(tokens + warps - 1) / warps, warps * 32, size_t(warps) * warp_bytes, st>>>(
        d_logits, d_bias, d_hash, tokens, experts, top_k, scaling, table_of(ctx),
        log1p_table_of(ctx), d_expert, d_weight, d_score, d_status, warp_bytes);
    URB_CUDA(ctx, cudaGetLastError());
    return URB_OK;
}

int launch_route_softmax(Ctx *ctx, const float *d_logits, int tokens, int experts, int top_k,
                         int32_t *d_expert, float *d_weight, int32_t *d_status,
                         cudaStream_t st, int bf16_weights) {
    if (tokens <= 0) return URB_OK;
    int warps = 4;
    size_t smem = size_t(warps) * experts * 5;
    k_route_softmax<<<(tokens + warps - 1) / warps, warps * 32, smem, st>>>(
        d_logits, tokens, experts, top_k, table_of(ctx), d_expert, d_weight, d_status,
        bf16_weights);
    URB_CUDA(ctx, cudaGetLastError());
    return URB_OK;
}

int launch_router_bf16_lanes(const uint16_t *w, int rows, const uint16_t *gate_row,
                             const float *d_x, int tokens, int cols, float *d_logits,
                             float *d_gate_logit, int32_t *d_status, cudaStream_t st) {
    if (tokens <= 0) return URB_OK;
    const int nrows = rows + (gate_row ? 1 : 0);
    if (nrows == 0) return URB_OK;
    const dim3 grid(unsigned((nrows + 127) / 128), unsigned((tokens + 3) / 4));
    const bool vec = cols % 8 == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(gate_row) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(d_x) & 15) == 0;
    if (vec)
        k_router_bf16_lanes<true><<<grid, 128, 0, st>>>(w, rows, gate_row, d_x, tokens, cols,
                                                        d_logits, d_gate_logit, d_status);
    else
        k_router_bf16_lanes<false><<<grid, 128, 0, st>>>(w, rows, gate_row, d_x, tokens, cols,
                                                         d_logits, d_gate_logit, d_status);
    return cudaGetLastError() == cudaSuccess ? URB_OK : URB_ERR_CUDA;
}

}  // namespace urb
