// moe.cu — the MoE layer on one GPU: grouping (permutation/histogram), the two grouped expert
// passes, and the weighted combine.
//
// Reference composition (src/models/glm/runtime/moe.rs:138-176): router logits -> route_noaux_tc
// -> shared GatedMlp -> every routed GatedMlp in selection order -> f64 combine.  Here the
// routed experts run grouped: routes are sorted experts-ascending / tokens-ascending
// (src/models/qwen3_6/runtime.rs:1123-1132), each expert's token run is one or more segments of
// a grouped pass, and the combine adds the route-weighted expert outputs per token in the
// reference's selection order with f64 accumulation.
#include <algorithm>

#include "numerics.cuh"
#include "route_noaux.cuh"
#include "urb_internal.cuh"
#include "urb_moe_internal.cuh"

namespace urb {
namespace {

constexpr int kPermThreads = 1024;

// Grouping on one CTA of kPermThreads threads (smem: permute_smem bytes).  See
// urb_moe_internal.cuh for the outputs.
__device__ void permute_block(const PermArgs &p, uint8_t *smem) {
    const int E = p.experts, TK = p.tokens * p.top_k;
    int *cnt = reinterpret_cast<int *>(smem);                 // [E]
    int *off = cnt + E;                                        // [E+1]
    int *running = off + E + 1;                                // [E]
    uint16_t *wcnt = reinterpret_cast<uint16_t *>(running + E);  // [32][E]
    __shared__ int warp_sums[32];
    __shared__ int bad;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) bad = (p.status && *p.status) ? 1 : 0;  // an earlier stage failed
    for (int e = tid; e < E; e += kPermThreads) { cnt[e] = 0; running[e] = 0; }
    for (int i = tid; i < 32 * E; i += kPermThreads) wcnt[i] = 0;
    __syncthreads();
    for (int i = tid; i < TK; i += kPermThreads) {
        int e = p.ids[i];
        if (e == -1 && p.allow_foreign) continue;  // a route held by another rank
        if (e < 0 || e >= E) bad = 1; else atomicAdd(&cnt[e], 1);
    }
    __syncthreads();
    if (bad) {
        // Empty grouping: every later stage sees zero work.
        if (tid == 0 && p.status) atomicCAS(p.status, 0, int32_t(URB_ERR_SHAPE));
        if (tid == 0 && p.nsegs_gu) { *p.nsegs_gu = 0; *p.total_rows_gu = 0; *p.nsegs_dn = 0; *p.total_rows_dn = 0; }
        for (int e = tid; e < E; e += kPermThreads) {
            if (p.counts) p.counts[e] = 0;
            if (p.offsets) p.offsets[e] = 0;
        }
        if (tid == 0 && p.offsets) p.offsets[E] = 0;
        for (int i = tid; i < TK; i += kPermThreads) p.inv[i] = 0;
        return;
    }
    // Exclusive scan of counts (E <= 32 * 1024).
    {
        int per = (E + kPermThreads - 1) / kPermThreads;
        int b = tid * per, s = 0;
        for (int e = b; e < min(E, b + per); ++e) s += cnt[e];
        int incl = s;
        for (int o = 1; o < 32; o <<= 1) {
            int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        if (lane == 31) warp_sums[warp] = incl;
        __syncthreads();
        if (warp == 0) {
            int v = warp_sums[lane];
            for (int o = 1; o < 32; o <<= 1) {
                int u = __shfl_up_sync(0xffffffffu, v, o);
                if (lane >= o) v += u;
            }
            warp_sums[lane] = v;
        }
        __syncthreads();
        int base = incl - s + (warp ? warp_sums[warp - 1] : 0);
        for (int e = b; e < min(E, b + per); ++e) { off[e] = base; base += cnt[e]; }
        if (tid == 0) off[E] = warp_sums[31];  // routes held here (TK unless some are foreign)
        __syncthreads();
    }
    // Stable placement, token-major route order -> (expert asc, token asc).
    for (int base = 0; base < TK; base += kPermThreads) {
        const int i = base + tid;
        const int e = i < TK ? p.ids[i] : -1;
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        const int rank_w = __popc(peers & ((1u << lane) - 1));
        if (e >= 0 && rank_w == 0) wcnt[warp * E + e] = uint16_t(__popc(peers));
        __syncthreads();
        if (e >= 0) {
            int before = 0;
            for (int w = 0; w < warp; ++w) before += wcnt[w * E + e];
            const int pos = off[e] + running[e] + before + rank_w;
            p.perm_token[pos] = i / p.top_k;
            p.perm_slot[pos] = i % p.top_k;
            p.inv[i] = pos;
            if (p.route_of) p.route_of[pos] = i;
            if (p.col_w) p.col_w[pos] = p.route_w[i];
        } else if (i < TK) {
            p.inv[i] = -1;  // foreign route
        }
        __syncthreads();
        for (int x = tid; x < E; x += kPermThreads) {
            int s = 0;
            for (int w = 0; w < 32; ++w) { s += wcnt[w * E + x]; wcnt[w * E + x] = 0; }
            running[x] += s;
        }
        __syncthreads();
    }
    // Segments: routed experts ascending, each cut into chunks of `cap` tokens, then the
    // shared expert's chunks.  (Skipped when only the grouping itself is requested.)
    const int cap = (p.lofree && *p.lofree) ? 2 * p.cap : p.cap;
    if (p.segs_gu) {
        int per = (E + kPermThreads - 1) / kPermThreads;
        int b = tid * per, s = 0;
        for (int e = b; e < min(E, b + per); ++e) s += (cnt[e] + cap - 1) / cap;
        int incl = s;
        for (int o = 1; o < 32; o <<= 1) {
            int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        __syncthreads();
        if (lane == 31) warp_sums[warp] = incl;
        __syncthreads();
        if (warp == 0) {
            int v = warp_sums[lane];
            for (int o = 1; o < 32; o <<= 1) {
                int u = __shfl_up_sync(0xffffffffu, v, o);
                if (lane >= o) v += u;
            }
            warp_sums[lane] = v;
        }
        __syncthreads();
        int sidx = incl - s + (warp ? warp_sums[warp - 1] : 0);
        for (int e = b; e < min(E, b + per); ++e) {
            for (int j = 0; j * cap < cnt[e]; ++j, ++sidx) {
                Seg gu, dn;
                gu.tiles_a = p.gate_tiles[e]; gu.rexp_a = p.gate_rexp[e];
                gu.tiles_b = p.up_tiles[e]; gu.rexp_b = p.up_rexp[e];
                gu.rbs = p.gu_rbs; gu.rows = p.inter; gu.kslices = p.gu_kslices; gu.cols = p.hidden;
                gu.col_begin = off[e] + j * cap; gu.ntok = min(cap, cnt[e] - j * cap);
                gu.row_begin = sidx * 16 * p.gu_rbs; gu.pad = e;
                dn.tiles_a = p.down_tiles[e]; dn.rexp_a = p.down_rexp[e];
                dn.tiles_b = nullptr; dn.rexp_b = nullptr;
                dn.rbs = p.dn_rbs; dn.rows = p.hidden; dn.kslices = p.dn_kslices; dn.cols = p.inter;
                dn.col_begin = gu.col_begin; dn.ntok = gu.ntok;
                dn.row_begin = sidx * 16 * p.dn_rbs; dn.pad = e;
                p.segs_gu[sidx] = gu;
                p.segs_dn[sidx] = dn;
            }
        }
        __syncthreads();
        if (tid == kPermThreads - 1) {
            int routed = sidx;  // thread owning the last experts ends at the total
            int nseg = routed;
            if (p.shared_in_pass) {
                for (int j = 0; j * cap < p.tokens; ++j, ++nseg) {
                    Seg gu, dn;
                    gu.tiles_a = p.sh_gate_tiles; gu.rexp_a = p.sh_gate_rexp;
                    gu.tiles_b = p.sh_up_tiles; gu.rexp_b = p.sh_up_rexp;
                    gu.rbs = p.gu_rbs; gu.rows = p.inter; gu.kslices = p.gu_kslices; gu.cols = p.hidden;
                    gu.col_begin = TK + j * cap; gu.ntok = min(cap, p.tokens - j * cap);
                    gu.row_begin = nseg * 16 * p.gu_rbs; gu.pad = -1;
                    dn.tiles_a = p.sh_down_tiles; dn.rexp_a = p.sh_down_rexp;
                    dn.tiles_b = nullptr; dn.rexp_b = nullptr;
                    dn.rbs = p.dn_rbs; dn.rows = p.hidden; dn.kslices = p.dn_kslices; dn.cols = p.inter;
                    dn.col_begin = gu.col_begin; dn.ntok = gu.ntok;
                    dn.row_begin = nseg * 16 * p.dn_rbs; dn.pad = -1;
                    p.segs_gu[nseg] = gu;
                    p.segs_dn[nseg] = dn;
                }
            }
            *p.nsegs_gu = nseg;
            *p.nsegs_dn = nseg;
            *p.total_rows_gu = nseg * 16 * p.gu_rbs;
            *p.total_rows_dn = nseg * 16 * p.dn_rbs;
        }
    }
    // Activation-column sources of the gate/up pass and SwiGLU max-exponent reset.
    if (p.col_src)
        for (int c = tid; c < TK + p.tokens; c += kPermThreads) {
            p.col_src[c] = c < TK ? p.perm_token[c] : c - TK;
            p.maxexp[c] = -1000;
        }
    if (p.col_w)
        for (int t = tid; t < p.tokens; t += kPermThreads) p.col_w[TK + t] = 1.0f;  // shared
    for (int e = tid; e < E; e += kPermThreads) {
        if (p.counts) p.counts[e] = cnt[e];
        if (p.offsets) p.offsets[e] = off[e];
    }
    if (tid == 0 && p.offsets) p.offsets[E] = off[E];
}

__global__ void __launch_bounds__(kPermThreads) k_permute(PermArgs p) {
    grid_dep_wait();  // programmatic dependent launch: the kernel ahead has completed
    grid_dep_trigger();
    extern __shared__ __align__(16) uint8_t smem[];
    permute_block(p, smem);
}

// out[t][h] = f32( f64(shared) + sum_k f64(w[t][k]) * f64(y[inv[t,k]][h]) ), k in selection
// order (glm/runtime/moe.rs:165-175).  inv == nullptr: y is already in route order t * top_k + k.
__global__ void k_combine(const float *y, const float *shared_y, const float *w,
                          const int32_t *inv, int tokens, int top_k, int hidden, float *out,
                          const int32_t *status) {
    grid_dep_wait();  // programmatic dependent launch: the kernel ahead has completed
    grid_dep_trigger();
    if (status && *status) return;
    const int t = blockIdx.y;
    const int h = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= tokens || h >= hidden) return;
    double acc = shared_y ? double(shared_y[size_t(t) * hidden + h]) : 0.0;
    for (int k = 0; k < top_k; ++k) {
        const int pos = inv ? inv[t * top_k + k] : t * top_k + k;
        acc += double(w[t * top_k + k]) * double(y[size_t(pos) * hidden + h]);
    }
    out[size_t(t) * hidden + h] = float(acc);
}

// The same for hidden % 4 == 0, four columns per thread: the routes' row indices and weights
// are loaded first, then every route's 16-byte slice, so all of a thread's loads are in flight
// together (the combine is bound by their latency otherwise).
__global__ void k_combine4(const float *y, const float *shared_y, const float *w,
                           const int32_t *inv, int tokens, int top_k, int hidden, float *out,
                           const int32_t *status) {
    grid_dep_wait();  // programmatic dependent launch: the kernel ahead has completed
    grid_dep_trigger();
    if (status && *status) return;
    const int t = blockIdx.y;
    const int h = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (t >= tokens || h >= hidden) return;
    double a0 = 0.0, a1 = 0.0, a2 = 0.0, a3 = 0.0;
    if (shared_y) {
        const float4 s = *reinterpret_cast<const float4 *>(shared_y + size_t(t) * hidden + h);
        a0 = s.x; a1 = s.y; a2 = s.z; a3 = s.w;
    }
    constexpr int kB = 8;
    for (int k0 = 0; k0 < top_k; k0 += kB) {
        int pos[kB];
        float wk[kB];
        float4 v[kB];
#pragma unroll
        for (int j = 0; j < kB; ++j) {
            const int k = k0 + j;
            pos[j] = k < top_k ? (inv ? inv[t * top_k + k] : t * top_k + k) : 0;
            wk[j] = k < top_k ? w[t * top_k + k] : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < kB; ++j)
            if (k0 + j < top_k) v[j] = *reinterpret_cast<const float4 *>(y + size_t(pos[j]) * hidden + h);
#pragma unroll
        for (int j = 0; j < kB; ++j) {
            if (k0 + j >= top_k) break;
            const double wd = wk[j];
            a0 += wd * double(v[j].x);
            a1 += wd * double(v[j].y);
            a2 += wd * double(v[j].z);
            a3 += wd * double(v[j].w);
        }
    }
    *reinterpret_cast<float4 *>(out + size_t(t) * hidden + h) = make_float4(float(a0), float(a1), float(a2), float(a3));
}

// DeepSeek-V4 combine: f32 sum of a token's routed rows in ascending expert id (ties keep the
// route order), the shared row added last, then round to BF16 (deepseek_v4/runtime.rs:2639-2647;
// the route weights were applied before the down projection).
__global__ void k_combine_deepseek(const float *y, const float *shared_y, const int32_t *ids,
                                   const int32_t *inv, int tokens, int top_k, int hidden,
                                   float *out, int32_t *status) {
    grid_dep_wait();  // programmatic dependent launch: the kernel ahead has completed
    grid_dep_trigger();
    if (*status) return;
    const int t = blockIdx.y;
    const int h = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= tokens || h >= hidden) return;
    int order[16];
    for (int k = 0; k < top_k; ++k) {  // stable insertion by expert id
        const int id = ids[t * top_k + k];
        int j = k;
        while (j > 0 && ids[t * top_k + order[j - 1]] > id) { order[j] = order[j - 1]; --j; }
        order[j] = k;
    }
    float acc = 0.0f;
    for (int j = 0; j < top_k; ++j) {
        const int pos = inv[t * top_k + order[j]];
        acc = __fadd_rn(acc, y[size_t(pos) * hidden + h]);
    }
    if (shared_y) acc = __fadd_rn(acc, shared_y[size_t(t) * hidden + h]);
    const uint32_t b = __float_as_uint(acc);
    const float r = __uint_as_float((b + 0x7fffu + ((b >> 16) & 1u)) & 0xffff0000u);
    if (!isfinite(r)) atomicCAS(status, 0, int32_t(URB_ERR_NONFINITE));
    out[size_t(t) * hidden + h] = r;
}

// MoE output of the Qwen3.6 numerics (execute_batched_moe, qwen3_6/runtime.rs:1123-1213):
// routed contributions BF16(BF16(w) * y) accumulated from +0.0 in ascending expert id (stable
// for repeated ids), each sum rounded to BF16; then the shared expert's BF16(s * y_shared)
// with s = BF16(sigmoid(gate logit)) evaluated as 1 / (1 + exp(-g)) for g >= 0 and
// exp(g) / (1 + exp(g)) otherwise (libm expf); the final sum rounded to BF16.
__global__ void k_combine_qwen(const float *y, const float *shared_y, const int32_t *ids,
                               const float *w, const int32_t *inv, const float *gate_logit,
                               ExpfTable tab, int tokens, int top_k, int hidden, float *out,
                               int32_t *status) {
    grid_dep_wait();  // programmatic dependent launch: the kernel ahead has completed
    grid_dep_trigger();
    if (*status) return;
    const int t = blockIdx.y;
    const int h = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= tokens || h >= hidden) return;
    int order[16];
    for (int k = 0; k < top_k; ++k) {  // stable insertion by expert id
        const int id = ids[t * top_k + k];
        int j = k;
        while (j > 0 && ids[t * top_k + order[j - 1]] > id) { order[j] = order[j - 1]; --j; }
        order[j] = k;
    }
    float acc = 0.0f;
    for (int j = 0; j < top_k; ++j) {
        const int r = t * top_k + order[j];
        const float c = num_round_bf16(__fmul_rn(num_round_bf16(w[r]), y[size_t(inv[r]) * hidden + h]));
        acc = num_round_bf16(__fadd_rn(acc, c));
    }
    if (shared_y) {
        const float g = gate_logit[t];
        float s;
        if (g >= 0.0f) {
            s = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf_libm(-g, tab)));
        } else {
            const float e = expf_libm(g, tab);
            s = __fdiv_rn(e, __fadd_rn(1.0f, e));
        }
        s = num_round_bf16(s);
        const float c = num_round_bf16(__fmul_rn(s, shared_y[size_t(t) * hidden + h]));
        acc = num_round_bf16(__fadd_rn(acc, c));
    }
    if (!isfinite(acc)) atomicCAS(status, 0, int32_t(URB_ERR_NONFINITE));
    out[size_t(t) * hidden + h] = acc;
}

// Groups of the tensor-core passes (single CTA).  Gate/up pass: per routed expert with tokens
// one paired group (gate and up tiles against the same activation stages), then the shared
// expert's; down pass: one group per routed expert, then the shared expert.  A group of c tokens has ceil(c / bs_cap) sub-segments; its units are mts * nsub.
// Activation-stage offsets are a prefix over owning groups of the bytes their stages take.
__device__ __forceinline__ int round16(int x) { return (x + 15) & ~15; }

// Bytes of the activation stages of a group of c tokens and ks stages.
__device__ __forceinline__ long long bs_group_bytes(int fmt, int c, int ks) {
    const int cap = bs_cap(fmt);
    const int nsub = (c + cap - 1) / cap;
    const int n_last = round16(bs_rows_per_tok(fmt) * (c - (nsub - 1) * cap));
    return (long long)ks * ((long long)(nsub - 1) * bs_bstage_bytes(fmt, kBsNmax) + bs_bstage_bytes(fmt, n_last));
}

// Activation slot of token j of a group whose stages start at boff.
__device__ __forceinline__ BsSlot slot_of(int fmt, long long boff, int ks, int c, int j) {
    const int cap = bs_cap(fmt);
    const int nsub = (c + cap - 1) / cap, sub = j / cap;
    BsSlot z;
    z.base = boff + sub * (long long)ks * bs_bstage_bytes(fmt, kBsNmax);
    z.slot = j - sub * cap;
    z.n = sub < nsub - 1 ? kBsNmax : round16(bs_rows_per_tok(fmt) * (c - (nsub - 1) * cap));
    return z;
}

// Dynamic shared memory: each routed expert's activation-stage base (s_boff [E + 1]), the
// unit_begin of every group of the pass (s_ub [2E + 4], binary-searched by the cooperative
// unit-map fill) and the experts' first columns (s_off [E + 1], binary-searched by the
// cooperative slot fill, so a large group's slots are not written by one thread).
__device__ void build_tc_block(const TcBuildArgs &b, long long *s_dyn) {
    long long *s_boff = s_dyn;
    int *s_ub = reinterpret_cast<int *>(s_boff + b.experts + 1);
    int *s_off = s_ub + 2 * b.experts + 4;
    __shared__ long long wsum[32], sh_boff;
    __shared__ int wcnt[32], wunits[32], s_groups, s_units;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (b.status && *b.status) {  // an earlier stage failed: no work for the passes
        if (tid < 4) b.scalars[tid] = 0;
        return;
    }
    const int E = b.experts, TK = b.tokens * b.top_k;
    const int sc = bs_stage_cols(b.fmt);
    for (int e = tid; e <= E; e += 1024) s_off[e] = b.offsets[e];
    for (int pass = 0; pass < 2; ++pass) {
        const int mats = 1;  // groups per expert (gate/up: one paired group)
        const int ks = pass == 0 ? (b.hidden + sc - 1) / sc : (b.inter + sc - 1) / sc;
        const int mts = pass == 0 ? (b.inter + 127) / 128 : (b.hidden + 127) / 128;
        const int mtu = pass == 1 && b.pair_down ? (mts + 1) / 2 : mts;  // tile units per group
        // Per thread: experts [e0, e1); groups, units and activation bytes.
        const int per_thr = (E + 1023) / 1024;
        const int e0 = min(E, tid * per_thr), e1 = min(E, e0 + per_thr);
        int ng = 0, nu = 0;
        long long nb = 0;
        for (int e = e0; e < e1; ++e) {
            const int c = b.counts[e];
            if (c <= 0) continue;
            ng += mats;
            nu += mats * mtu * ((c + bs_cap(b.fmt) - 1) / bs_cap(b.fmt));
            nb += bs_group_bytes(b.fmt, c, ks);
        }
        // Block-wide exclusive scans of (groups, units, bytes).
        int ig = ng, iu = nu;
        long long ib = nb;
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, ig, o);
            const int vu = __shfl_up_sync(0xffffffffu, iu, o);
            const long long w = __shfl_up_sync(0xffffffffu, ib, o);
            if (lane >= o) { ig += v; iu += vu; ib += w; }
        }
        __syncthreads();
        if (lane == 31) { wcnt[warp] = ig; wunits[warp] = iu; wsum[warp] = ib; }
        __syncthreads();
        if (warp == 0) {
            int v = wcnt[lane], vu = wunits[lane];
            long long w = wsum[lane];
            for (int o = 1; o < 32; o <<= 1) {
                const int v2 = __shfl_up_sync(0xffffffffu, v, o);
                const int vu2 = __shfl_up_sync(0xffffffffu, vu, o);
                const long long w2 = __shfl_up_sync(0xffffffffu, w, o);
                if (lane >= o) { v += v2; vu += vu2; w += w2; }
            }
            wcnt[lane] = v;
            wunits[lane] = vu;
            wsum[lane] = w;
        }
        __syncthreads();
        int gi = ig - ng + (warp ? wcnt[warp - 1] : 0);
        int ub = iu - nu + (warp ? wunits[warp - 1] : 0);
        long long boff = ib - nb + (warp ? wsum[warp - 1] : 0);
        TcSeg *out = pass == 0 ? b.gu : b.dn;
        BsSlot *sl = pass == 0 ? b.gu_slots : b.dn_slots;
        const bool shx = pass == 0 && b.shared_x;  // one token: every group reads stage set 0
        auto emit = [&](const uint8_t *wg, const uint8_t *wu, int m, int col0, int c) {
            TcSeg s;
            s.w = wg;
            s.w2 = wu;
            s.b_off = shx ? 0 : boff;
            s.mts = mts;
            s.ks = ks;
            s.rows = pass == 0 ? b.inter : b.hidden;
            s.cols = pass == 0 ? b.hidden : b.inter;
            s.col_begin = col0;
            s.ntok = c;
            s.nsub = (c + bs_cap(b.fmt) - 1) / bs_cap(b.fmt);
            s.unit_begin = ub;
            s.out_off = m * b.inter;  // gate | up halves of a gate/up output row
            s.pad = 0;
            s_ub[gi] = ub;
            out[gi++] = s;
            ub += mtu * s.nsub;
        };
        for (int e = e0; e < e1; ++e) {
            const int c = b.counts[e];
            if (c <= 0) continue;
            const int col0 = b.offsets[e];
            if (pass == 0) {
                emit(b.gate_tc[e], b.up_tc[e], 0, col0, c);
            } else {
                emit(b.down_tc[e], nullptr, 0, col0, c);
            }
            s_boff[e] = boff;  // the expert's activation slots are filled below, by all threads
            boff += bs_group_bytes(b.fmt, c, ks);
        }
        __syncthreads();
        // Activation slots of the routed columns: column col belongs to the expert e with
        // s_off[e] <= col < s_off[e + 1].
        for (int col = tid; col < s_off[E]; col += 1024) {
            int lo = 0, hi = E - 1;
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (s_off[mid] <= col) lo = mid; else hi = mid - 1;
            }
            sl[col] = shx ? slot_of(b.fmt, 0, ks, 1, 0)
                          : slot_of(b.fmt, s_boff[lo], ks, s_off[lo + 1] - s_off[lo], col - s_off[lo]);
        }
        if (tid == 1023) {
            // gi / ub / boff of the last thread are the routed totals; append the shared expert.
            sh_boff = boff;
            if (b.has_shared && b.shared_tokens > 0) {
                if (pass == 0) {
                    emit(b.sh_gate_tc, b.sh_up_tc, 0, TK, b.shared_tokens);
                } else {
                    emit(b.sh_down_tc, nullptr, 0, TK, b.shared_tokens);
                }
            }
            s_groups = gi;
            s_units = ub;
            b.scalars[2 * pass] = gi;
            b.scalars[2 * pass + 1] = ub;
        }
        __syncthreads();
        // Shared expert's activation slots and the unit -> group map, by all threads.
        if (b.has_shared)
            for (int j = tid; j < b.shared_tokens; j += 1024)
                sl[TK + j] = shx ? slot_of(b.fmt, 0, ks, 1, 0) : slot_of(b.fmt, sh_boff, ks, b.shared_tokens, j);
        int *um = pass == 0 ? b.gu_units : b.dn_units;
        const int G = s_groups, U = s_units;
        for (int u = tid; u < U; u += 1024) {
            int lo = 0, hi = G - 1;
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (s_ub[mid] <= u) lo = mid; else hi = mid - 1;
            }
            um[u] = lo;
        }
        __syncthreads();
    }
}

__global__ void __launch_bounds__(1024) k_build_tc_segs(TcBuildArgs b) {
    grid_dep_wait();  // programmatic dependent launch: the kernel ahead has completed
    grid_dep_trigger();
    extern __shared__ long long s_dyn[];
    build_tc_block(b, s_dyn);
}

// Decode (tokens <= 32): routing (warp t routes token t), grouping and the tensor-core pass
// tables in one CTA, each phase reading the previous one's outputs after a block barrier.
__global__ void __launch_bounds__(1024) k_decode_group(RouteNoauxArgs ra, PermArgs p, TcBuildArgs b) {
    grid_dep_wait();  // programmatic dependent launch: the kernel ahead has completed
    grid_dep_trigger();
    extern __shared__ __align__(16) uint8_t smem[];
    const int warp = threadIdx.x >> 5;
    if (warp < ra.tokens) route_noaux_token<true>(ra, warp, smem + size_t(warp) * ra.warp_bytes);
    __syncthreads();
    permute_block(p, smem);
    __syncthreads();
    build_tc_block(b, reinterpret_cast<long long *>(smem));
}

size_t permute_smem(int experts) {
    const size_t v = size_t(experts) * 4 * 3 + 4 + size_t(32) * experts * 2;
    return (v + 15) & ~size_t(15);
}
size_t build_smem(int experts) {
    return size_t(experts + 1) * sizeof(long long) + size_t(3 * experts + 5) * sizeof(int);
}

}  // namespace

int launch_decode_group(Ctx *ctx, const RouterGates &rg, int tokens, int experts, const urb_moe_geometry &g,
                        int32_t *d_expert, float *d_weight, float *d_score, const PermArgs &p,
                        const TcBuildArgs &b, cudaStream_t st) {
    if (tokens < 1 || tokens > 32) return URB_ERR_UNSUPPORTED;
    const RouteNoauxArgs ra = route_noaux_args(ctx, nullptr, nullptr, tokens, experts, g, d_expert, d_weight,
                                               d_score, rg.status, &rg);
    const size_t smem = std::max(std::max(size_t(tokens) * ra.warp_bytes, permute_smem(experts)), build_smem(experts));
    if (smem > 200 * 1024) return URB_ERR_UNSUPPORTED;
    URB_CUDA(ctx, cudaFuncSetAttribute(k_decode_group, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
    URB_LAUNCH_DEP(k_decode_group, 1, 1024, smem, st, ra, p, b);
    URB_CUDA(ctx, cudaGetLastError());
    return URB_OK;
}

int launch_build_tc_segs(Ctx *ctx, const TcBuildArgs &b, cudaStream_t st) {
    const size_t smem = build_smem(b.experts);
    if (smem > 200 * 1024) return set_error(ctx, URB_ERR_UNSUPPORTED, "too many experts for the group builder");
    URB_CUDA(ctx, cudaFuncSetAttribute(k_build_tc_segs, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
    URB_LAUNCH_DEP(k_build_tc_segs, 1, 1024, smem, st, b);
    URB_CUDA(ctx, cudaGetLastError());
    return URB_OK;
}

int launch_permute(Ctx *ctx, const PermArgs &p, cudaStream_t st) {
    const size_t smem = permute_smem(p.experts);
    if (smem > 200 * 1024) return set_error(ctx, URB_ERR_UNSUPPORTED, "too many experts for the grouping kernel");
    URB_CUDA(ctx, cudaFuncSetAttribute(k_permute, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
    URB_LAUNCH_DEP(k_permute, 1, kPermThreads, smem, st, p);
    URB_CUDA(ctx, cudaGetLastError());
    return URB_OK;
}

int launch_combine_deepseek(Ctx *ctx, const float *y, const float *shared_y, const int32_t *ids,
                            const int32_t *inv, int tokens, int top_k, int hidden, float *out,
                            cudaStream_t st, int32_t *status) {
    if (tokens <= 0) return URB_OK;
    if (top_k > 16) return set_error(ctx, URB_ERR_UNSUPPORTED, "DeepSeek combine: top_k > 16");
    dim3 grid(unsigned((hidden + 255) / 256), unsigned(tokens));
    URB_LAUNCH_DEP(k_combine_deepseek, grid, 256, 0, st, y, shared_y, ids, inv, tokens, top_k, hidden, out,
                                             status);
    URB_CUDA(ctx, cudaGetLastError());
    return URB_OK;
}

int launch_combine_qwen(Ctx *ctx, const float *y, const float *shared_y, const int32_t *ids,
                        const float *w, const int32_t *inv, const float *gate_logit, int tokens,
                        int top_k, int hidden, float *out, cudaStream_t st, int32_t *status) {
    if (tokens <= 0) return URB_OK;
    if (top_k > 16) return set_error(ctx, URB_ERR_UNSUPPORTED, "Qwen3.6 combine takes top_k <= 16");
    dim3 grid(unsigned((hidden + 255) / 256), unsigned(tokens));
    URB_LAUNCH_DEP(k_combine_qwen, grid, 256, 0, st, y, shared_y, ids, w, inv, gate_logit, expf_table_of(ctx),
                                         tokens, top_k, hidden, out, status);
    URB_CUDA(ctx, cudaGetLastError());
    return URB_OK;
}

int launch_combine(Ctx *ctx, const float *y, const float *shared_y, const float *w,
                   const int32_t *inv, int tokens, int top_k, int hidden, float *out,
                   cudaStream_t st, const int32_t *status) {
    if (tokens <= 0) return URB_OK;
    const bool vec = hidden % 4 == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(out) & 15) == 0 &&
                     (!shared_y || (reinterpret_cast<uintptr_t>(shared_y) & 15) == 0);
    if (vec) {
        dim3 grid(unsigned((hidden / 4 + 127) / 128), unsigned(tokens));
        URB_LAUNCH_DEP(k_combine4, grid, 128, 0, st, y, shared_y, w, inv, tokens, top_k, hidden, out, status);
    } else {
        dim3 grid(unsigned((hidden + 255) / 256), unsigned(tokens));
        URB_LAUNCH_DEP(k_combine, grid, 256, 0, st, y, shared_y, w, inv, tokens, top_k, hidden, out, status);
    }
    URB_CUDA(ctx, cudaGetLastError());
    return URB_OK;
}

}  // namespace urb
