// route_noaux.cuh — route_noaux_tc (src/math/routing.rs:38-155) for one token, on one warp:
// IEEE f32 arithmetic in the reference's order, libm-exact expf, total_cmp ranking with the
// lower id winning ties.  Shared by the routing kernel (router.cu) and the decode grouping
// kernel that runs routing, grouping and the unit tables in one launch (moe.cu).
#pragma once
#include "expf_glibc.cuh"
#include "urb_internal.cuh"

namespace urb {
namespace {

struct RouteNoauxArgs {
    const float *logits, *bias;  // PRE: gates [tokens, E] and selection scores [tokens, E]
    int tokens, E, top_k, n_group, topk_group, normalize;
    float scaling;
    ExpfTable tab;
    int32_t *out_e;
    float *out_w, *out_s;
    int32_t *status;
    int warp_bytes;              // shared memory per token: gate[E], sel[E], group scores, flags
};

__device__ __forceinline__ bool rn_better(int32_t ka, int ia, int32_t kb, int ib) {
    return ka > kb || (ka == kb && ia < ib);
}

// Warp argmax over (key desc, id asc).
__device__ __forceinline__ void rn_warp_best(int32_t &key, int &id) {
    for (int o = 16; o > 0; o >>= 1) {
        int32_t k2 = __shfl_xor_sync(0xffffffffu, key, o);
        int i2 = __shfl_xor_sync(0xffffffffu, id, o);
        if (rn_better(k2, i2, key, id)) { key = k2; id = i2; }
    }
}

__device__ __forceinline__ void rn_set_status(int32_t *status, int code) {
    if (status) atomicCAS(status, 0, int32_t(code));
}

// Token t on the calling warp, wsmem its warp_bytes of shared memory; every return is taken by
// the whole warp together.  PRE: the gates and
// selection scores come precomputed (logits kernel epilogue, which also reported non-finite
// logits or biases) in `logits` / `bias` as [tokens, E] arrays.
template <bool PRE>
__device__ void route_noaux_token(const RouteNoauxArgs &ra, int t, uint8_t *wsmem) {
    const float *logits = ra.logits, *bias = ra.bias;
    const int E = ra.E, top_k = ra.top_k, n_group = ra.n_group, topk_group = ra.topk_group;
    const int normalize = ra.normalize;
    const float scaling = ra.scaling;
    const ExpfTable &tab = ra.tab;
    int32_t *out_e = ra.out_e;
    float *out_w = ra.out_w, *out_s = ra.out_s;
    int32_t *status = ra.status;
    const int lane = threadIdx.x & 31;
    float *gate = reinterpret_cast<float *>(wsmem);
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
        if (lane == 0) rn_set_status(status, URB_ERR_NONFINITE);
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
                if (rn_better(total_key(gscore[o]), o, kg, grp)) ++rank;
            const uint8_t allowed = rank < topk_group ? 1 : 0;
            for (int i = grp * gs; i < (grp + 1) * gs; ++i) flags[i] = allowed;
        }
        __syncwarp();
    }
    // routing.rs:131-141: top_k by selection desc, lower id wins ties.  The chosen ids go
    // straight to the output row; lane 0 accumulates the f32 denominator in ranking order.
    int32_t *oe = out_e + size_t(t) * top_k;
    float den = -0.0f;
    // Up to 512 experts: each lane keeps the keys of experts lane + 32 j in registers
    // (INT32_MIN marks masked or taken experts; no finite selection score has that key).
    constexpr int kRegKeys = 16;
    const bool in_regs = E <= 32 * kRegKeys;
    int32_t kr[kRegKeys];
#pragma unroll
    for (int j = 0; j < kRegKeys; ++j) {
        const int i = lane + 32 * j;
        kr[j] = in_regs && i < E && flags[i] == 1 ? total_key(sel[i]) : INT32_MIN;
    }
    for (int r = 0; r < top_k; ++r) {
        int32_t key = INT32_MIN;
        int id = INT32_MAX;
        if (in_regs) {
#pragma unroll
            for (int j = 0; j < kRegKeys; ++j)
                if (kr[j] != INT32_MIN && rn_better(kr[j], lane + 32 * j, key, id)) { key = kr[j]; id = lane + 32 * j; }
        } else {
            for (int i = lane; i < E; i += 32) {
                if (flags[i] == 1) {
                    int32_t k = total_key(sel[i]);
                    if (rn_better(k, i, key, id)) { key = k; id = i; }
                }
            }
        }
        rn_warp_best(key, id);
        if (id == INT32_MAX) {  // fewer allowed experts than top_k
            if (lane == 0) rn_set_status(status, URB_ERR_INVALID_GEOMETRY);
            for (int r2 = lane; r2 < top_k; r2 += 32) {
                out_e[size_t(t) * top_k + r2] = r2;
                out_w[size_t(t) * top_k + r2] = 0.0f;
            }
            return;
        }
        if (lane == (id & 31)) flags[id] = 2;
#pragma unroll
        for (int j = 0; j < kRegKeys; ++j)
            if (lane + 32 * j == id) kr[j] = INT32_MIN;
        if (lane == 0) {
            oe[r] = id;
            den = __fadd_rn(den, gate[id]);
        }
        __syncwarp();
    }
    if (lane == 0) den = __fadd_rn(den, 1e-20f);  // routing.rs:143-146
    den = __shfl_sync(0xffffffffu, den, 0);
    // Every lane leaves together (the caller may synchronise the block after this function).
    if (normalize && !isfinite(den)) {
        if (lane == 0) rn_set_status(status, URB_ERR_NONFINITE);
        return;
    }
    for (int r = lane; r < top_k; r += 32) {
        const int id = oe[r];
        const float w = normalize ? __fdiv_rn(gate[id], den) : gate[id];
        out_w[size_t(t) * top_k + r] = __fmul_rn(w, scaling);
        if (out_s) out_s[size_t(t) * top_k + r] = sel[id];
    }
}

// Arguments of route_noaux_token for tokens [0, tokens) (pre: the router epilogue's gates).
inline RouteNoauxArgs route_noaux_args(Ctx *ctx, const float *d_logits, const float *d_bias, int tokens,
                                int experts, const urb_moe_geometry &g, int32_t *d_expert,
                                float *d_weight, float *d_score, int32_t *d_status, const RouterGates *pre) {
    RouteNoauxArgs ra{};
    ra.logits = pre ? pre->gate : d_logits;
    ra.bias = pre ? pre->sel : d_bias;
    ra.tokens = tokens;
    ra.E = experts;
    ra.top_k = int(g.top_k);
    ra.n_group = int(g.n_group);
    ra.topk_group = int(g.topk_group);
    ra.normalize = g.normalize;
    ra.scaling = g.routed_scaling_factor;
    ra.tab = ExpfTable{ctx->expf_keys, ctx->expf_vals, ctx->expf_index};
    ra.out_e = d_expert;
    ra.out_w = d_weight;
    ra.out_s = d_score;
    ra.status = d_status;
    ra.warp_bytes = int(((2 * size_t(experts) + g.n_group) * 4 + experts + 15) & ~size_t(15));
    return ra;
}

}  // namespace
}  // namespace urb
