// layer.cu — MoE layer C ABI: construction checks of RuntimeMoeLayer::new and the forward
// pipeline (src/models/glm/runtime/moe.rs:88-176), all stream-ordered on the device:
//   row shifts -> exact router logits -> route_noaux_tc -> grouping -> grouped gate/up with
//   fused SwiGLU -> grouped down -> weighted f64 combine.
#include <cmath>
#include <cstdlib>
#include <cstring>

#include "urb_internal.cuh"
#include "urb_moe_internal.cuh"
#include "numerics.cuh"

namespace urb {
namespace {

size_t div_ceil(size_t a, size_t b) { return (a + b - 1) / b; }

struct Carve {
    uint8_t *base;
    size_t off = 0;
    template <class T>
    T *take(size_t n) {
        off = (off + 255) & ~size_t(255);
        T *p = reinterpret_cast<T *>(base + off);
        off += n * sizeof(T);
        return p;
    }
};

constexpr int kCap = 4;  // tokens per segment: hi/lo halves fill one 8-column n-block

size_t max_segments(size_t tokens, size_t K, size_t experts) {
    size_t TK = tokens * K;
    return std::min(TK, experts) + TK / kCap + div_ceil(tokens, kCap) + 2;
}

}  // namespace

// Upper bound of the work units of one tensor-core pass (mts 128-row tiles per sub-segment).
size_t max_bs_units(int fmt, size_t tokens, size_t K, size_t experts, size_t mts) {
    const size_t TK = tokens * K, cap = size_t(bs_cap(fmt));
    return mts * (TK / cap + std::min(TK, experts) + div_ceil(tokens, cap) + 1);
}

// Upper bound of the activation-stage bytes of one tensor-core pass: every sub-segment at the
// full MMA N (routed: at most TK / cap full ones plus one partial per expert; shared: T tokens).
size_t max_bs_bytes(int fmt, size_t tokens, size_t K, size_t experts, size_t ks) {
    const size_t TK = tokens * K;
    const size_t cap = size_t(bs_cap(fmt));
    const size_t subs = TK / cap + std::min(TK, experts) + div_ceil(tokens, cap) + 1;
    return subs * ks * size_t(bs_bstage_bytes(fmt, kBsNmax));
}

int route_device(Layer *L, const float *d_x, int T, const MoeWork &w, int32_t *d_status,
                 cudaStream_t st) {
    Ctx *ctx = L->ctx;
    const int E = int(L->experts), H = int(L->hidden);
    prof_begin(ctx, URB_K_ROUTER_LOGITS, st);
    // Exact logits, with the sigmoid gates and biased selection scores in the same kernel.
    const RouterGates rg{ctx, L->d_bias, w.gate, w.sel, d_status};
    int rc = launch_router_logits_f64(L->router64, E, d_x, T, H, w.x64, w.logits, st, &rg);
    prof_end(ctx, st);
    if (rc) return cuda_fail(ctx, cudaGetLastError(), "router logits");
    prof_begin(ctx, URB_K_ROUTE, st);
    rc = launch_route_noaux(ctx, w.logits, L->d_bias, T, E, L->geo, w.ids, w.w, w.score,
                            d_status, st, &rg);
    prof_end(ctx, st);
    return rc;
}

int moe_forward_device(Layer *L, const float *d_x, int T, float *d_out, MoeWork *wout,
                       int32_t *d_status, cudaStream_t st, const int32_t *d_ids_in,
                       const float *d_w_in, const Numerics *num) {
    Ctx *ctx = L->ctx;
    if (L->generic)
        return set_error(ctx, URB_ERR_UNSUPPORTED,
                         "layers with INT or mixed-format experts run through urb_moe_forward");
    const size_t E = L->experts, K = L->geo.top_k, H = L->hidden, I = L->inter;
    const size_t TK = size_t(T) * K, cols = TK + T;
    const size_t nseg = max_segments(T, K, E);
    size_t need = T * 4 + T * E * 4 + TK * 12 + E * 8 + 8 + TK * 12 + 2 * nseg * sizeof(Seg) +
                  64 + cols * 8 + cols * I * 4 + cols * H * 4 + T * 4 + 33 * 256;
    int rc;
    uint8_t *ws = static_cast<uint8_t *>(workspace(ctx, need, &rc));
    if (!ws) return rc;
    Carve cv{ws};
    MoeWork w{};
    w.shift = cv.take<int32_t>(T);
    w.logits = cv.take<float>(size_t(T) * E);
    w.x64 = cv.take<double>(router_f64_elems(T, int(H)));
    w.gate = cv.take<float>(size_t(T) * E);
    w.sel = cv.take<float>(size_t(T) * E);
    w.ids = cv.take<int32_t>(TK);
    w.w = cv.take<float>(TK);
    w.score = cv.take<float>(TK);
    w.counts = cv.take<int32_t>(E);
    w.offsets = cv.take<int32_t>(E + 1);
    w.perm_token = cv.take<int32_t>(TK);
    w.perm_slot = cv.take<int32_t>(TK);
    w.inv = cv.take<int32_t>(TK);
    w.segs_gu = cv.take<Seg>(nseg);
    w.segs_dn = cv.take<Seg>(nseg);
    w.scalars = cv.take<int>(4);
    w.col_src = cv.take<int32_t>(cols);
    w.maxexp = cv.take<int32_t>(cols);
    w.h = cv.take<float>(cols * I);
    w.y = cv.take<float>(cols * H);
    w.lofree = cv.take<int32_t>(1);
    w.col_w = cv.take<float>(cols);
    float *gate_logit = cv.take<float>(T);
    const bool deepseek = num && num->mode == URB_NUMERICS_DEEPSEEK_V4;
    const bool qwen = num && num->mode == URB_NUMERICS_QWEN36;
    if (deepseek && (!L->use_tc || !d_ids_in))
        return set_error(ctx, URB_ERR_UNSUPPORTED,
                         "DeepSeek-V4 numerics run on the tensor-core passes with caller routes");
    if (qwen) {
        // Qwen3.6: MX experts need the E4M3 simulation of the tensor-core prep; BF16 experts
        // run on the tensor-core passes too, or on the mma.sync passes (URB_MOE_PATH=mma).
        if (!d_ids_in || !L->sg || !L->shared_gate_row)
            return set_error(ctx, URB_ERR_UNSUPPORTED,
                             "Qwen3.6 numerics need caller routes, a shared expert and its gate");
        if (!L->use_tc && L->fmt != URB_FMT_BF16)
            return set_error(ctx, URB_ERR_UNSUPPORTED,
                             "Qwen3.6 numerics run MX experts on the tensor-core passes");
        if (K > 16) return set_error(ctx, URB_ERR_UNSUPPORTED, "Qwen3.6 combine takes top_k <= 16");
    }
    const size_t ngrp_gu = 2 * std::min(TK, E) + 2, ngrp_dn = std::min(TK, E) + 1;
    const size_t sc = size_t(bs_stage_cols(L->fmt));
    const size_t ks_gu = div_ceil(H, sc), ks_dn = div_ceil(I, sc);
    if (L->use_tc) {
        w.tsegs_gu = cv.take<TcSeg>(ngrp_gu);
        w.tsegs_dn = cv.take<TcSeg>(ngrp_dn);
        w.bslots_gu = cv.take<BsSlot>(cols);
        w.bslots_dn = cv.take<BsSlot>(cols);
        w.units_gu = cv.take<int>(max_bs_units(L->fmt, T, K, E, 2 * div_ceil(I, 128)));
        w.units_dn = cv.take<int>(max_bs_units(L->fmt, T, K, E, div_ceil(H, 128)));
        w.tscalars = cv.take<int>(4);
        w.bbuf_gu = cv.take<uint8_t>(max_bs_bytes(L->fmt, T, K, E, ks_gu));
        w.bbuf_dn = cv.take<uint8_t>(max_bs_bytes(L->fmt, T, K, E, ks_dn));
    }
    int32_t *own_status = cv.take<int32_t>(1);
    if (cv.off > ctx->ws_size) {
        // Grow to the exact size of this forward (nothing has been enqueued yet) and restart.
        if (!workspace(ctx, cv.off, &rc)) return rc;
        return moe_forward_device(L, d_x, T, d_out, wout, d_status, st, d_ids_in, d_w_in, num);
    }
    if (!d_status) {
        // No status word from the caller: the stages still short-circuit on a private one.
        d_status = own_status;
        URB_CUDA(ctx, cudaMemsetAsync(d_status, 0, 4, st));
    }
    w.status = d_status;
    if (!L->use_tc) {
        const int one = 1;
        URB_CUDA(ctx, cudaMemcpyAsync(w.lofree, &one, 4, cudaMemcpyHostToDevice, st));
        // Power-of-two row shifts of the mma.sync passes' f16 hi/lo activation columns.  The
        // tensor-core passes need none: non-finite inputs surface as non-finite router logits
        // (rejected by the routing kernel) or non-finite activations (rejected by the prep).
        prof_begin(ctx, URB_K_ROW_SHIFT, st);
        rc = launch_row_shift(d_x, T, int(H), int(H), w.shift, d_status, st, w.lofree,
                              L->fmt == URB_FMT_BF16 ? 1 : 0);
        prof_end(ctx, st);
        if (rc) return cuda_fail(ctx, cudaGetLastError(), "row shift");
    }
    if (qwen && !num->gate_logit) {
        // The shared expert's BF16 gate logit per token (qwen3_6/runtime.rs:1176-1186).
        prof_begin(ctx, URB_K_ROUTER_LOGITS, st);
        rc = launch_router_bf16_lanes(nullptr, 0,
                                      static_cast<const uint16_t *>(L->shared_gate_row->raw_values),
                                      d_x, T, int(H), nullptr, gate_logit, d_status, st);
        prof_end(ctx, st);
        if (rc) return cuda_fail(ctx, cudaGetLastError(), "shared expert gate");
    }
    const float *d_gate_logit = qwen ? (num->gate_logit ? num->gate_logit : gate_logit) : nullptr;
    // Decode (internal routing, tensor-core passes, up to 32 tokens): routing, grouping and
    // the pass tables run as one kernel after the router logits.
    const bool fused = !d_ids_in && L->use_tc && T <= 32;
    const bool x_ahead = fused && T == 1 && L->d_xslot && ctx->aux;
    const RouterGates rg{ctx, L->d_bias, w.gate, w.sel, d_status};
    if (d_ids_in) {
        // Routes chosen by the caller: the grouping validates the expert ids.
        w.ids = const_cast<int32_t *>(d_ids_in);
        w.w = const_cast<float *>(d_w_in);
    } else if (fused) {
        if (x_ahead) {
            // One token: every gate/up group multiplies the same x, so its activation terms
            // (one stage set, slot 0) need no routing and are written on the side stream while
            // the router runs; the gate/up pass joins it.
            TcArgs xa{};
            xa.bbuf = w.bbuf_gu;
            xa.src = d_x;
            xa.src_stride = int(H);
            xa.nrows = 1;
            xa.cols = int(H);
            xa.ks = int(ks_gu);
            xa.shared_col0 = -1;
            xa.slots = L->d_xslot;
            xa.status = d_status;
            URB_CUDA(ctx, cudaEventRecord(ctx->ev_fork, st));
            URB_CUDA(ctx, cudaStreamWaitEvent(ctx->aux, ctx->ev_fork, 0));
            rc = launch_tc_prep(ctx, L->fmt, xa, ctx->aux);
            if (rc) return rc;
            URB_CUDA(ctx, cudaEventRecord(ctx->ev_join, ctx->aux));
        }
        prof_begin(ctx, URB_K_ROUTER_LOGITS, st);
        rc = launch_router_logits_f64(L->router64, int(E), d_x, T, int(H), w.x64, w.logits, st, &rg);
        prof_end(ctx, st);
        if (rc) return cuda_fail(ctx, cudaGetLastError(), "router logits");
    } else {
        rc = route_device(L, d_x, T, w, d_status, st);
        if (rc) return rc;
    }

    const Mat *g0 = L->gate[0], *d0 = L->down[0];
    void **tb = L->d_tables;
    const size_t S = L->e_count + 1;  // table stride
    PermArgs p{};
    p.ids = w.ids;
    p.tokens = T;
    p.top_k = int(K);
    p.experts = int(E);
    p.cap = kCap;
    p.counts = w.counts;
    p.offsets = w.offsets;
    p.perm_token = w.perm_token;
    p.perm_slot = w.perm_slot;
    p.inv = w.inv;
    p.segs_gu = w.segs_gu;
    p.segs_dn = w.segs_dn;
    p.nsegs_gu = w.scalars;
    p.total_rows_gu = w.scalars + 1;
    p.nsegs_dn = w.scalars + 2;
    p.total_rows_dn = w.scalars + 3;
    p.col_src = w.col_src;
    p.maxexp = w.maxexp;
    p.gate_tiles = reinterpret_cast<const uint8_t *const *>(tb);
    p.up_tiles = reinterpret_cast<const uint8_t *const *>(tb + S);
    p.down_tiles = reinterpret_cast<const uint8_t *const *>(tb + 2 * S);
    p.gate_rexp = reinterpret_cast<const int8_t *const *>(tb + 3 * S);
    p.up_rexp = reinterpret_cast<const int8_t *const *>(tb + 4 * S);
    p.down_rexp = reinterpret_cast<const int8_t *const *>(tb + 5 * S);
    p.shared_in_pass = L->sg ? 1 : 0;
    if (L->sg) {
        p.sh_gate_tiles = L->sg->tiles; p.sh_gate_rexp = L->sg->row_exp;
        p.sh_up_tiles = L->su->tiles; p.sh_up_rexp = L->su->row_exp;
        p.sh_down_tiles = L->sd->tiles; p.sh_down_rexp = L->sd->row_exp;
    }
    p.hidden = int(H);
    p.inter = int(I);
    p.gu_rbs = g0->rbs;
    p.gu_kslices = g0->kslices;
    p.dn_rbs = d0->rbs;
    p.dn_kslices = d0->kslices;
    p.status = d_status;
    p.lofree = w.lofree;
    if (L->use_tc) {  // the tensor-core passes need only the grouping itself
        p.segs_gu = nullptr;
        p.col_src = nullptr;
    }
    if (deepseek) {  // route weights move to the columns (applied before the down projection)
        p.route_w = w.w;
        p.col_w = w.col_w;
    }
    if (!fused) {
        prof_begin(ctx, URB_K_PERMUTE, st);
        rc = launch_permute(ctx, p, st);
        prof_end(ctx, st);
        if (rc) return rc;
    }

    if (L->use_tc) {
        TcBuildArgs bb{};
        bb.counts = w.counts;
        bb.offsets = w.offsets;
        bb.fmt = L->fmt;
        bb.tokens = T;
        bb.top_k = int(K);
        bb.experts = int(E);
        bb.gate_tc = reinterpret_cast<const uint8_t *const *>(tb + 6 * S);
        bb.up_tc = reinterpret_cast<const uint8_t *const *>(tb + 7 * S);
        bb.down_tc = reinterpret_cast<const uint8_t *const *>(tb + 8 * S);
        bb.has_shared = L->sg ? 1 : 0;
        bb.shared_tokens = T;
        bb.pair_down = 1;
        if (L->sg) {
            bb.sh_gate_tc = tc_src(L->sg);
            bb.sh_up_tc = tc_src(L->su);
            bb.sh_down_tc = tc_src(L->sd);
        }
        bb.hidden = int(H);
        bb.inter = int(I);
        bb.gu = w.tsegs_gu;
        bb.dn = w.tsegs_dn;
        bb.gu_slots = w.bslots_gu;
        bb.dn_slots = w.bslots_dn;
        bb.gu_units = w.units_gu;
        bb.dn_units = w.units_dn;
        bb.scalars = w.tscalars;
        bb.status = d_status;
        bb.shared_x = x_ahead ? 1 : 0;
        if (fused) {
            prof_begin(ctx, URB_K_ROUTE, st);
            rc = launch_decode_group(ctx, rg, T, int(E), L->geo, w.ids, w.w, w.score, p, bb, st);
            prof_end(ctx, st);
            if (rc == URB_ERR_UNSUPPORTED) {  // too many experts for one CTA's shared memory
                rc = launch_route_noaux(ctx, w.logits, L->d_bias, T, int(E), L->geo, w.ids, w.w, w.score,
                                        d_status, st, &rg);
                if (!rc) rc = launch_permute(ctx, p, st);
                if (!rc) rc = launch_build_tc_segs(ctx, bb, st);
            }
        } else {
            prof_begin(ctx, URB_K_GROUP_BUILD, st);
            rc = launch_build_tc_segs(ctx, bb, st);
            prof_end(ctx, st);
        }
        if (rc) return rc;

        // Gate and up projections of every (expert, token) column: [cols, 2I] gate | up.
        TcArgs ga{};
        ga.segs = w.tsegs_gu;
        ga.nsegs = w.tscalars;
        ga.total_units = w.tscalars + 1;
        ga.unit_group = w.units_gu;
        ga.bbuf = w.bbuf_gu;
        ga.src = d_x;
        ga.src_stride = int(H);
        ga.nrows = T;
        ga.cols = int(H);
        ga.ks = int(ks_gu);
        ga.swiglu = 0;
        ga.inv = w.inv;
        ga.top_k = int(K);
        ga.shared_col0 = L->sg ? int(TK) : -1;
        ga.shared_row0 = 0;
        ga.shared_rows = T;
        ga.slots = w.bslots_gu;
        ga.pair = 1;  // gate and up tiles of an expert together; the epilogue writes h
        // MX weights see the checkpoint's E4M3 activation simulation; BF16 weights see the
        // activations as they are (qwen3_8/math.rs:10-26).
        const bool mx = L->fmt != URB_FMT_BF16;
        if (deepseek) {
            ga.variant = 1;
            ga.sim128 = mx ? 1 : 0;
            ga.limit = num->limit;
            ga.col_w = w.col_w;
        } else if (qwen) {
            ga.variant = 2;
            ga.sim128 = mx ? 2 : 0;
            ga.full_terms = 1;
            ga.expf = expf_table_of(ctx);
        }
        ga.out = w.h;
        ga.out_stride = int(I);
        ga.status = d_status;
        if (x_ahead) {
            ga.skip_prep = 1;
            URB_CUDA(ctx, cudaStreamWaitEvent(st, ctx->ev_join, 0));
        }
        rc = launch_tc_grouped(ctx, L->fmt, ga, URB_K_GATE_UP, st);
        if (rc) return rc;

        // Down projection of h = silu(gate) * up.
        TcArgs da{};
        da.segs = w.tsegs_dn;
        da.nsegs = w.tscalars + 2;
        da.total_units = w.tscalars + 3;
        da.unit_group = w.units_dn;
        da.bbuf = w.bbuf_dn;
        da.src = w.h;
        da.src_stride = int(I);
        da.nrows = int(L->sg ? TK + T : TK);
        da.pair = 2;  // neighbouring row tiles share each activation stage
        if (deepseek || qwen) {
            da.variant = deepseek ? 1 : 2;
            da.sim128 = !mx ? 0 : (deepseek ? 1 : 2);
            da.full_terms = qwen ? 1 : 0;
        }
        da.cols = int(I);
        da.ks = int(ks_dn);
        da.slots = w.bslots_dn;
        da.out = w.y;
        da.out_stride = int(H);
        da.status = d_status;
        rc = launch_tc_grouped(ctx, L->fmt, da, URB_K_DOWN, st);
        if (rc) return rc;

        prof_begin(ctx, URB_K_COMBINE, st);
        if (deepseek)
            rc = launch_combine_deepseek(ctx, w.y, L->sg ? w.y + TK * H : nullptr, w.ids, w.inv, T,
                                         int(K), int(H), d_out, st, d_status);
        else if (qwen)
            rc = launch_combine_qwen(ctx, w.y, w.y + TK * H, w.ids, w.w, w.inv, d_gate_logit, T,
                                     int(K), int(H), d_out, st, d_status);
        else
            rc = launch_combine(ctx, w.y, L->sg ? w.y + TK * H : nullptr, w.w, w.inv, T, int(K),
                                int(H), d_out, st, d_status);
        prof_end(ctx, st);
        if (rc) return rc;
        if (wout) *wout = w;
        return URB_OK;
    }

    // Upper bound of work rows per SM picks how many warps share a row block.
    const long est_rows_gu = long(std::min(nseg, TK + div_ceil(T, kCap))) * 16 * g0->rbs;
    const long est_per_sm = est_rows_gu / std::max(1, ctx->num_sms);
    const int ksplit = est_per_sm < 64 ? 8 : (est_per_sm < 256 ? 2 : 1);

    GroupArgs gu{};
    gu.segs = w.segs_gu;
    gu.nsegs = w.scalars;
    gu.total_rows = w.scalars + 1;
    gu.src = d_x;
    gu.src_stride = int(H);
    gu.col_src = w.col_src;
    gu.src_shift = w.shift;
    gu.out = w.h;
    gu.out_stride = int(I);
    gu.out_maxexp = w.maxexp;
    gu.hilo = 1;
    gu.lofree = w.lofree;  // bf16-exact tokens: 8 per segment in one f16 column each
    if (qwen) {
        gu.variant = 2;
        gu.status = d_status;
        gu.expf = expf_table_of(ctx);
    }
    prof_begin(ctx, URB_K_GATE_UP, st);
    rc = launch_grouped_ex(ctx, L->fmt, true, ksplit, gu, 2 * kCap, g0->kslices, st);
    prof_end(ctx, st);
    if (rc) return rc;

    GroupArgs dn{};
    dn.segs = w.segs_dn;
    dn.nsegs = w.scalars + 2;
    dn.total_rows = w.scalars + 3;
    dn.src = w.h;
    dn.src_stride = int(I);
    dn.col_src = nullptr;
    dn.src_shift = nullptr;
    dn.src_maxexp = w.maxexp;
    dn.out = w.y;
    dn.out_stride = int(H);
    dn.hilo = 1;
    if (qwen) {
        dn.variant = 2;
        dn.status = d_status;
    }
    prof_begin(ctx, URB_K_DOWN, st);
    rc = launch_grouped_ex(ctx, L->fmt, false, ksplit == 8 ? 2 : ksplit, dn, 4 * kCap,
                           d0->kslices, st);
    prof_end(ctx, st);
    if (rc) return rc;

    prof_begin(ctx, URB_K_COMBINE, st);
    if (qwen)
        rc = launch_combine_qwen(ctx, w.y, w.y + TK * H, w.ids, w.w, w.inv, d_gate_logit, T,
                                 int(K), int(H), d_out, st, d_status);
    else
        rc = launch_combine(ctx, w.y, L->sg ? w.y + TK * H : nullptr, w.w, w.inv, T, int(K),
                            int(H), d_out, st, d_status);
    prof_end(ctx, st);
    if (rc) return rc;
    if (wout) *wout = w;
    return URB_OK;
}

// GatedMlp::forward (src/model/mlp.rs:90-99) for `T` tokens on the device: one grouped pair
// pass (gate/up with fused SwiGLU) and one grouped down pass, host-built segments; BF16
// projections with few tokens take the streaming CUDA-core passes instead.
// h = silu(gate) * up in f32 with libm's expf (src/model/mlp.rs:90-99, src/math/ops.rs:36-38).
__global__ void k_swiglu_rows(const float *gate, const float *up, size_t n, ExpfTable tab, float *h) {
    const size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x;
    if (i < n) h[i] = __fmul_rn(num_silu_libm(gate[i], tab), up[i]);
}

// GatedMlp::forward over projections without one shared tiled layout: INT8 / INT4 (GLM's
// converted experts), F32, MX shapes the tiles do not cover, or the mixed formats
// GatedMlp::new_mixed accepts (mlp.rs:60-81).  Three row products (each format's own kernel)
// and one SwiGLU pass.
int gated_mlp_generic(Ctx *ctx, const Mat *g, const Mat *u, const Mat *d, const float *d_x, int T,
                      float *d_out, int32_t *d_status, cudaStream_t st) {
    const size_t I = g->rows, n = size_t(T) * I;
    float *buf = nullptr;
    URB_CUDA(ctx, cudaMallocAsync(&buf, 2 * n * sizeof(float), st));
    int rc = product_device(ctx, g, 0, I, d_x, size_t(T), buf, d_status, st);
    if (rc == URB_OK) rc = product_device(ctx, u, 0, I, d_x, size_t(T), buf + n, d_status, st);
    if (rc == URB_OK) {
        k_swiglu_rows<<<unsigned((n + 255) / 256), 256, 0, st>>>(buf, buf + n, n, expf_table_of(ctx), buf);
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) rc = cuda_fail(ctx, e, "swiglu");
    }
    if (rc == URB_OK) rc = product_device(ctx, d, 0, d->rows, buf, size_t(T), d_out, d_status, st);
    cudaFreeAsync(buf, st);
    return rc;
}

// dst[i] = src[idx[i]] (rows of H floats).
__global__ void k_gather_rows(const float *src, const int32_t *idx, size_t n, int H, float *dst) {
    const size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x;
    if (i < n * H) dst[i] = src[size_t(idx[i / H]) * H + i % H];
}

// dst[idx[i]] = src[i] (rows of H floats).
__global__ void k_scatter_rows(const float *src, const int32_t *idx, size_t n, int H, float *dst) {
    const size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x;
    if (i < n * H) dst[size_t(idx[i / H]) * H + i % H] = src[i];
}

// glm/runtime/moe.rs:164-175: out = f32(f64(shared) + sum over routes in selection order of
// f64(weight) * f64(expert output)); the product of two f32 values is exact in f64.
__global__ void k_combine_glm(const float *shared, const float *y, const float *w, int T, int K,
                              int H, float *out) {
    const size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x;
    if (i >= size_t(T) * H) return;
    const size_t t = i / H, h = i % H;
    double acc = shared ? double(shared[i]) : 0.0;
    for (int k = 0; k < K; ++k)
        acc = __dadd_rn(acc, __dmul_rn(double(w[t * K + k]), double(y[(t * K + k) * H + h])));
    out[i] = float(acc);
}

int gated_mlp_device(Ctx *ctx, const Mat *g, const Mat *u, const Mat *d, const float *d_x, int T,
                     float *d_out, int32_t *d_status, cudaStream_t st);

// RuntimeMoeLayer::forward (glm/runtime/moe.rs:138-176) for layers whose experts have no
// shared tiled layout: the exact router and noaux_tc routing on the device, the routes read
// back, each selected expert's GatedMlp over its tokens (grouped experts ascending, tokens
// ascending, as qwen3_6/runtime.rs:1083-1132), then the f64 combine.  Host outputs as
// urb_moe_forward; the grouping outputs are filled on the host.
int moe_forward_generic(Layer *L, const float *d_x, int T, float *d_out, int32_t *h_ids,
                        float *h_w, float *h_score, float *h_logits, int32_t *h_counts,
                        int32_t *h_perm_token, int32_t *h_perm_slot, int32_t *d_status,
                        cudaStream_t st) {
    Ctx *ctx = L->ctx;
    const size_t E = L->experts, K = L->geo.top_k, H = L->hidden, TK = size_t(T) * K;
    const size_t bytes = size_t(T) * E * 4 * 3 + router_f64_elems(T, int(H)) * 8 + TK * 4 * 5 +
                         3 * TK * H * 4 + size_t(T) * H * 4 + 16 * 256;
    uint8_t *buf = nullptr;
    URB_CUDA(ctx, cudaMallocAsync(&buf, bytes, st));
    // Every exit after the allocation releases it (stream-ordered).
#define URB_CUDA_DONE(expr)                                                    \
    do {                                                                       \
        cudaError_t _e = (expr);                                               \
        if (_e != cudaSuccess) return done(cuda_fail(ctx, _e, #expr));         \
    } while (0)
    Carve cv{buf};
    MoeWork w{};
    w.logits = cv.take<float>(size_t(T) * E);
    w.gate = cv.take<float>(size_t(T) * E);
    w.sel = cv.take<float>(size_t(T) * E);
    w.x64 = cv.take<double>(router_f64_elems(T, int(H)));
    w.ids = cv.take<int32_t>(TK);
    w.w = cv.take<float>(TK);
    w.score = cv.take<float>(TK);
    int32_t *d_tok = cv.take<int32_t>(TK), *d_slot = cv.take<int32_t>(TK);
    float *xe = cv.take<float>(TK * H), *ye = cv.take<float>(TK * H), *y = cv.take<float>(TK * H);
    float *shared = cv.take<float>(size_t(T) * H);
    auto done = [&](int rc) { cudaFreeAsync(buf, st); return rc; };
    int rc = route_device(L, d_x, T, w, d_status, st);
    if (rc) return done(rc);
    std::vector<int32_t> ids(TK);
    int32_t status = 0;
    URB_CUDA_DONE(cudaMemcpyAsync(ids.data(), w.ids, TK * 4, cudaMemcpyDeviceToHost, st));
    URB_CUDA_DONE(cudaMemcpyAsync(&status, d_status, 4, cudaMemcpyDeviceToHost, st));
    URB_CUDA_DONE(cudaStreamSynchronize(st));
    if (status) return done(set_error(ctx, status, "MoE forward rejected its input"));
    std::vector<int32_t> counts(E, 0), offsets(E + 1, 0), tok(TK), slot(TK), pslot(TK);
    for (size_t i = 0; i < TK; ++i) counts[ids[i]]++;
    for (size_t e = 0; e < E; ++e) offsets[e + 1] = offsets[e] + counts[e];
    std::vector<int32_t> cursor(offsets.begin(), offsets.end() - 1);
    for (size_t t = 0; t < size_t(T); ++t)
        for (size_t k = 0; k < K; ++k) {
            const int32_t p = cursor[ids[t * K + k]]++;
            tok[p] = int32_t(t);
            pslot[p] = int32_t(k);
            slot[p] = int32_t(t * K + k);
        }
    URB_CUDA_DONE(cudaMemcpyAsync(d_tok, tok.data(), TK * 4, cudaMemcpyHostToDevice, st));
    URB_CUDA_DONE(cudaMemcpyAsync(d_slot, slot.data(), TK * 4, cudaMemcpyHostToDevice, st));
    const unsigned gb = unsigned((TK * H + 255) / 256);
    k_gather_rows<<<gb, 256, 0, st>>>(d_x, d_tok, TK, int(H), xe);
    for (size_t e = 0; e < E && rc == URB_OK; ++e)
        if (counts[e])
            rc = gated_mlp_device(ctx, L->gate[e], L->up[e], L->down[e], xe + size_t(offsets[e]) * H,
                                  counts[e], ye + size_t(offsets[e]) * H, d_status, st);
    if (rc) return done(rc);
    k_scatter_rows<<<gb, 256, 0, st>>>(ye, d_slot, TK, int(H), y);
    if (L->sg) rc = gated_mlp_device(ctx, L->sg, L->su, L->sd, d_x, T, shared, d_status, st);
    if (rc) return done(rc);
    k_combine_glm<<<unsigned((size_t(T) * H + 255) / 256), 256, 0, st>>>(L->sg ? shared : nullptr, y, w.w,
                                                                       T, int(K), int(H), d_out);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return done(cuda_fail(ctx, e, "generic MoE forward"));
    if (h_ids) std::copy(ids.begin(), ids.end(), h_ids);
    if (h_w) URB_CUDA_DONE(cudaMemcpyAsync(h_w, w.w, TK * 4, cudaMemcpyDefault, st));
    if (h_score) URB_CUDA_DONE(cudaMemcpyAsync(h_score, w.score, TK * 4, cudaMemcpyDefault, st));
    if (h_logits) URB_CUDA_DONE(cudaMemcpyAsync(h_logits, w.logits, size_t(T) * E * 4, cudaMemcpyDefault, st));
    if (h_counts) std::copy(counts.begin(), counts.end(), h_counts);
    if (h_perm_token) std::copy(tok.begin(), tok.end(), h_perm_token);
    if (h_perm_slot) std::copy(pslot.begin(), pslot.end(), h_perm_slot);
    return done(URB_OK);
#undef URB_CUDA_DONE
}

int gated_mlp_device(Ctx *ctx, const Mat *g, const Mat *u, const Mat *d, const float *d_x, int T,
                     float *d_out, int32_t *d_status, cudaStream_t st) {
    const size_t H = g->cols, I = g->rows;
    int rc;
    // BF16 projections, 1..32 tokens: split-K tcgen05 passes (split_tc.cu).
    if (split_tc_applies(g, size_t(T)) && u->format == g->format && d->format == g->format) {
        float *h = static_cast<float *>(workspace(ctx, size_t(T) * I * 4 + 256, &rc));
        if (!h) return rc;
        rc = split_tc_mlp(ctx, g, u, d, d_x, T, h, d_out, d_status, st);
        if (rc != URB_ERR_UNSUPPORTED) return rc;
    }
    // MX projections (resident tcgen05 tiles) and BF16 ones (tensor maps): the grouped
    // tensor-core passes with every token in one group.
    if (dense_tc_mlp_applies(g, u, d))
        return dense_tc_mlp(ctx, g, u, d, d_x, T, d_out, d_status, st, nullptr, 0);
    if (!(g->tiled && u->tiled && d->tiled && g->format == u->format))
        return gated_mlp_generic(ctx, g, u, d, d_x, T, d_out, d_status, st);
    const int nseg = int(div_ceil(T, kCap));
    if (bf16_gemv_applies(g, T) && bf16_gemv_applies(u, T) && bf16_gemv_applies(d, T)) {
        // BF16 projections, a few tokens: two streaming passes (gate/up with SwiGLU, down).
        float *h = static_cast<float *>(workspace(ctx, size_t(T) * I * 4 + 256, &rc));
        if (!h) return rc;
        rc = launch_bf16_swiglu(ctx, g, u, d, d_x, T, h, d_out, d_status, st);
        if (rc != URB_ERR_UNSUPPORTED) return rc;
    }
    size_t need = T * 4 + 2 * nseg * sizeof(Seg) + 64 + T * 4 + size_t(T) * I * 4 + 8 * 256;
    uint8_t *ws = static_cast<uint8_t *>(workspace(ctx, need, &rc));
    if (!ws) return rc;
    Carve cv{ws};
    int32_t *shift = cv.take<int32_t>(T);
    Seg *segs = cv.take<Seg>(2 * nseg);
    int *sc = cv.take<int>(4);
    int32_t *maxexp = cv.take<int32_t>(T);
    float *h = cv.take<float>(size_t(T) * I);
    std::vector<Seg> hs(2 * nseg);
    for (int i = 0; i < nseg; ++i) {
        Seg &a = hs[i], &b = hs[nseg + i];
        a.tiles_a = g->tiles; a.rexp_a = g->row_exp; a.tiles_b = u->tiles; a.rexp_b = u->row_exp;
        a.rbs = g->rbs; a.rows = int(I); a.kslices = g->kslices; a.cols = int(H);
        a.col_begin = i * kCap; a.ntok = std::min(kCap, T - i * kCap);
        a.row_begin = i * 16 * g->rbs; a.pad = 0;
        b.tiles_a = d->tiles; b.rexp_a = d->row_exp; b.tiles_b = nullptr; b.rexp_b = nullptr;
        b.rbs = d->rbs; b.rows = int(H); b.kslices = d->kslices; b.cols = int(I);
        b.col_begin = a.col_begin; b.ntok = a.ntok; b.row_begin = i * 16 * d->rbs; b.pad = 0;
    }
    int hsc[4] = {nseg, nseg * 16 * g->rbs, nseg, nseg * 16 * d->rbs};
    URB_CUDA(ctx, cudaMemcpyAsync(segs, hs.data(), hs.size() * sizeof(Seg), cudaMemcpyHostToDevice, st));
    URB_CUDA(ctx, cudaMemcpyAsync(sc, hsc, sizeof(hsc), cudaMemcpyHostToDevice, st));
    if (launch_row_shift(d_x, T, int(H), int(H), shift, d_status, st))
        return cuda_fail(ctx, cudaGetLastError(), "row shift");
    std::vector<int32_t> neg(T, -1000);
    URB_CUDA(ctx, cudaMemcpyAsync(maxexp, neg.data(), size_t(T) * 4, cudaMemcpyHostToDevice, st));
    GroupArgs a{};
    a.segs = segs; a.nsegs = sc; a.total_rows = sc + 1;
    a.src = d_x; a.src_stride = int(H); a.src_shift = shift;
    a.out = h; a.out_stride = int(I); a.out_maxexp = maxexp; a.hilo = 1;
    const long per_sm_gu = long(hsc[1]) / std::max(1, ctx->num_sms);
    prof_begin(ctx, URB_K_GATE_UP, st);
    rc = launch_grouped_ex(ctx, g->format, true, per_sm_gu < 64 ? 8 : per_sm_gu < 256 ? 2 : 1, a,
                           2 * kCap, g->kslices, st);
    prof_end(ctx, st);
    if (rc) return rc;
    GroupArgs b{};
    b.segs = segs + nseg; b.nsegs = sc + 2; b.total_rows = sc + 3;
    b.src = h; b.src_stride = int(I); b.src_maxexp = maxexp;
    b.out = d_out; b.out_stride = int(H); b.hilo = 1;
    const long per_sm_dn = long(hsc[3]) / std::max(1, ctx->num_sms);
    prof_begin(ctx, URB_K_DOWN, st);
    rc = launch_grouped_ex(ctx, d->format, false, per_sm_dn < 64 ? 8 : per_sm_dn < 256 ? 2 : 1,
                           b, 2 * kCap, d->kslices, st);
    prof_end(ctx, st);
    return rc;
}

}  // namespace urb

using namespace urb;

extern "C" {

static int create_layer(urb_ctx *ctx, const urb_mat *router, const float *bias, size_t experts,
                        size_t e_begin, size_t e_count, const urb_mat *const *gate,
                        const urb_mat *const *up, const urb_mat *const *down, const urb_mat *sg,
                        const urb_mat *su, const urb_mat *sd, const urb_moe_geometry *geo,
                        urb_layer **out) {
    if (!ctx || !router || !bias || !gate || !up || !down || !geo || !out || e_count == 0)
        return URB_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    cudaSetDevice(ctx->device);
    *out = nullptr;
    // RuntimeMoeLayer::new (glm/runtime/moe.rs:88-129).
    if (router->rows == 0 || router->cols == 0)
        return set_error(ctx, URB_ERR_INVALID_GEOMETRY, "router dimensions must be non-zero");
    if (experts != router->rows)
        return set_error(ctx, URB_ERR_SHAPE, "router rows differ from the correction bias length");
    for (size_t e = 0; e < experts; ++e)
        if (!std::isfinite(bias[e]))
            return set_error(ctx, URB_ERR_INVALID_GEOMETRY, "correction bias contains NaN or infinity");
    const size_t H = router->cols;
    bool have_shared = sg && su && sd;
    if (!have_shared && (sg || su || sd))
        return set_error(ctx, URB_ERR_INVALID_ARGUMENT, "shared expert needs gate, up and down");
    if (have_shared && sg->cols != H)
        return set_error(ctx, URB_ERR_SHAPE, "router hidden size differs from the shared expert");
    // route_noaux_tc on zero logits validates the geometry (moe.rs:113-121).
    if (!std::isfinite(geo->routed_scaling_factor))
        return set_error(ctx, URB_ERR_NONFINITE, "routed_scaling_factor is not finite");
    if (geo->routed_scaling_factor <= 0.0f || geo->n_group == 0 || experts % geo->n_group ||
        geo->top_k == 0 || geo->top_k > experts || geo->topk_group == 0 ||
        geo->topk_group > geo->n_group || experts / geo->n_group < 2 ||
        size_t(geo->topk_group) * (experts / geo->n_group) < geo->top_k)
        return set_error(ctx, URB_ERR_INVALID_GEOMETRY, "invalid noaux_tc geometry");
    if (router->format != URB_FMT_BF16 && router->format != URB_FMT_F32)
        return set_error(ctx, URB_ERR_UNSUPPORTED, "router must be BF16 or F32 for exact logits");
    // GatedMlp::new_mixed shape contract (src/model/mlp.rs:60-81) for every expert, plus this
    // build's requirement that all experts share one tiled format and shape.
    const int fmt = gate[0]->format;
    const size_t I = gate[0]->rows;
    auto check_mlp = [&](const urb_mat *g, const urb_mat *u, const urb_mat *d) -> int {
        if (!g || !u || !d) return URB_ERR_INVALID_ARGUMENT;
        if (g->rows != u->rows || g->cols != u->cols) return URB_ERR_SHAPE;
        if (d->cols != g->rows || d->rows != g->cols) return URB_ERR_SHAPE;
        if (g->cols != H || g->rows != I) return URB_ERR_SHAPE;
        return URB_OK;
    };
    // Experts outside one shared tiled format compose per-expert GatedMlp calls.
    auto tiled_mlp = [&](const urb_mat *g, const urb_mat *u, const urb_mat *d) {
        return g->tiled && u->tiled && d->tiled && g->format == fmt && u->format == fmt &&
               d->format == fmt;
    };
    if (e_begin + e_count > experts || e_begin + e_count < e_begin)
        return set_error(ctx, URB_ERR_SHAPE, "expert shard range exceeds the router's experts");
    for (size_t e = 0; e < e_count; ++e) {
        int rc = check_mlp(gate[e], up[e], down[e]);
        if (rc) return set_error(ctx, rc, "routed expert shape/format is not supported");
    }
    if (have_shared) {
        int rc = check_mlp(sg, su, sd);
        if (rc) return set_error(ctx, rc, "shared expert shape/format is not supported");
    }
    // MX experts with tcgen05 tiles take the tensor-core passes whatever their scale range; BF16
    // experts take them (kind::f16) through their tensor maps.
    auto tc_mlp = [&](const urb_mat *g, const urb_mat *u, const urb_mat *d) {
        return (fmt == URB_FMT_MXFP4 || fmt == URB_FMT_MXFP8 || fmt == URB_FMT_BF16) &&
               g->format == fmt && u->format == fmt && d->format == fmt && tc_src(g) && tc_src(u) &&
               tc_src(d);
    };
    bool generic = false;
    for (size_t e = 0; e < e_count; ++e)
        generic |= !(tiled_mlp(gate[e], up[e], down[e]) || tc_mlp(gate[e], up[e], down[e]));
    if (have_shared) generic |= !(tiled_mlp(sg, su, sd) || tc_mlp(sg, su, sd));
    const char *path = std::getenv("URB_MOE_PATH");
    bool have_tc = !generic && (fmt == URB_FMT_MXFP4 || fmt == URB_FMT_MXFP8 || fmt == URB_FMT_BF16);
    for (size_t e = 0; e < e_count && have_tc; ++e) have_tc = tc_mlp(gate[e], up[e], down[e]);
    if (have_shared) have_tc = have_tc && tc_mlp(sg, su, sd);
    // tcgen05 passes by default; URB_MOE_PATH=mma selects the mma.sync passes, which need every
    // expert in that layout (MX experts build it now from their tcgen05 tiles).
    const bool use_tc = have_tc && !(path && std::strcmp(path, "mma") == 0);
    if (!use_tc && !generic) {
        for (size_t e = 0; e < e_count; ++e) generic |= !tiled_mlp(gate[e], up[e], down[e]);
        if (have_shared) generic |= !tiled_mlp(sg, su, sd);
    }
    if (!use_tc && !generic) {
        auto build = [&](const urb_mat *m) { return ensure_mma_tiles(ctx, m, ctx->stream); };
        for (size_t e = 0; e < e_count; ++e) {
            int rc = build(gate[e]);
            if (!rc) rc = build(up[e]);
            if (!rc) rc = build(down[e]);
            if (rc) return rc;
        }
        if (have_shared) {
            int rc = build(sg);
            if (!rc) rc = build(su);
            if (!rc) rc = build(sd);
            if (rc) return rc;
        }
    }
    urb_layer *L = new urb_layer();
    L->generic = generic;
    L->ctx = ctx;
    L->router = router;
    L->experts = experts;
    L->e_begin = e_begin;
    L->e_count = e_count;
    L->hidden = H;
    L->inter = I;
    L->fmt = fmt;
    L->geo = *geo;
    L->gate.assign(gate, gate + e_count);
    L->up.assign(up, up + e_count);
    L->down.assign(down, down + e_count);
    if (have_shared) { L->sg = sg; L->su = su; L->sd = sd; }
    const size_t S = e_count + 1;  // held experts, then the shared expert
    std::vector<void *> tables(9 * S, nullptr);
    auto put = [&](size_t e, const Mat *g, const Mat *u, const Mat *d) {
        tables[e] = g->tiles;
        tables[S + e] = u->tiles;
        tables[2 * S + e] = d->tiles;
        tables[3 * S + e] = g->row_exp;
        tables[4 * S + e] = u->row_exp;
        tables[5 * S + e] = d->row_exp;
        tables[6 * S + e] = const_cast<uint8_t *>(tc_src(g));
        tables[7 * S + e] = const_cast<uint8_t *>(tc_src(u));
        tables[8 * S + e] = const_cast<uint8_t *>(tc_src(d));
    };
    for (size_t e = 0; e < e_count; ++e) put(e, gate[e], up[e], down[e]);
    if (have_shared) put(e_count, sg, su, sd);
    L->use_tc = use_tc && !generic;
    if (e_count != experts && !have_tc) {
        delete L;
        return set_error(ctx, URB_ERR_UNSUPPORTED,
                         "expert shards need experts the tensor-core passes take (MX, or BF16 with cols % 8 == 0)");
    }
    cudaError_t err = cudaMalloc(&L->d_tables, tables.size() * sizeof(void *));
    if (err == cudaSuccess)
        err = cudaMalloc(&L->router64, router_f64_elems(int(experts), int(H)) * sizeof(double));
    if (err == cudaSuccess && widen_router_f64(router, L->router64, ctx->stream) != URB_OK)
        err = cudaGetLastError();
    if (err == cudaSuccess) err = cudaMalloc(&L->d_bias, experts * 4);
    if (err == cudaSuccess && L->use_tc) {
        const BsSlot xs{0, 0, (bs_rows_per_tok(L->fmt) + 15) & ~15};
        err = cudaMalloc(&L->d_xslot, sizeof(BsSlot));
        if (err == cudaSuccess) err = cudaMemcpy(L->d_xslot, &xs, sizeof(BsSlot), cudaMemcpyHostToDevice);
    }
    if (err == cudaSuccess)
        err = cudaMemcpy(L->d_tables, tables.data(), tables.size() * sizeof(void *), cudaMemcpyHostToDevice);
    if (err == cudaSuccess) err = cudaMemcpy(L->d_bias, bias, experts * 4, cudaMemcpyDefault);
    if (err == cudaSuccess) err = cudaStreamSynchronize(ctx->stream);  // router64 is ready
    if (err != cudaSuccess) {
        urb_moe_layer_free(L);
        return cuda_fail(ctx, err, "layer tables");
    }
    *out = L;
    return URB_OK;
}

int urb_moe_layer_create(urb_ctx *ctx, const urb_mat *router, const float *bias, size_t experts,
                         const urb_mat *const *gate, const urb_mat *const *up,
                         const urb_mat *const *down, const urb_mat *sg, const urb_mat *su,
                         const urb_mat *sd, const urb_moe_geometry *geo, urb_layer **out) {
    return create_layer(ctx, router, bias, experts, 0, experts, gate, up, down, sg, su, sd, geo, out);
}

int urb_moe_layer_create_sharded(urb_ctx *ctx, const urb_mat *router, const float *bias,
                                 size_t experts, size_t expert_begin, size_t expert_count,
                                 const urb_mat *const *gate, const urb_mat *const *up,
                                 const urb_mat *const *down, const urb_mat *sg, const urb_mat *su,
                                 const urb_mat *sd, const urb_moe_geometry *geo, urb_layer **out) {
    return create_layer(ctx, router, bias, experts, expert_begin, expert_count, gate, up, down,
                        sg, su, sd, geo, out);
}

int urb_moe_layer_free(urb_layer *L) {
    if (!L) return URB_ERR_INVALID_ARGUMENT;
    if (L->ctx) {
        cudaSetDevice(L->ctx->device);
        cudaStreamSynchronize(L->ctx->stream);
    }
    if (L->d_tables) cudaFree(L->d_tables);
    if (L->router64) cudaFree(L->router64);
    if (L->d_bias) cudaFree(L->d_bias);
    if (L->d_xslot) cudaFree(L->d_xslot);
    delete L;
    return URB_OK;
}

int urb_moe_forward_device(urb_ctx *ctx, urb_layer *L, const float *d_x, size_t tokens,
                           float *d_out, int32_t *d_route_expert, float *d_route_weight,
                           int32_t *d_status) {
    if (!ctx || !L || !d_x || !d_out) return URB_ERR_INVALID_ARGUMENT;
    if (L->e_count != L->experts)
        return set_error(ctx, URB_ERR_UNSUPPORTED, "an expert shard runs through urb_ep_forward");
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    cudaSetDevice(ctx->device);
    if (tokens == 0) return URB_OK;
    MoeWork w{};
    int rc = moe_forward_device(L, d_x, int(tokens), d_out, &w, d_status, ctx->stream);
    if (rc) return rc;
    size_t TK = tokens * L->geo.top_k;
    if (d_route_expert)
        URB_CUDA(ctx, cudaMemcpyAsync(d_route_expert, w.ids, TK * 4, cudaMemcpyDeviceToDevice, ctx->stream));
    if (d_route_weight)
        URB_CUDA(ctx, cudaMemcpyAsync(d_route_weight, w.w, TK * 4, cudaMemcpyDeviceToDevice, ctx->stream));
    return URB_OK;
}

int urb_moe_forward(urb_ctx *ctx, urb_layer *L, const float *x, size_t tokens, float *out,
                    int32_t *route_expert, float *route_weight, float *route_score,
                    float *router_logits, int32_t *counts, int32_t *perm_token,
                    int32_t *perm_slot) {
    if (!ctx || !L || !x || !out) return URB_ERR_INVALID_ARGUMENT;
    if (L->e_count != L->experts)
        return set_error(ctx, URB_ERR_UNSUPPORTED, "an expert shard runs through urb_ep_forward");
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    cudaSetDevice(ctx->device);
    if (tokens == 0) return URB_OK;
    cudaStream_t st = ctx->stream;
    const size_t H = L->hidden, TK = tokens * L->geo.top_k, E = L->experts;
    int io_rc;
    float *d_io = static_cast<float *>(io_buffer(ctx, 2 * tokens * H * 4, &io_rc));
    if (!d_io) return io_rc;
    float *d_x = d_io, *d_out = d_io + tokens * H;
    URB_CUDA(ctx, cudaMemsetAsync(ctx->d_status, 0, 4, st));
    URB_CUDA(ctx, cudaMemcpyAsync(d_x, x, tokens * H * 4, cudaMemcpyDefault, st));
    if (L->generic) {
        int rc = moe_forward_generic(L, d_x, int(tokens), d_out, route_expert, route_weight,
                                     route_score, router_logits, counts, perm_token, perm_slot,
                                     ctx->d_status, st);
        if (rc == URB_OK) rc = [&] {
            URB_CUDA(ctx, cudaMemcpyAsync(out, d_out, tokens * H * 4, cudaMemcpyDefault, st));
            URB_CUDA(ctx, cudaStreamSynchronize(st));
            return int(URB_OK);
        }();
        cudaStreamSynchronize(st);
        return rc;
    }
    MoeWork w{};
    int rc = moe_forward_device(L, d_x, int(tokens), d_out, &w, ctx->d_status, st);
    if (rc) return rc;
    int32_t status = 0;
    URB_CUDA(ctx, cudaMemcpyAsync(out, d_out, tokens * H * 4, cudaMemcpyDefault, st));
    if (route_expert) URB_CUDA(ctx, cudaMemcpyAsync(route_expert, w.ids, TK * 4, cudaMemcpyDefault, st));
    if (route_weight) URB_CUDA(ctx, cudaMemcpyAsync(route_weight, w.w, TK * 4, cudaMemcpyDefault, st));
    if (route_score) URB_CUDA(ctx, cudaMemcpyAsync(route_score, w.score, TK * 4, cudaMemcpyDefault, st));
    if (router_logits) URB_CUDA(ctx, cudaMemcpyAsync(router_logits, w.logits, tokens * E * 4, cudaMemcpyDefault, st));
    if (counts) URB_CUDA(ctx, cudaMemcpyAsync(counts, w.counts, E * 4, cudaMemcpyDefault, st));
    if (perm_token) URB_CUDA(ctx, cudaMemcpyAsync(perm_token, w.perm_token, TK * 4, cudaMemcpyDefault, st));
    if (perm_slot) URB_CUDA(ctx, cudaMemcpyAsync(perm_slot, w.perm_slot, TK * 4, cudaMemcpyDefault, st));
    URB_CUDA(ctx, cudaMemcpyAsync(&status, ctx->d_status, 4, cudaMemcpyDeviceToHost, st));
    URB_CUDA(ctx, cudaStreamSynchronize(st));
    if (status) return set_error(ctx, status, "MoE forward rejected its input");
    return URB_OK;
}

static int numerics_of(urb_ctx *ctx, const urb_moe_numerics *n, Numerics *out) {
    if (!n) return URB_OK;
    if (n->mode == URB_NUMERICS_GLM) return URB_OK;
    if (n->mode == URB_NUMERICS_QWEN36) {
        out->mode = n->mode;
        return URB_OK;
    }
    if (n->mode != URB_NUMERICS_DEEPSEEK_V4)
        return set_error(ctx, URB_ERR_INVALID_ARGUMENT, "unknown numerics mode");
    // validate_positive("SwiGLU limit") of deepseek_v4/math.rs:531.
    if (!std::isfinite(n->swiglu_limit) || n->swiglu_limit <= 0.0f)
        return set_error(ctx, URB_ERR_INVALID_ARGUMENT, "SwiGLU limit must be finite and positive");
    out->mode = n->mode;
    out->limit = n->swiglu_limit;
    return URB_OK;
}

int urb_moe_forward_routed_ex_device(urb_ctx *ctx, urb_layer *L, const float *d_x,
                                     size_t tokens, const int32_t *d_route_expert,
                                     const float *d_route_weight, const urb_moe_numerics *numerics,
                                     float *d_out, int32_t *d_status) {
    if (!ctx || !L || !d_x || !d_out || !d_route_expert || !d_route_weight)
        return URB_ERR_INVALID_ARGUMENT;
    if (L->e_count != L->experts)
        return set_error(ctx, URB_ERR_UNSUPPORTED, "an expert shard runs through urb_ep_forward");
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    cudaSetDevice(ctx->device);
    Numerics num;
    int rc = numerics_of(ctx, numerics, &num);
    if (rc) return rc;
    if (tokens == 0) return URB_OK;
    return moe_forward_device(L, d_x, int(tokens), d_out, nullptr, d_status, ctx->stream,
                              d_route_expert, d_route_weight, &num);
}

int urb_moe_forward_routed_device(urb_ctx *ctx, urb_layer *L, const float *d_x, size_t tokens,
                                  const int32_t *d_route_expert, const float *d_route_weight,
                                  float *d_out, int32_t *d_status) {
    if (!ctx || !L || !d_x || !d_out || !d_route_expert || !d_route_weight)
        return URB_ERR_INVALID_ARGUMENT;
    if (L->e_count != L->experts)
        return set_error(ctx, URB_ERR_UNSUPPORTED, "an expert shard runs through urb_ep_forward");
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    cudaSetDevice(ctx->device);
    if (tokens == 0) return URB_OK;
    return moe_forward_device(L, d_x, int(tokens), d_out, nullptr, d_status, ctx->stream,
                              d_route_expert, d_route_weight);
}

int urb_moe_forward_routed_ex(urb_ctx *ctx, urb_layer *L, const float *x, size_t tokens,
                              const int32_t *route_expert, const float *route_weight,
                              const urb_moe_numerics *numerics, float *out) {
    if (!ctx || !L || !x || !out || !route_expert || !route_weight) return URB_ERR_INVALID_ARGUMENT;
    if (L->e_count != L->experts)
        return set_error(ctx, URB_ERR_UNSUPPORTED, "an expert shard runs through urb_ep_forward");
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    cudaSetDevice(ctx->device);
    Numerics num;
    int rc0 = numerics_of(ctx, numerics, &num);
    if (rc0) return rc0;
    if (tokens == 0) return URB_OK;
    const size_t H = L->hidden, K = L->geo.top_k, TK = tokens * K;
    for (size_t i = 0; i < TK; ++i)
        if (route_expert[i] < 0 || size_t(route_expert[i]) >= L->experts)
            return set_error(ctx, URB_ERR_SHAPE, "route expert id out of range");
    if (num.mode == URB_NUMERICS_DEEPSEEK_V4)
        for (size_t i = 0; i < TK; ++i)  // deepseek_v4/runtime.rs:3091-3095
            if (!std::isfinite(route_weight[i]) || route_weight[i] < 0.0f)
                return set_error(ctx, URB_ERR_INVALID_ARGUMENT,
                                 "routed expert weight must be finite and non-negative");
    cudaStream_t st = ctx->stream;
    const size_t bytes = 2 * tokens * H * 4 + 2 * TK * 4;
    int io_rc;
    uint8_t *d_io = static_cast<uint8_t *>(io_buffer(ctx, bytes, &io_rc));
    if (!d_io) return io_rc;
    float *d_x = reinterpret_cast<float *>(d_io), *d_out = d_x + tokens * H;
    int32_t *d_ids = reinterpret_cast<int32_t *>(d_out + tokens * H);
    float *d_w = reinterpret_cast<float *>(d_ids + TK);
    URB_CUDA(ctx, cudaMemsetAsync(ctx->d_status, 0, 4, st));
    URB_CUDA(ctx, cudaMemcpyAsync(d_x, x, tokens * H * 4, cudaMemcpyDefault, st));
    URB_CUDA(ctx, cudaMemcpyAsync(d_ids, route_expert, TK * 4, cudaMemcpyDefault, st));
    URB_CUDA(ctx, cudaMemcpyAsync(d_w, route_weight, TK * 4, cudaMemcpyDefault, st));
    int rc = moe_forward_device(L, d_x, int(tokens), d_out, nullptr, ctx->d_status, st, d_ids, d_w,
                                &num);
    if (rc) return rc;
    int32_t status = 0;
    URB_CUDA(ctx, cudaMemcpyAsync(out, d_out, tokens * H * 4, cudaMemcpyDefault, st));
    URB_CUDA(ctx, cudaMemcpyAsync(&status, ctx->d_status, 4, cudaMemcpyDeviceToHost, st));
    URB_CUDA(ctx, cudaStreamSynchronize(st));
    if (status) return set_error(ctx, status, "MoE forward rejected its input");
    return URB_OK;
}

int urb_moe_forward_ex(urb_ctx *ctx, urb_layer *L, const float *x, size_t tokens,
                       const urb_moe_numerics *numerics, const int32_t *hash_experts, float *out,
                       int32_t *route_expert, float *route_weight) {
    if (!ctx || !L || !x || !out) return URB_ERR_INVALID_ARGUMENT;
    Numerics num;
    {
        std::lock_guard<std::recursive_mutex> lk(ctx->mu);
        int rc = numerics_of(ctx, numerics, &num);
        if (rc) return rc;
    }
    if (num.mode == URB_NUMERICS_GLM) {
        if (hash_experts)
            return set_error(ctx, URB_ERR_INVALID_ARGUMENT, "hash routing needs the DeepSeek-V4 numerics");
        return urb_moe_forward(ctx, L, x, tokens, out, route_expert, route_weight, nullptr,
                               nullptr, nullptr, nullptr, nullptr);
    }
    if (L->e_count != L->experts)
        return set_error(ctx, URB_ERR_UNSUPPORTED, "an expert shard runs through urb_ep_forward");
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    cudaSetDevice(ctx->device);
    const bool qwen = num.mode == URB_NUMERICS_QWEN36;
    if (qwen) {
        if (hash_experts)
            return set_error(ctx, URB_ERR_INVALID_ARGUMENT, "hash routing needs the DeepSeek-V4 numerics");
        if (L->router->format != URB_FMT_BF16 || !L->router->raw_values)
            return set_error(ctx, URB_ERR_UNSUPPORTED, "Qwen3.6 numerics need a BF16 router");
        if (!L->sg || !L->shared_gate_row)
            return set_error(ctx, URB_ERR_UNSUPPORTED,
                             "Qwen3.6 numerics need a shared expert and its gate");
    }
    if (tokens == 0) return URB_OK;
    const size_t H = L->hidden, K = L->geo.top_k, E = L->experts, TK = tokens * K;
    if (hash_experts)
        for (size_t i = 0; i < TK; ++i)
            if (hash_experts[i] < 0 || size_t(hash_experts[i]) >= E)
                return set_error(ctx, URB_ERR_INVALID_ARGUMENT, "hash expert IDs must be in range");
    // MoeWeights::forward for DeepSeek-V4 (deepseek_v4/runtime.rs:2484-2700): exact router
    // logits, route_sqrt_softplus with the layer's correction bias (or the token's hash experts),
    // then the routed experts with the checkpoint numerics.
    cudaStream_t st = ctx->stream;
    auto align = [](size_t b) { return (b + 255) & ~size_t(255); };
    const size_t o_x = 0, o_out = align(o_x + tokens * H * 4), o_l = align(o_out + tokens * H * 4);
    const size_t o_x64 = align(o_l + tokens * E * 4);
    const size_t o_ids = align(o_x64 + router_f64_elems(int(tokens), int(H)) * 8);
    const size_t o_w = align(o_ids + TK * 4), o_s = align(o_w + TK * 4), o_h = align(o_s + TK * 4);
    const size_t o_g = align(o_h + TK * 4);
    const size_t bytes = align(o_g + tokens * 4);
    int io_rc;
    uint8_t *d = static_cast<uint8_t *>(io_buffer(ctx, bytes, &io_rc));
    if (!d) return io_rc;
    float *d_x = reinterpret_cast<float *>(d + o_x), *d_out = reinterpret_cast<float *>(d + o_out);
    float *d_l = reinterpret_cast<float *>(d + o_l);
    double *d_x64 = reinterpret_cast<double *>(d + o_x64);
    int32_t *d_ids = reinterpret_cast<int32_t *>(d + o_ids), *d_hash = reinterpret_cast<int32_t *>(d + o_h);
    float *d_w = reinterpret_cast<float *>(d + o_w), *d_s = reinterpret_cast<float *>(d + o_s);
    URB_CUDA(ctx, cudaMemsetAsync(ctx->d_status, 0, 4, st));
    URB_CUDA(ctx, cudaMemcpyAsync(d_x, x, tokens * H * 4, cudaMemcpyDefault, st));
    if (hash_experts) URB_CUDA(ctx, cudaMemcpyAsync(d_hash, hash_experts, TK * 4, cudaMemcpyDefault, st));
    int rc;
    if (qwen) {
        // execute_batched_moe (qwen3_6/runtime.rs:1067-1090): BF16 router and shared-expert gate
        // logits in one launch, route_softmax_top_k with BF16 weights.
        float *d_g = reinterpret_cast<float *>(d + o_g);
        prof_begin(ctx, URB_K_ROUTER_LOGITS, st);
        rc = launch_router_bf16_lanes(static_cast<const uint16_t *>(L->router->raw_values), int(E),
                                      static_cast<const uint16_t *>(L->shared_gate_row->raw_values),
                                      d_x, int(tokens), int(H), d_l, d_g, ctx->d_status, st);
        prof_end(ctx, st);
        if (rc) { return cuda_fail(ctx, cudaGetLastError(), "router logits"); }
        prof_begin(ctx, URB_K_ROUTE, st);
        rc = launch_route_softmax(ctx, d_l, int(tokens), int(E), int(K), d_ids, d_w, ctx->d_status,
                                  st, 1);
        prof_end(ctx, st);
        num.gate_logit = d_g;
    } else {
        const RouterGates rg{ctx, nullptr, nullptr, nullptr, ctx->d_status};
        prof_begin(ctx, URB_K_ROUTER_LOGITS, st);
        rc = launch_router_logits_f64(L->router64, int(E), d_x, int(tokens), int(H), d_x64, d_l, st, &rg);
        prof_end(ctx, st);
        if (rc) { return cuda_fail(ctx, cudaGetLastError(), "router logits"); }
        prof_begin(ctx, URB_K_ROUTE, st);
        rc = launch_route_sqrt_softplus(ctx, d_l, L->d_bias, hash_experts ? d_hash : nullptr,
                                        int(tokens), int(E), int(K), L->geo.routed_scaling_factor,
                                        d_ids, d_w, d_s, ctx->d_status, st);
        prof_end(ctx, st);
    }
    if (rc == URB_OK)
        rc = moe_forward_device(L, d_x, int(tokens), d_out, nullptr, ctx->d_status, st, d_ids,
                                d_w, &num);
    if (rc) return rc;
    int32_t status = 0;
    URB_CUDA(ctx, cudaMemcpyAsync(out, d_out, tokens * H * 4, cudaMemcpyDefault, st));
    if (route_expert) URB_CUDA(ctx, cudaMemcpyAsync(route_expert, d_ids, TK * 4, cudaMemcpyDefault, st));
    if (route_weight) URB_CUDA(ctx, cudaMemcpyAsync(route_weight, d_w, TK * 4, cudaMemcpyDefault, st));
    URB_CUDA(ctx, cudaMemcpyAsync(&status, ctx->d_status, 4, cudaMemcpyDeviceToHost, st));
    URB_CUDA(ctx, cudaStreamSynchronize(st));
    if (status) return set_error(ctx, status, "MoE forward rejected its input");
    return URB_OK;
}

int urb_moe_forward_routed(urb_ctx *ctx, urb_layer *L, const float *x, size_t tokens,
                           const int32_t *route_expert, const float *route_weight, float *out) {
    return urb_moe_forward_routed_ex(ctx, L, x, tokens, route_expert, route_weight, nullptr, out);
}

int urb_moe_layer_set_shared_expert_gate(urb_ctx *ctx, urb_layer *L, const urb_mat *gate) {
    if (!ctx || !L) return URB_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    if (gate && (gate->rows != 1 || gate->cols != L->hidden))
        return set_error(ctx, URB_ERR_SHAPE, "shared expert gate must be [1, hidden]");
    if (gate && (gate->format != URB_FMT_BF16 || !gate->raw_values))
        return set_error(ctx, URB_ERR_UNSUPPORTED, "shared expert gate must be a BF16 matrix");
    L->shared_gate_row = gate;
    return URB_OK;
}

int urb_gated_mlp_forward(urb_ctx *ctx, const urb_mat *g, const urb_mat *u, const urb_mat *d,
                          const float *x, size_t tokens, float *out) {
    if (!ctx || !g || !u || !d || !x || !out) return URB_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    cudaSetDevice(ctx->device);
    // GatedMlp::new_mixed (src/model/mlp.rs:60-81).
    if (g->rows != u->rows || g->cols != u->cols || d->cols != g->rows || d->rows != g->cols)
        return set_error(ctx, URB_ERR_SHAPE, "gated MLP projections have inconsistent shapes");
    if (tokens == 0) return URB_OK;
    for (size_t i = 0; i < tokens * g->cols; ++i)
        if (!std::isfinite(x[i])) return set_error(ctx, URB_ERR_NONFINITE, "gated MLP input is not finite");
    cudaStream_t st = ctx->stream;
    const size_t H = g->cols;
    int io_rc;
    float *d_io = static_cast<float *>(io_buffer(ctx, 2 * tokens * H * 4, &io_rc));
    if (!d_io) return io_rc;
    URB_CUDA(ctx, cudaMemcpyAsync(d_io, x, tokens * H * 4, cudaMemcpyDefault, st));
    int rc = gated_mlp_device(ctx, g, u, d, d_io, int(tokens), d_io + tokens * H, nullptr, st);
    if (rc == URB_OK)
        URB_CUDA(ctx, cudaMemcpyAsync(out, d_io + tokens * H, tokens * H * 4, cudaMemcpyDefault, st));
    URB_CUDA(ctx, cudaStreamSynchronize(st));
    return rc;
}

int urb_gated_mlp_forward_device(urb_ctx *ctx, const urb_mat *g, const urb_mat *u,
                                 const urb_mat *d, const float *d_x, size_t tokens, float *d_out,
                                 int32_t *d_status) {
    if (!ctx || !g || !u || !d || !d_x || !d_out) return URB_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    cudaSetDevice(ctx->device);
    if (g->rows != u->rows || g->cols != u->cols || d->cols != g->rows || d->rows != g->cols)
        return set_error(ctx, URB_ERR_SHAPE, "gated MLP projections have inconsistent shapes");
    if (tokens == 0) return URB_OK;
    return gated_mlp_device(ctx, g, u, d, d_x, int(tokens), d_out, d_status, ctx->stream);
}

}  // extern "C"
