// urb_moe_internal.cuh — MoE-layer structures shared by moe.cu and api.cu.
#pragma once
#include "urb_internal.cuh"
#include "urb_tc.cuh"

namespace urb {

// Inputs/outputs of the single-CTA grouping kernel.
struct PermArgs {
    const int32_t *ids;  // [tokens, top_k] expert ids in selection order
    int tokens, top_k, experts, cap;
    int32_t *counts;      // [experts] or nullptr
    int32_t *offsets;     // [experts+1] or nullptr
    int32_t *perm_token;  // [tokens*top_k] grouped order: token of each route
    int32_t *perm_slot;   // [tokens*top_k] grouped order: selection rank of each route
    int32_t *inv;         // [tokens*top_k] (token, rank) -> grouped position
    Seg *segs_gu, *segs_dn;
    int *nsegs_gu, *total_rows_gu, *nsegs_dn, *total_rows_dn;
    int32_t *col_src;     // [tokens*top_k + tokens] gate/up activation column -> x row
    int32_t *maxexp;      // [tokens*top_k + tokens] reset to -1000
    const uint8_t *const *gate_tiles, *const *up_tiles, *const *down_tiles;
    const int8_t *const *gate_rexp, *const *up_rexp, *const *down_rexp;
    const uint8_t *sh_gate_tiles, *sh_up_tiles, *sh_down_tiles;
    const int8_t *sh_gate_rexp, *sh_up_rexp, *sh_down_rexp;
    int shared_in_pass;
    int hidden, inter, gu_rbs, gu_kslices, dn_rbs, dn_kslices;
    int32_t *status;
    const int *lofree;    // optional: when *lofree, segments hold 2*cap tokens
    int allow_foreign;    // ids == -1 are routes held by another rank: not grouped, inv = -1
    int32_t *route_of;    // optional [tokens*top_k]: route index of each grouped position
    const float *route_w; // optional [tokens*top_k] route weights, with col_w:
    float *col_w;         // [tokens*top_k + tokens] weight of each activation column (shared: 1)
};

int launch_permute(Ctx *ctx, const PermArgs &p, cudaStream_t st);

// Groups of the two tensor-core passes, built on the device from the grouping.
struct TcBuildArgs {
    const int32_t *counts, *offsets;  // from the grouping kernel
    int fmt;
    int tokens, top_k, experts;
    const uint8_t *const *gate_tc, *const *up_tc, *const *down_tc;
    const uint8_t *sh_gate_tc, *sh_up_tc, *sh_down_tc;
    int has_shared, shared_tokens;  // shared-expert columns [tokens*top_k, +shared_tokens)
    int pair_down;  // down-pass units pair neighbouring row tiles (TcArgs::pair == 2)
    // One token: every gate/up group reads the one activation-stage set at offset 0 (slot 0),
    // written by a prep that needs no routing.
    int shared_x;
    int hidden, inter;
    TcSeg *gu, *dn;
    BsSlot *gu_slots, *dn_slots;  // [TK + T] activation slots of each column, per pass
    int *gu_units, *dn_units;     // group of each work unit, per pass
    int *scalars;  // ngroups_gu, units_gu, ngroups_dn, units_dn
    const int32_t *status;  // non-zero: an earlier stage failed; build no work
};
int launch_build_tc_segs(Ctx *ctx, const TcBuildArgs &b, cudaStream_t st);
// Decode (1..32 tokens): route_noaux_tc over the router epilogue's gates (rg), the grouping
// `p` (whose ids are d_expert) and the tensor-core tables `b`, in one single-CTA launch.
int launch_decode_group(Ctx *ctx, const RouterGates &rg, int tokens, int experts, const urb_moe_geometry &g,
                        int32_t *d_expert, float *d_weight, float *d_score, const PermArgs &p,
                        const TcBuildArgs &b, cudaStream_t st);
int launch_combine(Ctx *ctx, const float *y, const float *shared_y, const float *w,
                   const int32_t *inv, int tokens, int top_k, int hidden, float *out,
                   cudaStream_t st, const int32_t *status = nullptr);
// DeepSeek-V4 combine (deepseek_v4/runtime.rs:2500-2650): per token, f32 sum of the routed rows
// (route weights already applied) in ascending expert id, plus the shared row, cast to BF16.
int launch_combine_deepseek(Ctx *ctx, const float *y, const float *shared_y, const int32_t *ids,
                            const int32_t *inv, int tokens, int top_k, int hidden, float *out,
                            cudaStream_t st, int32_t *status);
// Qwen3.6 MoE output (qwen3_6/runtime.rs:1123-1213): expert-id-order BF16 accumulation of
// BF16(BF16(w) * y), then the shared expert scaled by BF16(sigmoid(gate_logit[t])).
int launch_combine_qwen(Ctx *ctx, const float *y, const float *shared_y, const int32_t *ids,
                        const float *w, const int32_t *inv, const float *gate_logit, int tokens,
                        int top_k, int hidden, float *out, cudaStream_t st, int32_t *status);
// Checkpoint numerics of a forward (urb_moe_numerics).
struct Numerics {
    int mode = 0;        // URB_NUMERICS_*
    float limit = 0.0f;  // bounded-SwiGLU limit (DeepSeek-V4)
    const float *gate_logit = nullptr;  // Qwen3.6: [T] BF16 shared-expert gate logits (device)
};

struct Layer {
    Ctx *ctx = nullptr;
    const Mat *router = nullptr;
    double *router64 = nullptr;  // router widened to f64, blocked (the logits' FP64 MMA operand)
    float *d_bias = nullptr;
    size_t experts = 0, hidden = 0, inter = 0;  // experts: routed experts in total (router rows)
    // Routed experts held by this layer: [e_begin, e_begin + e_count) (all of them unless the
    // layer is one expert-parallel shard).
    size_t e_begin = 0, e_count = 0;
    int fmt = 0;
    std::vector<const Mat *> gate, up, down;
    BsSlot *d_xslot = nullptr;  // the one-token gate/up activation slot {0, 0, 16} (device)
    const Mat *sg = nullptr, *su = nullptr, *sd = nullptr;
    // Qwen3.6 shared_expert_gate: a [1, hidden] BF16 row (urb_moe_layer_set_shared_expert_gate).
    const Mat *shared_gate_row = nullptr;
    urb_moe_geometry geo{};
    // Device pointer tables, 9 kinds of (e_count + 1) entries (held experts, then the shared
    // expert or null): gate/up/down mma tiles, their row exponents, gate/up/down bs tiles.
    void **d_tables = nullptr;
    bool use_tc = true;  // block-scaled tcgen05 passes (false: mma.sync register-dequant)
    // Experts without one shared tiled format (INT8 / INT4 GLM experts, F32, mixed formats):
    // the forward composes per-expert GatedMlp calls (moe_forward_generic).
    bool generic = false;
};

// Device workspace of one forward, carved from the context workspace.
struct MoeWork {
    int32_t *shift;       // [T]
    float *logits;        // [T, E]
    float *gate, *sel;    // [T, E] sigmoid gates and biased selection scores
    double *x64;          // x widened to f64 in the router's blocked layout
    int32_t *ids;         // [T, K]
    float *w, *score;     // [T, K]
    int32_t *counts, *offsets, *perm_token, *perm_slot, *inv;
    Seg *segs_gu, *segs_dn;
    int *scalars;         // nsegs_gu, total_rows_gu, nsegs_dn, total_rows_dn
    int32_t *col_src, *maxexp;
    float *h;             // [TK+T, inter]
    float *y;             // [TK+T, hidden]
    int32_t *status;
    int32_t *lofree;
    float *gu;            // [TK+T, 2*inter] gate | up outputs of the tensor-core pass
    TcSeg *tsegs_gu, *tsegs_dn;
    BsSlot *bslots_gu, *bslots_dn;
    int *units_gu, *units_dn;
    int *tscalars;
    uint8_t *bbuf_gu, *bbuf_dn;
    float *col_w;         // [TK+T] route weight of each activation column (DeepSeek-V4 numerics)
};

// d_ids_in / d_w_in ([tokens, top_k], optional): routes chosen by the caller; the router is
// skipped and these are grouped and combined instead.
int moe_forward_device(Layer *L, const float *d_x, int tokens, float *d_out, MoeWork *work_out,
                       int32_t *d_status, cudaStream_t st, const int32_t *d_ids_in = nullptr,
                       const float *d_w_in = nullptr, const Numerics *num = nullptr);
// Exact router logits and route_noaux_tc of `tokens` rows into w.logits / x64 / gate / sel /
// ids / w / score.
int route_device(Layer *L, const float *d_x, int tokens, const MoeWork &w, int32_t *d_status,
                 cudaStream_t st);
// Bounds of the tensor-core passes' work tables (units of a pass over `mts` row tiles, bytes of
// its activation stages over `ks` K stages) for tokens * top_k routes over `experts` experts
// plus `tokens` shared-expert columns.
size_t max_bs_units(int fmt, size_t tokens, size_t top_k, size_t experts, size_t mts);
size_t max_bs_bytes(int fmt, size_t tokens, size_t top_k, size_t experts, size_t ks);

}  // namespace urb

struct urb_layer : urb::Layer {};
