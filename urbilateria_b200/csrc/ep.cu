// ep.cu — expert-parallel MoE layer over the GPUs of one node, one process per GPU.
//
// The layer forward of glm/runtime/moe.rs:138-176 split by experts: rank g holds routed experts
// [e_begin, e_begin + e_count) (its sharded urb_layer) plus the replicated router and shared
// expert, and owns the tokens it is given.  The exchange runs over peer memory through
// NVLink / NVSwitch, inside the compute kernels, with no collective library call:
//
//   route (own tokens)  ->  publish ids + x in this rank's window  ->  barrier
//   -> gather every rank's routes to the held experts (peer loads of ids)
//   -> grouping -> gate/up prep reads each token row from its owner's window (peer loads)
//   -> grouped gate/up -> grouped down, whose epilogue stores each routed output row straight
//      into the owning rank's window (peer stores)  ->  barrier
//   -> combine of the own tokens in selection order (f64), from the own window.
//
// Results are bit-identical to the single-GPU layer: every expert output row is the same
// computation on the same inputs, and the owner combines its routes in the reference order.
//
// Windows are cudaMalloc'd and shared by CUDA IPC (urb_ep_export / urb_ep_connect); the
// handles travel through the caller's host-side process group.  Barriers are flag words in
// the windows (release / acquire at system scope), each wait bounded by a timeout after which
// the kernel records URB_ERR_TIMEOUT and returns.  A rank's failure (its device status) rides
// on its barrier word, so every rank of the group fails the same forward (URB_ERR_PEER).
//
// Ranks wait on one another, so they must run on distinct GPUs: urb_ep_connect refuses a group
// in which two ranks share a device.
#include <cstring>
#include <vector>

#include "urb_internal.cuh"
#include "urb_moe_internal.cuh"

namespace urb {
namespace {

constexpr int kEpMaxWorld = URB_EP_MAX_WORLD;
constexpr uint64_t kEpMagic = 0x3170455f4252554fULL;

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }
size_t ceil_div(size_t a, size_t b) { return (a + b - 1) / b; }

// Byte offsets inside one rank's window.
struct EpLayout {
    size_t sig;   // [2][kEpMaxWorld] uint64 barrier words (by parity, then writer rank)
    size_t ntok;  // int32 tokens published for the current forward
    size_t ids;   // [tmax * K] int32 routed experts of the published tokens (selection order)
    size_t x;     // [tmax * H] f32 activations of the published tokens
    size_t y;     // [tmax * K * H] f32 routed expert outputs of the published tokens, by route
    size_t bytes;
};

EpLayout make_layout(size_t tmax, size_t K, size_t H) {
    EpLayout l{};
    size_t o = 0;
    l.sig = o; o = align256(o + 2 * kEpMaxWorld * sizeof(uint64_t));
    l.ntok = o; o = align256(o + sizeof(int32_t));
    l.ids = o; o = align256(o + tmax * K * sizeof(int32_t));
    l.x = o; o = align256(o + tmax * H * sizeof(float));
    l.y = o; o = align256(o + tmax * K * H * sizeof(float));
    l.bytes = o;
    return l;
}

// Handle blob exchanged between ranks (URB_EP_HANDLE_BYTES).
struct EpBlob {
    cudaIpcMemHandle_t ipc;
    char pci[32];
    uint64_t magic;
    int64_t world, rank, tmax, hidden, top_k, experts, e_begin, e_count, bytes;
};
static_assert(sizeof(EpBlob) <= URB_EP_HANDLE_BYTES, "handle blob");

struct EpPeers {
    uint8_t *win[kEpMaxWorld];
};

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void st_release_sys(uint64_t *p, uint64_t v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t *p) {
    uint64_t v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Group barrier of one forward step.  Thread i < world posts (epoch, own status) into rank i's
// window, then waits for rank i's post of this epoch in the own window.  Barriers alternate
// between two word sets by epoch parity; a rank cannot post epoch e + 2 before every rank has
// passed epoch e + 1, so the word read for epoch e holds epoch e.  A wait that exceeds
// timeout_ns records URB_ERR_TIMEOUT; a peer's non-zero status becomes URB_ERR_PEER here.
__global__ void k_ep_barrier(EpPeers P, size_t sig_off, int world, int rank, uint32_t epoch,
                             int32_t *status, unsigned long long timeout_ns) {
    const int i = threadIdx.x;
    if (i >= world) return;
    const int32_t mine = *status;
    const int parity = int(epoch & 1u);
    __threadfence_system();  // this rank's earlier writes (own window and peers') come first
    uint64_t *dst = reinterpret_cast<uint64_t *>(P.win[i] + sig_off) + parity * kEpMaxWorld + rank;
    st_release_sys(dst, (uint64_t(epoch) << 32) | uint32_t(mine));
    const uint64_t *src = reinterpret_cast<const uint64_t *>(P.win[rank] + sig_off) + parity * kEpMaxWorld + i;
    const uint64_t t0 = globaltimer_ns();
    uint64_t v = 0;
    bool ok = false;
    for (uint32_t it = 0;; ++it) {
        v = ld_acquire_sys(src);
        if (int32_t(uint32_t(v >> 32) - epoch) >= 0) { ok = true; break; }
        if ((it & 63u) == 63u && globaltimer_ns() - t0 > timeout_ns) break;
        __nanosleep(128);
    }
    if (!ok) {
        atomicCAS(status, 0, int32_t(URB_ERR_TIMEOUT));
    } else if (int32_t(uint32_t(v)) != 0 && i != rank) {
        atomicCAS(status, 0, int32_t(URB_ERR_PEER));
    }
}

// Publishes this rank's routes and token count (x is copied by the caller).
__global__ void k_ep_publish(const int32_t *ids, int n_ids, int tokens, int32_t *win_ids,
                             int32_t *win_ntok) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n_ids) win_ids[i] = ids[i];
    if (i == 0) *win_ntok = tokens;
}

// Routes of every rank's published tokens to the experts held here: lids[(q * tmax + t) * K + k]
// = local expert index, or -1 for a route held elsewhere and for rows past rank q's tokens.
__global__ void k_ep_gather(EpPeers P, size_t ntok_off, size_t ids_off, int world, int tmax,
                            int K, int e_begin, int e_count, int32_t *lids, const int32_t *status) {
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    const int per_rank = tmax * K;
    if (idx >= world * per_rank) return;
    const int q = idx / per_rank, j = idx - q * per_rank, t = j / K;
    int lid = -1;
    if (!*status) {
        const int ntok = __ldcv(reinterpret_cast<const int32_t *>(P.win[q] + ntok_off));
        if (t < ntok) {
            const int e = __ldcv(reinterpret_cast<const int32_t *>(P.win[q] + ids_off) + j);
            if (e >= e_begin && e < e_begin + e_count) lid = e - e_begin;
        }
    }
    lids[idx] = lid;
}

}  // namespace

struct Ep {
    Ctx *ctx = nullptr;
    Layer *L = nullptr;
    int world = 1, rank = 0;
    size_t tmax = 0;
    EpLayout lay{};
    uint8_t *win = nullptr;              // own window
    uint8_t *peer[kEpMaxWorld] = {};     // every rank's window as mapped here (own included)
    bool opened[kEpMaxWorld] = {};       // peer[] entries opened through CUDA IPC
    bool connected = false;
    const float **d_x_ranks = nullptr;   // [world] x of each rank's window
    float **d_y_ranks = nullptr;         // [world] y of each rank's window
    uint32_t epoch = 0;
    unsigned long long timeout_ns = 0;
    float *d_io = nullptr;               // host-pointer forward: x and out [tmax, H]
    int32_t *d_routes = nullptr;         // host-pointer forward: ids [tmax, K]
    float *d_rw = nullptr;               // host-pointer forward: weights [tmax, K]
};

namespace {

int barrier(Ep *ep, int32_t *status, cudaStream_t st) {
    EpPeers P{};
    for (int i = 0; i < ep->world; ++i) P.win[i] = ep->peer[i];
    ++ep->epoch;
    k_ep_barrier<<<1, 32, 0, st>>>(P, ep->lay.sig, ep->world, ep->rank, ep->epoch, status,
                                   ep->timeout_ns);
    URB_CUDA(ep->ctx, cudaGetLastError());
    return URB_OK;
}

}  // namespace

// One expert-parallel forward of T own tokens (device pointers, stream-ordered).
int ep_forward_device(Ep *ep, const float *d_x, int T, float *d_out, int32_t *d_route_expert,
                      float *d_route_weight, int32_t *d_status, cudaStream_t st) {
    Ctx *ctx = ep->ctx;
    Layer *L = ep->L;
    const size_t E = L->experts, El = L->e_count, K = L->geo.top_k, H = L->hidden, I = L->inter;
    const size_t tmax = ep->tmax, R = size_t(ep->world) * tmax, RK = R * K, cols = RK + tmax;
    const size_t sc = size_t(bs_stage_cols(L->fmt));
    const size_t ks_gu = ceil_div(H, sc), ks_dn = ceil_div(I, sc);
    const size_t ngrp_gu = 2 * std::min(RK, El) + 2, ngrp_dn = std::min(RK, El) + 1;
    int rc;
    // Workspace: sized by carving once into a null base.
    auto carve = [&](uint8_t *base, MoeWork &w, int32_t *&lids, int32_t *&route_of,
                     float *&y_sh) -> size_t {
        size_t off = 0;
        auto take = [&](size_t bytes) {
            off = align256(off);
            uint8_t *p = base ? base + off : nullptr;
            off += bytes;
            return p;
        };
        w.logits = reinterpret_cast<float *>(take(tmax * E * 4));
        w.x64 = reinterpret_cast<double *>(take(router_f64_elems(int(tmax), int(H)) * 8));
        w.gate = reinterpret_cast<float *>(take(tmax * E * 4));
        w.sel = reinterpret_cast<float *>(take(tmax * E * 4));
        w.ids = reinterpret_cast<int32_t *>(take(tmax * K * 4));
        w.w = reinterpret_cast<float *>(take(tmax * K * 4));
        w.score = reinterpret_cast<float *>(take(tmax * K * 4));
        lids = reinterpret_cast<int32_t *>(take(RK * 4));
        route_of = reinterpret_cast<int32_t *>(take(RK * 4));
        w.counts = reinterpret_cast<int32_t *>(take(El * 4));
        w.offsets = reinterpret_cast<int32_t *>(take((El + 1) * 4));
        w.perm_token = reinterpret_cast<int32_t *>(take(RK * 4));
        w.perm_slot = reinterpret_cast<int32_t *>(take(RK * 4));
        w.inv = reinterpret_cast<int32_t *>(take(RK * 4));
        y_sh = reinterpret_cast<float *>(take(tmax * H * 4));
        w.h = reinterpret_cast<float *>(take(cols * I * 4));
        w.tsegs_gu = reinterpret_cast<TcSeg *>(take(ngrp_gu * sizeof(TcSeg)));
        w.tsegs_dn = reinterpret_cast<TcSeg *>(take(ngrp_dn * sizeof(TcSeg)));
        w.bslots_gu = reinterpret_cast<BsSlot *>(take(cols * sizeof(BsSlot)));
        w.bslots_dn = reinterpret_cast<BsSlot *>(take(cols * sizeof(BsSlot)));
        w.units_gu = reinterpret_cast<int *>(take(max_bs_units(L->fmt, R, K, El, 2 * ceil_div(I, 128)) * 4));
        w.units_dn = reinterpret_cast<int *>(take(max_bs_units(L->fmt, R, K, El, ceil_div(H, 128)) * 4));
        w.tscalars = reinterpret_cast<int *>(take(4 * 4));
        w.bbuf_gu = take(max_bs_bytes(L->fmt, R, K, El, ks_gu));
        w.bbuf_dn = take(max_bs_bytes(L->fmt, R, K, El, ks_dn));
        return align256(off);
    };
    MoeWork w{};
    int32_t *lids = nullptr, *route_of = nullptr;
    float *y_sh = nullptr;
    const size_t need = carve(nullptr, w, lids, route_of, y_sh);
    uint8_t *ws = static_cast<uint8_t *>(workspace(ctx, need, &rc));
    if (!ws) return rc;
    carve(ws, w, lids, route_of, y_sh);
    int32_t *status = d_status;

    // 1. Route the own tokens and publish them.
    uint8_t *win = ep->win;
    if (T > 0) {
        rc = route_device(L, d_x, T, w, status, st);
        if (rc) return rc;
        URB_CUDA(ctx, cudaMemcpyAsync(win + ep->lay.x, d_x, size_t(T) * H * 4,
                                      cudaMemcpyDeviceToDevice, st));
    }
    prof_begin(ctx, URB_K_EXCHANGE, st);
    const int n_ids = int(size_t(T) * K);
    k_ep_publish<<<unsigned(std::max<size_t>(1, ceil_div(n_ids, 256))), 256, 0, st>>>(
        w.ids, n_ids, T, reinterpret_cast<int32_t *>(win + ep->lay.ids),
        reinterpret_cast<int32_t *>(win + ep->lay.ntok));
    prof_end(ctx, st);
    URB_CUDA(ctx, cudaGetLastError());
    prof_begin(ctx, URB_K_EXCHANGE, st);
    rc = barrier(ep, status, st);
    prof_end(ctx, st);
    if (rc) return rc;

    // 2. Routes of all ranks' tokens to the held experts, grouped by expert.
    EpPeers P{};
    for (int i = 0; i < ep->world; ++i) P.win[i] = ep->peer[i];
    prof_begin(ctx, URB_K_EXCHANGE, st);
    k_ep_gather<<<unsigned(ceil_div(RK, 256)), 256, 0, st>>>(P, ep->lay.ntok, ep->lay.ids,
                                                            ep->world, int(tmax), int(K),
                                                            int(L->e_begin), int(El), lids, status);
    prof_end(ctx, st);
    URB_CUDA(ctx, cudaGetLastError());
    PermArgs p{};
    p.ids = lids;
    p.tokens = int(R);
    p.top_k = int(K);
    p.experts = int(El);
    p.cap = 4;
    p.counts = w.counts;
    p.offsets = w.offsets;
    p.perm_token = w.perm_token;
    p.perm_slot = w.perm_slot;
    p.inv = w.inv;
    p.status = status;
    p.allow_foreign = 1;
    p.route_of = route_of;
    prof_begin(ctx, URB_K_PERMUTE, st);
    rc = launch_permute(ctx, p, st);
    prof_end(ctx, st);
    if (rc) return rc;

    void **tb = L->d_tables;
    const size_t S = El + 1;
    const bool shared = L->sg != nullptr && T > 0;
    TcBuildArgs bb{};
    bb.counts = w.counts;
    bb.offsets = w.offsets;
    bb.fmt = L->fmt;
    bb.tokens = int(R);
    bb.top_k = int(K);
    bb.experts = int(El);
    bb.gate_tc = reinterpret_cast<const uint8_t *const *>(tb + 6 * S);
    bb.up_tc = reinterpret_cast<const uint8_t *const *>(tb + 7 * S);
    bb.down_tc = reinterpret_cast<const uint8_t *const *>(tb + 8 * S);
    bb.has_shared = shared ? 1 : 0;
    bb.shared_tokens = T;
    bb.pair_down = 1;
    if (shared) {
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
    bb.status = status;
    prof_begin(ctx, URB_K_GROUP_BUILD, st);
    rc = launch_build_tc_segs(ctx, bb, st);
    prof_end(ctx, st);
    if (rc) return rc;

    // 3. Gate/up over every held route (token rows read from their owners' windows) and the
    // shared expert over the own tokens.
    TcArgs ga{};
    ga.segs = w.tsegs_gu;
    ga.nsegs = w.tscalars;
    ga.total_units = w.tscalars + 1;
    ga.unit_group = w.units_gu;
    ga.bbuf = w.bbuf_gu;
    ga.src = nullptr;
    ga.src_ranks = ep->d_x_ranks;
    ga.rows_per_rank = int(tmax);
    ga.src_stride = int(H);
    ga.nrows = int(R);
    ga.cols = int(H);
    ga.ks = int(ks_gu);
    ga.swiglu = 0;
    ga.inv = w.inv;
    ga.top_k = int(K);
    ga.shared_col0 = shared ? int(RK) : -1;
    ga.shared_row0 = ep->rank * int(tmax);
    ga.shared_rows = T;
    ga.slots = w.bslots_gu;
    ga.pair = 1;  // gate and up tiles of an expert together; the epilogue writes h
    ga.out = w.h;
    ga.out_stride = int(I);
    ga.status = status;
    rc = launch_tc_grouped(ctx, L->fmt, ga, URB_K_GATE_UP, st);
    if (rc) return rc;

    // 4. Down projection of h = silu(gate) * up; routed rows land in their owners' windows,
    // shared rows in y_sh.
    TcArgs da{};
    da.segs = w.tsegs_dn;
    da.nsegs = w.tscalars + 2;
    da.total_units = w.tscalars + 3;
    da.unit_group = w.units_dn;
    da.bbuf = w.bbuf_dn;
    da.src = w.h;
    da.src_stride = int(I);
    da.nrows = int(RK) + (shared ? T : 0);
    da.pair = 2;  // neighbouring row tiles share each activation stage
    da.cols = int(I);
    da.ks = int(ks_dn);
    da.slots = w.bslots_dn;
    da.nvalid = w.offsets + El;
    da.routed_cols = int(RK);
    da.out_rows = route_of;
    da.out_ranks = ep->d_y_ranks;
    da.out_rank_rows = int(tmax * K);
    da.out = y_sh;
    da.out_stride = int(H);
    da.status = status;
    rc = launch_tc_grouped(ctx, L->fmt, da, URB_K_DOWN, st);
    if (rc) return rc;

    prof_begin(ctx, URB_K_EXCHANGE, st);
    rc = barrier(ep, status, st);
    prof_end(ctx, st);
    if (rc) return rc;

    // 5. Combine of the own tokens from the own window (route order t * K + k).
    if (T > 0) {
        prof_begin(ctx, URB_K_COMBINE, st);
        rc = launch_combine(ctx, reinterpret_cast<const float *>(win + ep->lay.y),
                            shared ? y_sh : nullptr, w.w, nullptr, T, int(K), int(H), d_out, st,
                            status);
        prof_end(ctx, st);
        if (rc) return rc;
        if (d_route_expert)
            URB_CUDA(ctx, cudaMemcpyAsync(d_route_expert, w.ids, size_t(T) * K * 4,
                                          cudaMemcpyDeviceToDevice, st));
        if (d_route_weight)
            URB_CUDA(ctx, cudaMemcpyAsync(d_route_weight, w.w, size_t(T) * K * 4,
                                          cudaMemcpyDeviceToDevice, st));
    }
    return URB_OK;
}

}  // namespace urb

using namespace urb;

struct urb_ep : urb::Ep {};

extern "C" {

int urb_ep_create(urb_ctx *ctx, urb_layer *L, int world, int rank, size_t max_tokens,
                  uint32_t timeout_ms, urb_ep **out) {
    if (!ctx || !L || !out) return URB_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    cudaSetDevice(ctx->device);
    *out = nullptr;
    if (world < 1 || world > URB_EP_MAX_WORLD || rank < 0 || rank >= world)
        return set_error(ctx, URB_ERR_INVALID_ARGUMENT, "expert-parallel world / rank out of range");
    if (L->ctx != ctx) return set_error(ctx, URB_ERR_INVALID_ARGUMENT, "layer belongs to another context");
    if (!L->use_tc)
        return set_error(ctx, URB_ERR_UNSUPPORTED, "expert parallelism runs the tensor-core passes (MX experts)");
    if (max_tokens == 0 || max_tokens > (1u << 16))
        return set_error(ctx, URB_ERR_SHAPE, "max_tokens per rank must be in 1..65536");
    const size_t K = L->geo.top_k, H = L->hidden;
    if (size_t(world) * max_tokens * (K + 1) >= (size_t(1) << 31))
        return set_error(ctx, URB_ERR_SHAPE, "expert-parallel route count exceeds 2^31");
    urb_ep *ep = new urb_ep();
    ep->ctx = ctx;
    ep->L = L;
    ep->world = world;
    ep->rank = rank;
    ep->tmax = max_tokens;
    ep->lay = make_layout(max_tokens, K, H);
    ep->timeout_ns = (unsigned long long)(timeout_ms ? timeout_ms : 5000) * 1000000ull;
    cudaError_t err = cudaMalloc(&ep->win, ep->lay.bytes);
    if (err == cudaSuccess) err = cudaMemset(ep->win, 0, ep->lay.bytes);
    if (err == cudaSuccess) err = cudaMalloc(&ep->d_x_ranks, sizeof(float *) * world);
    if (err == cudaSuccess) err = cudaMalloc(&ep->d_y_ranks, sizeof(float *) * world);
    if (err == cudaSuccess) err = cudaMalloc(&ep->d_io, 2 * max_tokens * H * 4);
    if (err == cudaSuccess) err = cudaMalloc(&ep->d_routes, max_tokens * K * 4);
    if (err == cudaSuccess) err = cudaMalloc(&ep->d_rw, max_tokens * K * 4);
    if (err == cudaSuccess) err = cudaDeviceSynchronize();
    if (err != cudaSuccess) {
        urb_ep_free(ep);
        return cuda_fail(ctx, err, "expert-parallel window");
    }
    ep->peer[rank] = ep->win;
    *out = ep;
    return URB_OK;
}

int urb_ep_export(urb_ep *ep, uint8_t *handle) {
    if (!ep || !handle) return URB_ERR_INVALID_ARGUMENT;
    Ctx *ctx = ep->ctx;
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    cudaSetDevice(ctx->device);
    EpBlob b{};
    std::memset(&b, 0, sizeof(b));
    URB_CUDA(ctx, cudaIpcGetMemHandle(&b.ipc, ep->win));
    URB_CUDA(ctx, cudaDeviceGetPCIBusId(b.pci, int(sizeof(b.pci)), ctx->device));
    b.magic = kEpMagic;
    b.world = ep->world;
    b.rank = ep->rank;
    b.tmax = int64_t(ep->tmax);
    b.hidden = int64_t(ep->L->hidden);
    b.top_k = int64_t(ep->L->geo.top_k);
    b.experts = int64_t(ep->L->experts);
    b.e_begin = int64_t(ep->L->e_begin);
    b.e_count = int64_t(ep->L->e_count);
    b.bytes = int64_t(ep->lay.bytes);
    std::memset(handle, 0, URB_EP_HANDLE_BYTES);
    std::memcpy(handle, &b, sizeof(b));
    return URB_OK;
}

int urb_ep_connect(urb_ep *ep, const uint8_t *handles) {
    if (!ep || !handles) return URB_ERR_INVALID_ARGUMENT;
    Ctx *ctx = ep->ctx;
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    cudaSetDevice(ctx->device);
    if (ep->connected) return set_error(ctx, URB_ERR_INVALID_ARGUMENT, "expert-parallel group already connected");
    std::vector<EpBlob> b(ep->world);
    for (int i = 0; i < ep->world; ++i) std::memcpy(&b[i], handles + size_t(i) * URB_EP_HANDLE_BYTES, sizeof(EpBlob));
    // Every rank must describe the same group and layer geometry, and the expert ranges must
    // tile [0, experts) exactly.
    std::vector<int> owner(ep->L->experts, -1);
    for (int i = 0; i < ep->world; ++i) {
        const EpBlob &x = b[i];
        if (x.magic != kEpMagic || x.world != ep->world || x.rank != i || x.tmax != int64_t(ep->tmax) ||
            x.hidden != int64_t(ep->L->hidden) || x.top_k != int64_t(ep->L->geo.top_k) ||
            x.experts != int64_t(ep->L->experts) || x.bytes != int64_t(ep->lay.bytes))
            return set_error(ctx, URB_ERR_INVALID_ARGUMENT, "expert-parallel handles describe different groups or layers");
        if (x.e_begin < 0 || x.e_count <= 0 || x.e_begin + x.e_count > x.experts)
            return set_error(ctx, URB_ERR_SHAPE, "expert-parallel shard range out of bounds");
        for (int64_t e = x.e_begin; e < x.e_begin + x.e_count; ++e) {
            if (owner[e] >= 0) return set_error(ctx, URB_ERR_SHAPE, "expert-parallel shards overlap");
            owner[e] = i;
        }
        for (int j = 0; j < i; ++j)
            if (std::strncmp(b[j].pci, x.pci, sizeof(x.pci)) == 0)
                return set_error(ctx, URB_ERR_UNSUPPORTED,
                                 "two ranks of an expert-parallel group share one GPU; its barriers "
                                 "need every rank on its own device");
    }
    for (int e : owner)
        if (e < 0) return set_error(ctx, URB_ERR_SHAPE, "expert-parallel shards leave an expert unowned");
    for (int i = 0; i < ep->world; ++i) {
        if (i == ep->rank) continue;
        void *p = nullptr;
        cudaError_t err = cudaIpcOpenMemHandle(&p, b[i].ipc, cudaIpcMemLazyEnablePeerAccess);
        if (err != cudaSuccess) {
            for (int j = 0; j < ep->world; ++j)
                if (ep->opened[j]) { cudaIpcCloseMemHandle(ep->peer[j]); ep->opened[j] = false; ep->peer[j] = nullptr; }
            return cuda_fail(ctx, err, "open a peer's expert-parallel window");
        }
        ep->peer[i] = static_cast<uint8_t *>(p);
        ep->opened[i] = true;
    }
    std::vector<const float *> xs(ep->world);
    std::vector<float *> ys(ep->world);
    for (int i = 0; i < ep->world; ++i) {
        xs[i] = reinterpret_cast<const float *>(ep->peer[i] + ep->lay.x);
        ys[i] = reinterpret_cast<float *>(ep->peer[i] + ep->lay.y);
    }
    URB_CUDA(ctx, cudaMemcpy(ep->d_x_ranks, xs.data(), sizeof(float *) * ep->world, cudaMemcpyHostToDevice));
    URB_CUDA(ctx, cudaMemcpy(ep->d_y_ranks, ys.data(), sizeof(float *) * ep->world, cudaMemcpyHostToDevice));
    ep->connected = true;
    return URB_OK;
}

int urb_ep_forward_device(urb_ctx *ctx, urb_ep *ep, const float *d_x, size_t tokens, float *d_out,
                          int32_t *d_route_expert, float *d_route_weight, int32_t *d_status) {
    if (!ctx || !ep || (tokens && (!d_x || !d_out)) || !d_status) return URB_ERR_INVALID_ARGUMENT;
    if (ep->ctx != ctx) return set_error(ctx, URB_ERR_INVALID_ARGUMENT, "expert-parallel group belongs to another context");
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    cudaSetDevice(ctx->device);
    if (!ep->connected) return set_error(ctx, URB_ERR_INVALID_ARGUMENT, "expert-parallel group is not connected");
    if (tokens > ep->tmax) return set_error(ctx, URB_ERR_SHAPE, "more tokens than the group's max_tokens");
    return ep_forward_device(ep, d_x, int(tokens), d_out, d_route_expert, d_route_weight, d_status,
                             ctx->stream);
}

int urb_ep_forward(urb_ctx *ctx, urb_ep *ep, const float *x, size_t tokens, float *out,
                   int32_t *route_expert, float *route_weight) {
    if (!ctx || !ep || (tokens && (!x || !out))) return URB_ERR_INVALID_ARGUMENT;
    if (ep->ctx != ctx) return set_error(ctx, URB_ERR_INVALID_ARGUMENT, "expert-parallel group belongs to another context");
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    cudaSetDevice(ctx->device);
    if (!ep->connected) return set_error(ctx, URB_ERR_INVALID_ARGUMENT, "expert-parallel group is not connected");
    if (tokens > ep->tmax) return set_error(ctx, URB_ERR_SHAPE, "more tokens than the group's max_tokens");
    cudaStream_t st = ctx->stream;
    const size_t H = ep->L->hidden, K = ep->L->geo.top_k;
    float *d_x = ep->d_io, *d_out = ep->d_io + ep->tmax * H;
    URB_CUDA(ctx, cudaMemsetAsync(ctx->d_status, 0, 4, st));
    if (tokens) URB_CUDA(ctx, cudaMemcpyAsync(d_x, x, tokens * H * 4, cudaMemcpyDefault, st));
    int rc = ep_forward_device(ep, d_x, int(tokens), d_out, ep->d_routes, ep->d_rw, ctx->d_status, st);
    if (rc) return rc;
    if (tokens) {
        URB_CUDA(ctx, cudaMemcpyAsync(out, d_out, tokens * H * 4, cudaMemcpyDefault, st));
        if (route_expert)
            URB_CUDA(ctx, cudaMemcpyAsync(route_expert, ep->d_routes, tokens * K * 4, cudaMemcpyDefault, st));
        if (route_weight)
            URB_CUDA(ctx, cudaMemcpyAsync(route_weight, ep->d_rw, tokens * K * 4, cudaMemcpyDefault, st));
    }
    int32_t status = 0;
    URB_CUDA(ctx, cudaMemcpyAsync(&status, ctx->d_status, 4, cudaMemcpyDeviceToHost, st));
    URB_CUDA(ctx, cudaStreamSynchronize(st));
    if (status == URB_ERR_PEER) return set_error(ctx, status, "another rank of the expert-parallel group failed this forward");
    if (status == URB_ERR_TIMEOUT) return set_error(ctx, status, "an expert-parallel barrier timed out");
    if (status) return set_error(ctx, status, "MoE forward rejected its input");
    return URB_OK;
}

int urb_ep_free(urb_ep *ep) {
    if (!ep) return URB_ERR_INVALID_ARGUMENT;
    Ctx *ctx = ep->ctx;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    for (int i = 0; i < URB_EP_MAX_WORLD; ++i)
        if (ep->opened[i]) cudaIpcCloseMemHandle(ep->peer[i]);
    if (ep->win) cudaFree(ep->win);
    if (ep->d_x_ranks) cudaFree(ep->d_x_ranks);
    if (ep->d_y_ranks) cudaFree(ep->d_y_ranks);
    if (ep->d_io) cudaFree(ep->d_io);
    if (ep->d_routes) cudaFree(ep->d_routes);
    if (ep->d_rw) cudaFree(ep->d_rw);
    delete ep;
    return URB_OK;
}

}  // extern "C"
