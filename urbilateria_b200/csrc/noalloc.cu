// noalloc.cu — GatedMlp::forward (src/model/mlp.rs:90-99) on device pointers without any
// allocation: urb_gated_mlp_forward_device_noalloc.  The reference has no counterpart (its
// CPU path allocates Vec buffers per call); this entry point exists for callers that cannot
// allocate device memory while they run the MLP:
//   * serving loops that reserve all free HBM up front (weights + KV cache) and leave none for
//     a library workspace to grow into;
//   * per-token decode loops, where a cudaMalloc synchronises the whole device and stalls the
//     other streams' work.
// Every temporary (segment table, row shifts, SwiGLU max-exponent words, the intermediate h)
// lives in one static device array of kNoallocScratchBytes, carved per call; calls whose
// temporaries do not fit are rejected with URB_ERR_UNSUPPORTED.  The segment table and the
// words that must start at -1000 are written by a set-up kernel on the stream, so no host
// buffer or host-to-device copy is involved either.
//
// The scratch is shared by every call on a device: calls that overlap in time (two streams,
// two contexts or two host threads on one device) race on it and must be serialised by the
// caller.  The first call on a context resolves the scratch's device address with
// cudaGetSymbolAddress (set-up work that should run before any stream capture) and keeps it in
// the context, so a context created after a device reset resolves it afresh.
//
// Only projections with one shared tiled format (MXFP4 / MXFP8 with 32-column groups, BF16)
// are accepted; the other formats compose per-projection products whose temporaries live in
// the context workspace, so they are rejected with URB_ERR_UNSUPPORTED.
#include "urb_internal.cuh"

namespace urb {
namespace {

constexpr size_t kNoallocScratchBytes = size_t(8) << 20;  // 8 MiB per device
constexpr int kMlpCap = 4;  // tokens per segment: hi/lo halves fill one 8-column n-block
__device__ __align__(256) uint8_t g_noalloc_scratch[kNoallocScratchBytes];

// Device address of the scratch for this context's device (the device is current).
int scratch_of(Ctx *ctx, uint8_t **out) {
    if (!ctx->noalloc_scratch) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaGetSymbolAddress(no-alloc scratch)");
        ctx->noalloc_scratch = static_cast<uint8_t *>(p);
    }
    *out = ctx->noalloc_scratch;
    return URB_OK;
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct MlpSetup {
    Seg gu, dn;   // segment 0 templates (col_begin, ntok, row_begin filled per segment)
    int nseg, tokens, gu_rb, dn_rb;
    Seg *segs;    // [2 * nseg]: gate/up pair segments, then down segments
    int *scalars; // nsegs_gu, total_rows_gu, nsegs_dn, total_rows_dn
    int32_t *maxexp;  // [tokens] reset to -1000 (no SwiGLU row seen yet)
};

__global__ void k_mlp_setup(MlpSetup s) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < s.nseg) {
        Seg a = s.gu, b = s.dn;
        a.col_begin = b.col_begin = i * kMlpCap;
        a.ntok = b.ntok = min(kMlpCap, s.tokens - i * kMlpCap);
        a.row_begin = i * 16 * s.gu_rb;
        b.row_begin = i * 16 * s.dn_rb;
        s.segs[i] = a;
        s.segs[s.nseg + i] = b;
    }
    if (i < s.tokens) s.maxexp[i] = -1000;
    if (i == 0) {
        s.scalars[0] = s.nseg;
        s.scalars[1] = s.nseg * 16 * s.gu_rb;
        s.scalars[2] = s.nseg;
        s.scalars[3] = s.nseg * 16 * s.dn_rb;
    }
}

}  // namespace
}  // namespace urb

using namespace urb;

extern "C" {

int urb_gated_mlp_forward_device_noalloc(urb_ctx *ctx, const urb_mat *g, const urb_mat *u,
                                         const urb_mat *d, const float *d_x, size_t tokens,
                                         float *d_out, int32_t *d_status) {
    if (!ctx || !g || !u || !d || !d_x || !d_out) return URB_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    cudaSetDevice(ctx->device);
    // GatedMlp::new_mixed (src/model/mlp.rs:60-81), as urb_gated_mlp_forward_device.
    if (g->rows != u->rows || g->cols != u->cols || d->cols != g->rows || d->rows != g->cols)
        return set_error(ctx, URB_ERR_SHAPE, "gated MLP projections have inconsistent shapes");
    if (tokens == 0) return URB_OK;
    const size_t H = g->cols, I = g->rows, T = tokens;
    // BF16 projections of 1..32 tokens: the split-K tensor-core passes of
    // urb_gated_mlp_forward_device (h in the scratch).
    if (split_tc_applies(g, T) && u->format == g->format && d->format == g->format &&
        T * I * 4 <= kNoallocScratchBytes) {
        uint8_t *base = nullptr;
        int rc = scratch_of(ctx, &base);
        if (rc) return rc;
        rc = split_tc_mlp(ctx, g, u, d, d_x, int(T), reinterpret_cast<float *>(base), d_out, d_status,
                          ctx->stream);
        if (rc != URB_ERR_UNSUPPORTED) return rc;
    }
    // BF16 projections of a few tokens without a tensor map stream the row-major copies.
    if (bf16_gemv_applies(g, T) && bf16_gemv_applies(u, T) && bf16_gemv_applies(d, T) &&
        T * I * 4 <= kNoallocScratchBytes) {
        // The same streaming BF16 passes as urb_gated_mlp_forward_device (h in the scratch).
        uint8_t *base = nullptr;
        int rc = scratch_of(ctx, &base);
        if (rc) return rc;
        rc = launch_bf16_swiglu(ctx, g, u, d, d_x, int(T), reinterpret_cast<float *>(base), d_out,
                                d_status, ctx->stream);
        if (rc != URB_ERR_UNSUPPORTED) return rc;
    }
    if (dense_tc_mlp_applies(g, u, d)) {
        // MX and BF16 projections: the grouped tensor-core passes (tcgen05 tiles / tensor maps),
        // every table, activation stage and h in the scratch (the same passes as the
        // allocating entry point).
        uint8_t *base = nullptr;
        int rc = scratch_of(ctx, &base);
        if (rc) return rc;
        return dense_tc_mlp(ctx, g, u, d, d_x, int(T), d_out, d_status, ctx->stream, base,
                            kNoallocScratchBytes);
    }
    if (!g->tiled || !u->tiled || !d->tiled || g->format != u->format)
        return set_error(ctx, URB_ERR_UNSUPPORTED,
                         "no-alloc gated MLP needs gate/up/down in one tiled format (MXFP4 / "
                         "MXFP8 with 32-column groups, or BF16)");
    const size_t nseg = (T + kMlpCap - 1) / kMlpCap;
    // Carve: row shifts [T], segments [2 nseg], scalars [4], max-exponent words [T], h [T, I].
    size_t off = 0;
    const size_t o_shift = off; off = align256(off + T * 4);
    const size_t o_segs = off; off = align256(off + 2 * nseg * sizeof(Seg));
    const size_t o_sc = off; off = align256(off + 4 * sizeof(int));
    const size_t o_max = off; off = align256(off + T * 4);
    const size_t o_h = off; off = align256(off + T * I * 4);
    if (off > kNoallocScratchBytes || T > size_t(INT32_MAX))
        return set_error(ctx, URB_ERR_UNSUPPORTED,
                         "gated MLP needs " + std::to_string(off) + " bytes of scratch; the no-alloc "
                         "scratch holds " + std::to_string(kNoallocScratchBytes) + " (8 MiB)");
    uint8_t *base = nullptr;
    int rc = scratch_of(ctx, &base);
    if (rc) return rc;
    int32_t *shift = reinterpret_cast<int32_t *>(base + o_shift);
    Seg *segs = reinterpret_cast<Seg *>(base + o_segs);
    int *sc = reinterpret_cast<int *>(base + o_sc);
    int32_t *maxexp = reinterpret_cast<int32_t *>(base + o_max);
    float *h = reinterpret_cast<float *>(base + o_h);
    cudaStream_t st = ctx->stream;

    MlpSetup s{};
    s.gu.tiles_a = g->tiles; s.gu.rexp_a = g->row_exp; s.gu.tiles_b = u->tiles; s.gu.rexp_b = u->row_exp;
    s.gu.rbs = g->rbs; s.gu.rows = int(I); s.gu.kslices = g->kslices; s.gu.cols = int(H);
    s.dn.tiles_a = d->tiles; s.dn.rexp_a = d->row_exp; s.dn.tiles_b = nullptr; s.dn.rexp_b = nullptr;
    s.dn.rbs = d->rbs; s.dn.rows = int(H); s.dn.kslices = d->kslices; s.dn.cols = int(I);
    s.nseg = int(nseg);
    s.tokens = int(T);
    s.gu_rb = g->rbs;
    s.dn_rb = d->rbs;
    s.segs = segs;
    s.scalars = sc;
    s.maxexp = maxexp;
    const size_t n = std::max(nseg, T);
    k_mlp_setup<<<unsigned((n + 255) / 256), 256, 0, st>>>(s);
    URB_CUDA(ctx, cudaGetLastError());

    if (launch_row_shift(d_x, int(T), int(H), int(H), shift, d_status, st))
        return cuda_fail(ctx, cudaGetLastError(), "row shift");
    GroupArgs a{};
    a.segs = segs; a.nsegs = sc; a.total_rows = sc + 1;
    a.src = d_x; a.src_stride = int(H); a.src_shift = shift;
    a.out = h; a.out_stride = int(I); a.out_maxexp = maxexp; a.hilo = 1;
    const long per_sm_gu = long(nseg) * 16 * g->rbs / std::max(1, ctx->num_sms);
    prof_begin(ctx, URB_K_GATE_UP, st);
    rc = launch_grouped_ex(ctx, g->format, true, per_sm_gu < 64 ? 8 : per_sm_gu < 256 ? 2 : 1, a,
                           2 * kMlpCap, g->kslices, st);
    prof_end(ctx, st);
    if (rc) return rc;
    GroupArgs b{};
    b.segs = segs + nseg; b.nsegs = sc + 2; b.total_rows = sc + 3;
    b.src = h; b.src_stride = int(I); b.src_maxexp = maxexp;
    b.out = d_out; b.out_stride = int(H); b.hilo = 1;
    const long per_sm_dn = long(nseg) * 16 * d->rbs / std::max(1, ctx->num_sms);
    prof_begin(ctx, URB_K_DOWN, st);
    rc = launch_grouped_ex(ctx, d->format, false, per_sm_dn < 64 ? 8 : per_sm_dn < 256 ? 2 : 1,
                           b, 2 * kMlpCap, d->kslices, st);
    prof_end(ctx, st);
    return rc;
}

}  // extern "C"
