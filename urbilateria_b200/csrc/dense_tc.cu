// dense_tc.cu — GatedMlp::forward (src/model/mlp.rs:90-99) and WeightMatrix::matmul_rows
// (src/model/weight.rs:106-153) for MX and BF16 matrices on the tensor-core passes of
// grouped_tc.cu, reading the same tiles as the MoE layer (MX: the resident 128-row tiles, of
// which MX matrices keep no other copy; BF16: boxes of the row-major matrix through its
// tensor map).
//
// Every token goes into one group (no routing): the gate/up pass pairs the gate and up tiles of
// the MLP against each activation stage and writes h = silu(gate) * up, the down pass pairs
// neighbouring row tiles; a single-matrix product is one down-style pass.  The group's tables
// (segment, unit map, activation slots) are written by a small kernel on the stream, so the path
// runs from any device memory the caller provides: the context workspace, or the no-alloc entry
// point's static scratch.
#include <algorithm>

#include "urb_internal.cuh"
#include "urb_tc.cuh"

namespace urb {
namespace {

constexpr size_t kAlign = 256;
size_t up256(size_t x) { return (x + kAlign - 1) & ~(kAlign - 1); }

// Bytes of the activation stages of one group of c tokens over ks K stages (sub-segments of
// bs_cap tokens; the last one only as wide as its tokens need).
__host__ __device__ long long dense_group_bytes(int fmt, int c, int ks) {
    const int cap = bs_cap(fmt);
    const int nsub = (c + cap - 1) / cap;
    const int n_last = (bs_rows_per_tok(fmt) * (c - (nsub - 1) * cap) + 15) & ~15;
    return (long long)ks * ((long long)(nsub - 1) * bs_bstage_bytes(fmt, kBsNmax) + bs_bstage_bytes(fmt, n_last));
}

struct DensePass {
    const uint8_t *w, *w2;  // bs tiles (gate/up pass: gate and up)
    int mts, ks, rows, cols;
    int mtu;                // tile units per sub-segment (paired row tiles: ceil(mts / 2))
};

int dense_units(int fmt, int T, const DensePass &p) { return p.mtu * ((T + bs_cap(fmt) - 1) / bs_cap(fmt)); }

// The tables of one pass: its single group, scalars (groups, units), the unit -> group map
// (all 0) and the activation slot of every token.
__global__ void k_dense_tables(int fmt, int T, DensePass p, TcSeg *seg, int *scalars, int *units,
                               BsSlot *slots) {
    const int cap = bs_cap(fmt), nsub = (T + cap - 1) / cap;
    const int U = p.mtu * nsub;
    const int tid = blockIdx.x * blockDim.x + threadIdx.x;
    if (tid == 0) {
        TcSeg s;
        s.w = p.w;
        s.w2 = p.w2;
        s.b_off = 0;
        s.mts = p.mts;
        s.ks = p.ks;
        s.rows = p.rows;
        s.cols = p.cols;
        s.col_begin = 0;
        s.ntok = T;
        s.nsub = nsub;
        s.unit_begin = 0;
        s.out_off = 0;
        s.pad = 0;
        *seg = s;
        scalars[0] = 1;
        scalars[1] = U;
    }
    for (int i = tid; i < max(U, T); i += gridDim.x * blockDim.x) {
        if (i < U) units[i] = 0;
        if (i < T) {
            const int sub = i / cap;
            BsSlot z;
            z.base = (long long)sub * p.ks * bs_bstage_bytes(fmt, kBsNmax);
            z.slot = i - sub * cap;
            z.n = sub < nsub - 1 ? kBsNmax : (bs_rows_per_tok(fmt) * (T - (nsub - 1) * cap) + 15) & ~15;
            slots[i] = z;
        }
    }
}

// Carves the tables and activation stages of one pass out of [*p, end).
struct PassMem {
    TcSeg *seg;
    int *scalars, *units;
    BsSlot *slots;
    uint8_t *bbuf;
};

size_t pass_bytes(int fmt, int T, const DensePass &p) {
    return up256(sizeof(TcSeg)) + up256(2 * sizeof(int)) + up256(size_t(dense_units(fmt, T, p)) * sizeof(int)) +
           up256(size_t(T) * sizeof(BsSlot)) + up256(size_t(dense_group_bytes(fmt, T, p.ks)));
}

PassMem carve_pass(uint8_t *&cur, int fmt, int T, const DensePass &p) {
    PassMem m;
    m.seg = reinterpret_cast<TcSeg *>(cur); cur += up256(sizeof(TcSeg));
    m.scalars = reinterpret_cast<int *>(cur); cur += up256(2 * sizeof(int));
    m.units = reinterpret_cast<int *>(cur); cur += up256(size_t(dense_units(fmt, T, p)) * sizeof(int));
    m.slots = reinterpret_cast<BsSlot *>(cur); cur += up256(size_t(T) * sizeof(BsSlot));
    m.bbuf = cur; cur += up256(size_t(dense_group_bytes(fmt, T, p.ks)));
    return m;
}

int build_tables(Ctx *ctx, int fmt, int T, const DensePass &p, const PassMem &m, cudaStream_t st) {
    const int n = std::max(dense_units(fmt, T, p), T);
    k_dense_tables<<<unsigned(std::min(1024, (n + 255) / 256)), 256, 0, st>>>(fmt, T, p, m.seg, m.scalars,
                                                                                m.units, m.slots);
    URB_CUDA(ctx, cudaGetLastError());
    return URB_OK;
}

TcArgs pass_args(const PassMem &m, const DensePass &p, const float *src, int src_stride, int T,
                 int pair, float *out, int out_stride, int32_t *status) {
    TcArgs a{};
    a.segs = m.seg;
    a.nsegs = m.scalars;
    a.total_units = m.scalars + 1;
    a.unit_group = m.units;
    a.bbuf = m.bbuf;
    a.src = src;
    a.src_stride = src_stride;
    a.nrows = T;
    a.cols = p.cols;
    a.ks = p.ks;
    a.inv = nullptr;        // source row t feeds activation column t
    a.shared_col0 = -1;
    a.slots = m.slots;
    a.pair = pair;
    a.out = out;
    a.out_stride = out_stride;
    a.status = status;
    return a;
}

DensePass gu_pass(const Mat *g, const Mat *u) {
    return DensePass{tc_src(g), tc_src(u), g->tc_mts, g->tc_ks, int(g->rows), int(g->cols), g->tc_mts};
}
DensePass single_pass(const Mat *m) {
    return DensePass{tc_src(m), nullptr, m->tc_mts, m->tc_ks, int(m->rows), int(m->cols), (m->tc_mts + 1) / 2};
}

}  // namespace

bool dense_tc_applies(const Mat *m) {
    const int f = m->format;
    return (f == URB_FMT_MXFP4 || f == URB_FMT_MXFP8 || f == URB_FMT_BF16) && tc_src(m);
}

bool dense_tc_mlp_applies(const Mat *g, const Mat *u, const Mat *d) {
    const int f = g->format;
    return u->format == f && d->format == f && dense_tc_applies(g) && dense_tc_applies(u) &&
           dense_tc_applies(d);
}

size_t dense_tc_mlp_bytes(const Mat *g, const Mat *u, const Mat *d, int T) {
    const int fmt = g->format;
    return pass_bytes(fmt, T, gu_pass(g, u)) + pass_bytes(fmt, T, single_pass(d)) +
           up256(size_t(T) * g->rows * sizeof(float));
}

int dense_tc_mlp(Ctx *ctx, const Mat *g, const Mat *u, const Mat *d, const float *d_x, int T,
                 float *d_out, int32_t *d_status, cudaStream_t st, uint8_t *mem, size_t mem_bytes) {
    if (T <= 0) return URB_OK;
    const int fmt = g->format;
    const DensePass pg = gu_pass(g, u), pd = single_pass(d);
    const size_t need = dense_tc_mlp_bytes(g, u, d, T);
    int rc;
    if (!mem) {
        mem = static_cast<uint8_t *>(workspace(ctx, need, &rc));
        if (!mem) return rc;
    } else if (need > mem_bytes) {
        return set_error(ctx, URB_ERR_UNSUPPORTED,
                         "gated MLP needs " + std::to_string(need) + " bytes of scratch; " +
                             std::to_string(mem_bytes) + " available");
    }
    uint8_t *cur = mem;
    const PassMem mg = carve_pass(cur, fmt, T, pg), md = carve_pass(cur, fmt, T, pd);
    float *h = reinterpret_cast<float *>(cur);
    if ((rc = build_tables(ctx, fmt, T, pg, mg, st))) return rc;
    if ((rc = build_tables(ctx, fmt, T, pd, md, st))) return rc;
    const int H = int(g->cols), I = int(g->rows);
    rc = launch_tc_grouped(ctx, fmt, pass_args(mg, pg, d_x, H, T, 1, h, I, d_status), URB_K_GATE_UP, st);
    if (rc) return rc;
    return launch_tc_grouped(ctx, fmt, pass_args(md, pd, h, I, T, 2, d_out, H, d_status), URB_K_DOWN, st);
}

int dense_tc_product(Ctx *ctx, const Mat *m, size_t start, size_t count, const float *d_x, int T,
                     float *d_y, int32_t *d_status, cudaStream_t st) {
    if (T <= 0 || count == 0) return URB_OK;
    const int fmt = m->format;
    const DensePass p = single_pass(m);
    // The passes write whole rows; a row range goes through a [T, rows] buffer.
    const bool direct = start == 0 && count == m->rows;
    const size_t tmp = direct ? 0 : up256(size_t(T) * m->rows * sizeof(float));
    int rc;
    uint8_t *mem = static_cast<uint8_t *>(workspace(ctx, pass_bytes(fmt, T, p) + tmp, &rc));
    if (!mem) return rc;
    uint8_t *cur = mem;
    const PassMem pm = carve_pass(cur, fmt, T, p);
    float *y = direct ? d_y : reinterpret_cast<float *>(cur);
    if ((rc = build_tables(ctx, fmt, T, p, pm, st))) return rc;
    rc = launch_tc_grouped(ctx, fmt, pass_args(pm, p, d_x, int(m->cols), T, 2, y, int(m->rows), d_status),
                           URB_K_PRODUCT, st);
    if (rc || direct) return rc;
    URB_CUDA(ctx, cudaMemcpy2DAsync(d_y, count * 4, y + start, m->rows * 4, count * 4, size_t(T),
                                    cudaMemcpyDeviceToDevice, st));
    return URB_OK;
}

}  // namespace urb
