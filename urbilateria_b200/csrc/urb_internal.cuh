// urb_internal.cuh — definitions shared by the CUDA translation units of liburb_moe.
//
// Device layout of a resident weight matrix ("tiled layout", built at upload):
//   The matrix is cut into tiles of 16 rows x 128 columns (rows padded to 16, columns to 128
//   with zero weights).  Tiles are stored row-block-major: tile(rb, s) at (rb*kslices + s).
//   Inside a tile, the bytes are ordered for the mma.sync m16n8k16 A fragment: lane
//   t = 4g + q owns one 32-column group (columns 128s + 32q .. +31) of two rows,
//   16rb+g and 16rb+g+8, stored back to back (MXFP4: 16 B + 16 B, MXFP8: 32 B + 32 B,
//   BF16: 64 B + 64 B).  MX tiles end with 64 B of E8M0 scales: lane t's two scale bytes
//   (row g, row g+8) at 2t.  So one warp reads one tile as one contiguous block.
//   A per-row exponent offset E0 (int8) makes every decoded weight exact in f16:
//   w_f16 = e2m1|e4m3 * 2^(scale-127-E0), and the epilogue multiplies by 2^E0.
#pragma once

#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <utility>
#include <string>
#include <vector>

#include "../../include/urb_moe.h"

namespace urb {

constexpr int kWarpSize = 32;
constexpr int kTileRows = 16;
constexpr int kTileCols = 128;

// Bytes of one tile's weight payload and the whole tile (payload + scales) per format.
__host__ __device__ constexpr int tile_payload_bytes(int fmt) {
    return fmt == URB_FMT_MXFP4 ? 1024 : fmt == URB_FMT_MXFP8 ? 2048 : 4096;
}
__host__ __device__ constexpr int tile_bytes(int fmt) {
    return tile_payload_bytes(fmt) + ((fmt == URB_FMT_MXFP4 || fmt == URB_FMT_MXFP8) ? 64 : 0);
}

struct Ctx;

// Device-resident matrix.
struct Mat {
    Ctx *ctx = nullptr;
    int format = 0;
    size_t rows = 0, cols = 0;
    size_t group_size = 0, block_rows = 0, block_cols = 0;
    size_t resident_bytes = 0;  // reference payload bytes (WeightMatrix::resident_bytes)
    // mma.sync layout: `tiled` says the matrix can take it (BF16 keeps it from the upload on;
    // MX matrices build it on first use from their tcgen05 tiles, ensure_mma_tiles).
    bool tiled = false;
    int rbs = 0, kslices = 0;
    uint8_t *tiles = nullptr;
    int8_t *row_exp = nullptr;  // [rbs*16]
    // Tensor-core (tcgen05) layout of MX matrices: 128-row x 128-byte tiles with their
    // scales, K-stage major (tc_mts row tiles x tc_ks K stages).
    uint8_t *tc_tiles = nullptr;
    // BF16 matrices (cols a multiple of 8): a TMA tensor map (CUtensorMap in device memory)
    // over the row-major copy, boxes of 128 rows x 64 columns in the 128-byte swizzle, and its
    // host copy (kernels that take it as a parameter).
    void *tc_map = nullptr;
    alignas(64) unsigned char tc_map_host[128] = {};
    int tc_mts = 0, tc_ks = 0;
    // Generic path: the reference layout on the device (used when !tiled).
    void *raw_values = nullptr;
    uint8_t *raw_scales = nullptr;
};

// What the grouped tensor-core passes read a matrix's tiles from: MX matrices' resident tiles,
// BF16 matrices' tensor map (null when the matrix cannot take the passes).
inline const uint8_t *tc_src(const Mat *m) {
    return m->format == URB_FMT_BF16 ? static_cast<const uint8_t *>(m->tc_map) : m->tc_tiles;
}

// One unit of grouped work: a matrix (or a gate/up pair) applied to a contiguous run of
// columns of the activation list.
struct Seg {
    const uint8_t *tiles_a;
    const int8_t *rexp_a;
    const uint8_t *tiles_b;  // pair partner (up projection) or nullptr
    const int8_t *rexp_b;
    int rbs;        // row blocks of the (each) matrix
    int rows;       // real rows (outputs written only below this)
    int kslices;    // 128-column slices
    int cols;       // real input columns
    int col_begin;  // first activation column of this segment
    int ntok;       // tokens in this segment
    int row_begin;  // prefix of 16*rbs over preceding segments (work space coordinate)
    int pad;
};

// Exception table of the libm expf evaluation (expf_glibc.cuh): sorted input keys, their
// libm results, and a bucket index over the top 20 bits of the input.
struct ExpfTable {
    const uint32_t *keys;
    const uint32_t *vals;
    const uint32_t *index;
};

// Arguments of one grouped pass.
struct GroupArgs {
    const Seg *segs;
    const int *nsegs;         // device scalar: number of segments
    const int *total_rows;    // device scalar: sum of 16*rbs
    const float *src;         // activation rows (f32), row stride src_stride
    int src_stride;
    const int32_t *col_src;   // activation column -> src row (nullptr: identity)
    const int32_t *src_shift; // src row -> power-of-two shift that puts max|x| in [2^14, 2^15)
    const int32_t *src_maxexp;// alternative to src_shift: src row -> ilogb(max|x|) or -1000
    float *out;               // output rows, stride out_stride, indexed by activation column
    int out_stride;
    int32_t *out_maxexp;      // SwiGLU: per output row ilogb(max|h|) (atomicMax), or nullptr
    int hilo;                 // 1: two f16/bf16 columns (hi, lo) per token
    const int *lofree;        // optional device flag: 1 -> every activation is exact in one
                              // f16/bf16 column, so the pass runs without lo columns
    // Checkpoint numerics (0: f32 outputs).  2 (Qwen3.6): gate and up round to BF16, h =
    // BF16(BF16(silu(gate)) * up) with the libm expf (expf); other passes round outputs to
    // BF16.  Non-finite results set status.
    int variant;
    int32_t *status;
    ExpfTable expf;
};

struct Ctx {
    int device = 0;
    int num_sms = 148;
    cudaStream_t stream = nullptr;
    bool own_stream = false;
    // Side stream of work that runs beside the caller's stream inside one call (forked and
    // joined by the two events, so that it also records into a CUDA graph).
    cudaStream_t aux = nullptr;
    cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
    std::recursive_mutex mu;
    std::string last_error;
    int last_status = 0;
    // Grow-only device workspace.
    void *ws = nullptr;
    size_t ws_size = 0;
    // Grow-only device buffer for the host-pointer entry points' staged inputs and outputs.
    void *io = nullptr;
    size_t io_size = 0;
    // Pinned host staging.
    void *pinned = nullptr;
    size_t pinned_size = 0;
    int32_t *d_status = nullptr;  // device status word for host-pointer calls
    // Device address of the no-alloc entry point's static scratch on this context's device
    // (resolved by its first call on the context; noalloc.cu).
    uint8_t *noalloc_scratch = nullptr;
    // glibc-expf exception table (see expf_glibc.cuh).
    const uint32_t *expf_keys = nullptr;
    const uint32_t *expf_vals = nullptr;
    const uint32_t *expf_index = nullptr;
    int expf_count = 0;
    // glibc-log1pf exception table over [0, 1] (same layout).
    const uint32_t *log1pf_keys = nullptr;
    const uint32_t *log1pf_vals = nullptr;
    const uint32_t *log1pf_index = nullptr;
    // Optional per-launch profiler (urb_profile_*).
    bool prof = false;
    struct ProfRec { int kind; cudaEvent_t a, b; };
    std::vector<ProfRec> prof_pending;
    std::vector<cudaEvent_t> prof_free;
    double prof_ms[URB_K_COUNT] = {};
    long long prof_n[URB_K_COUNT] = {};
    int prof_open = -1;
    cudaEvent_t prof_open_ev = nullptr;
};

// Brackets one launch for the profiler (no-op when profiling is off).
void prof_begin(Ctx *ctx, int kind, cudaStream_t st);
void prof_end(Ctx *ctx, cudaStream_t st);

int set_error(Ctx *ctx, int status, const std::string &msg);
int cuda_fail(Ctx *ctx, cudaError_t err, const char *what);
void *workspace(Ctx *ctx, size_t bytes, int *status);
void *pinned_staging(Ctx *ctx, size_t bytes, int *status);
// Device buffer of the host-pointer entry points (x in, results out); never carved by the
// device paths, which use workspace().
void *io_buffer(Ctx *ctx, size_t bytes, int *status);

#define URB_CUDA(ctx, expr)                                                  \
    do {                                                                     \
        cudaError_t _e = (expr);                                             \
        if (_e != cudaSuccess) return ::urb::cuda_fail((ctx), _e, #expr);    \
    } while (0)

// ---- kernels exposed across translation units (host launchers) -------------------------

// upload.cu
int upload_matrix(Ctx *ctx, Mat *m, const void *values, const uint8_t *scales);
// skinny.cu: grouped register-dequant tensor-core pass over segments on the device.
// ksplit: warps cooperating on one 16-row block (1, 2 or 8); max_cols <= 16.
int launch_grouped_ex(Ctx *ctx, int fmt, bool pair, int ksplit, const GroupArgs &args,
                      int max_cols, int kslices_max, cudaStream_t stream);
// generic.cu: fallback for matrices without the tiled layout (CUDA cores, fp32).
int launch_generic_matmul(Ctx *ctx, const Mat *m, size_t start, size_t count, const float *d_x,
                          size_t batch, float *d_y, cudaStream_t stream);
// prep: per-row shift and non-finite check; optionally clears *d_lofree when some row is not
// exactly representable in one f16 (bf16_check=0) / bf16 (bf16_check=1) column after its shift.
int launch_row_shift(const float *d_src, int rows, int cols, int stride, int32_t *d_shift,
                     int32_t *d_status, cudaStream_t stream, int32_t *d_lofree = nullptr,
                     int bf16_check = 0);
// router.cu
// Gates and selection scores of route_noaux_tc computed in the logits kernel's epilogue.
struct RouterGates {
    const Ctx *ctx;
    const float *bias;
    float *gate, *sel;  // [tokens, experts]
    int32_t *status;    // non-finite logit or bias -> URB_ERR_NONFINITE
};

int launch_route_noaux(Ctx *ctx, const float *d_logits, const float *d_bias, int tokens,
                       int experts, const urb_moe_geometry &g, int32_t *d_expert,
                       float *d_weight, float *d_score, int32_t *d_status, cudaStream_t st,
                       const RouterGates *pre = nullptr);
// Router logits on f64 copies in the router's blocked layout: 8-row blocks cut into chunks of
// kRc columns, each chunk one contiguous [8][kRrow] tile (rows padded; zero past the matrix).
// w64 (widen_router_f64, resident) holds router_f64_elems(experts, cols) doubles, the x64
// scratch router_f64_elems(tokens, cols), widened from d_x by launch_router_logits_f64.  The
// logits are bit-identical to the sequential F64 chain.
constexpr int kRc = 128;                  // columns per chunk (one shared-memory stage)
constexpr int kRrow = kRc + 4;            // doubles per staged row
constexpr int kRnb = 3;                   // stages in flight per block (many blocks)
constexpr int kRstage = 16 * kRrow;       // doubles per stage (x tile + router tile)
__host__ __device__ constexpr int router_smem(int nb) { return nb * kRstage * 8 + 2 * nb * 8; }
__host__ __device__ constexpr int router_chunks(int cols) { return (cols + kRc - 1) / kRc; }
__host__ __device__ constexpr size_t router_f64_elems(int rows, int cols) {
    return size_t((rows + 7) / 8) * router_chunks(cols) * 8 * kRrow;
}
int widen_router_f64(const Mat *router, double *dst, cudaStream_t st);
// Single-token product of rows [start, start + count) of a tiled MXFP4 / MXFP8 matrix.
// BF16 products of at most kBf16GemvMaxTokens tokens on CUDA cores (gemv_bf16.cu): rows
// [start, start + count) of m times x [tokens, cols] into y [tokens, count]; and the gated MLP
// with BF16 gate / up / down (h [tokens, inter] is the caller's scratch).
constexpr size_t kBf16GemvMaxTokens = 32;
bool bf16_gemv_applies(const Mat *m, size_t tokens);
int launch_bf16_gemv(Ctx *ctx, const Mat *m, size_t start, size_t count, const float *d_x,
                     size_t tokens, float *d_y, int32_t *d_status, cudaStream_t st);
int launch_bf16_swiglu(Ctx *ctx, const Mat *g, const Mat *u, const Mat *d, const float *d_x,
                       int tokens, float *d_h, float *d_out, int32_t *d_status, cudaStream_t st);
int launch_matvec1(Ctx *ctx, const Mat *m, size_t start, size_t count, const float *d_x,
                   float *d_y, cudaStream_t st);
// dense_tc.cu: MX and BF16 gated MLP and batched products on the grouped tensor-core passes
// (MX: the resident tcgen05 tiles; BF16: the tensor map), all tokens in one group.
// dense_tc_mlp uses `mem` (mem_bytes of device memory, at least dense_tc_mlp_bytes) when
// given, else the context workspace.
bool dense_tc_mlp_applies(const Mat *g, const Mat *u, const Mat *d);
size_t dense_tc_mlp_bytes(const Mat *g, const Mat *u, const Mat *d, int T);
int dense_tc_mlp(Ctx *ctx, const Mat *g, const Mat *u, const Mat *d, const float *d_x, int T,
                 float *d_out, int32_t *d_status, cudaStream_t st, uint8_t *mem, size_t mem_bytes);
// Rows [start, start + count) of a matrix the passes take (dense_tc_applies) times d_x
// [T, cols] into d_y [T, count].
bool dense_tc_applies(const Mat *m);
int dense_tc_product(Ctx *ctx, const Mat *m, size_t start, size_t count, const float *d_x, int T,
                     float *d_y, int32_t *d_status, cudaStream_t st);
// split_tc.cu: BF16 products and gated MLPs of 1..32 tokens on tcgen05 kind::f16 with K split
// over thread-block clusters (whole rows; d_h [T, I] holds the MLP's h).
bool split_tc_applies(const Mat *m, size_t T);
int split_tc_product(Ctx *ctx, const Mat *m, const float *d_x, int T, float *d_y, int32_t *d_status,
                     cudaStream_t st);
int split_tc_mlp(Ctx *ctx, const Mat *g, const Mat *u, const Mat *d, const float *d_x, int T,
                 float *d_h, float *d_out, int32_t *d_status, cudaStream_t st);
// upload.cu: the 16-row mma.sync tiles of an MX matrix, built from its tcgen05 tiles on first
// use (the mma.sync layer passes and the CUDA-core single-token fallback); MX uploads keep only
// the tcgen05 tiles.
int ensure_mma_tiles(Ctx *ctx, const Mat *m, cudaStream_t st);
// Single-token product on the block-scaled tensor cores over the resident tcgen05 tiles
// (matvec_tc.cu); d_status (may be null) receives URB_ERR_NONFINITE for a non-finite input.
bool matvec_tc_applies(const Mat *m);
int launch_matvec_tc(Ctx *ctx, const Mat *m, size_t start, size_t count, const float *d_x,
                     float *d_y, int32_t *d_status, cudaStream_t st);
// api.cu: y[batch, count] = rows start..start+count of any matrix times d_x [batch, cols]
// (device pointers, stream-ordered; every format and layout).
int product_device(Ctx *ctx, const Mat *m, size_t start, size_t count, const float *d_x,
                   size_t batch, float *d_y, int32_t *d_status, cudaStream_t st);
// quant.cu: Int8Matrix / Int4Matrix row products and the INT4 grouped quantiser.
int launch_int_matmul(Ctx *ctx, const Mat *m, size_t start, size_t count, const float *d_x,
                      size_t batch, float *d_y, int32_t *d_status, cudaStream_t st);
int int4_quantize_device(Ctx *ctx, size_t rows, size_t cols, size_t group, const float *d_values,
                         uint8_t *d_packed, float *d_scales, int32_t *d_flag, cudaStream_t st);
inline bool is_int_format(int fmt) { return fmt == URB_FMT_INT8 || fmt == URB_FMT_INT4; }
int launch_router_logits_f64(const double *w64, int experts, const float *d_x, int tokens,
                             int cols, double *x64, float *d_logits, cudaStream_t st,
                             const RouterGates *gates = nullptr);
// route_sqrt_softplus (deepseek_v4/math.rs:451-516): bias and hash ([tokens, top_k] fixed
// experts) optional; outputs [tokens, top_k] in selection order.
int launch_route_sqrt_softplus(Ctx *ctx, const float *d_logits, const float *d_bias,
                               const int32_t *d_hash, int tokens, int experts, int top_k,
                               float scaling, int32_t *d_expert, float *d_weight, float *d_score,
                               int32_t *d_status, cudaStream_t st);
// bf16_weights: the selected weights round to BF16 (qwen3_6/runtime.rs:1086-1090).
int launch_route_softmax(Ctx *ctx, const float *d_logits, int tokens, int experts, int top_k,
                         int32_t *d_expert, float *d_weight, int32_t *d_status,
                         cudaStream_t stream, int bf16_weights = 0);
// Qwen3.6 BF16 linear (dot_bf16_fp32_avx2_fma, src/model/bf16.rs:591-613, rounded to BF16):
// logits[t, r] for the `rows` rows of w (row-major BF16 [rows, cols]) and, when gate_row is
// set, gate_logit[t] for that [1, cols] BF16 row.  Non-finite results set status.
int launch_router_bf16_lanes(const uint16_t *w, int rows, const uint16_t *gate_row,
                             const float *d_x, int tokens, int cols, float *d_logits,
                             float *d_gate_logit, int32_t *d_status, cudaStream_t st);
inline ExpfTable expf_table_of(const Ctx *ctx) {
    return ExpfTable{ctx->expf_keys, ctx->expf_vals, ctx->expf_index};
}
// expf_glibc.cu
int expf_table_init(Ctx *ctx);

// ---- device helpers ----------------------------------------------------------------------
#if defined(__CUDACC__)
// Rust f32::total_cmp as a signed-integer key (IEEE totalOrder on the bit pattern).
__device__ __forceinline__ int32_t total_key(float v) {
    int32_t b = __float_as_int(v);
    return b ^ int32_t(uint32_t(b >> 31) >> 1);
}

// Programmatic dependent launch.  The kernels of the layer path each start with grid_dep_wait
// (all their reads and writes come after the kernel ahead of them has completed and its
// memory is visible) and then grid_dep_trigger, and are launched with launch_dep, so the
// launch of each overlaps the run of the one before it (also inside a CUDA graph).  Launched
// without the attribute, both instructions do nothing.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
template <typename... P, typename... A>
cudaError_t launch_dep(void (*k)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, A &&...args) {
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t c = {};
    c.gridDim = grid;
    c.blockDim = block;
    c.dynamicSmemBytes = smem;
    c.stream = st;
    c.attrs = at;
    c.numAttrs = 1;
    return cudaLaunchKernelEx(&c, k, std::forward<A>(args)...);
}
// A dependent launch written like k<<<g, b, smem, st>>>(args...): a launch error is left for
// cudaGetLastError.  (A kernel name with template arguments goes through a variable first.)
#define URB_LAUNCH_DEP(k, g, b, sm, st, ...) (void)::urb::launch_dep(k, dim3(g), dim3(b), size_t(sm), st, __VA_ARGS__)
#endif

}  // namespace urb

struct urb_ctx : urb::Ctx {};
struct urb_mat : urb::Mat {};
struct urb_layer;
