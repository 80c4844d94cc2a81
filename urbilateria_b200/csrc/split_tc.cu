// split_tc.cu — BF16 products and gated MLPs of a few tokens (Bf16Matrix::matmul_rows,
// src/model/bf16.rs:116-416; GatedMlp::forward, src/model/mlp.rs:90-99) on tcgen05 kind::f16
// with the K dimension split over thread-block clusters.
//
// A few tokens leave a dense product with a handful of 128-row tiles, far fewer than the SMs,
// so every row tile is a cluster of `ksplit` CTAs, each one a contiguous K range of stages
// (64 columns each):
//   * lane 0 of warp 0 requests the CTA's weight boxes first (2-D tiled TMA through the
//     matrix's tensor map, the 128-byte swizzled K-major layout the MMA reads), before the
//     kernel waits for the one ahead of it (programmatic dependent launch);
//   * all warps then write the CTA's K range of x as three BF16 terms per value (hi, mid, lo;
//     exact), token t's terms in MMA rows 3t .. 3t + 2;
//   * two issuing threads run the MMAs (gated MLP: gate and up, one each; a single matrix:
//     alternate stages), each into its own TMEM accumulator;
//   * every warp then sums its tokens' term columns and scatters the partial sums over the
//     cluster (distributed shared memory, st.async completing on the owner's barrier): rank q
//     owns rows [q, q + 1) * 128 / ksplit of the tile, adds the ksplit partials in rank
//     order (deterministic) and writes the outputs (gated MLP: h = silu(gate) * up).
// Every wait is bounded (URB_ERR_TIMEOUT); every copy in flight lands before a CTA exits.
#include <cuda.h>

#include <algorithm>
#include <atomic>
#include <cstring>

#include "tc_common.cuh"
#include "urb_internal.cuh"
#include "urb_tc.cuh"

namespace urb {
namespace {

constexpr int kSpThreads = 256;
constexpr int kSpMaxTok = 32;                // tokens of one launch
constexpr int kSpTileBytes = 16384;          // a 128 x 64 BF16 box
constexpr int kSpStageCols = 64;
constexpr uint32_t kSpAccStride = 128;       // TMEM columns between the two accumulators
constexpr int kSpMaxStages = 8;              // K stages per CTA (all resident at once)
constexpr int kSpSmemMax = 226 * 1024;       // dynamic shared memory (the static part aside)

__host__ __device__ constexpr int sp_rows(int T) { return (3 * T + 15) & ~15; }  // MMA N
__host__ __device__ constexpr int sp_tpad(int T) { return (T + 3) & ~3; }
// Dynamic shared memory: weight boxes, activation stages, the cluster's partial sums; at
// least 80 KB, so that no more than two CTAs share an SM (each allocates 256 TMEM columns of
// the SM's 512: a third one would wait in its allocation while its cluster waits for it).
__host__ __device__ constexpr int sp_smem(int spc, int nmat, int T) {
    return spc * nmat * kSpTileBytes + spc * sp_rows(T) * 128 + 128 * sp_tpad(T) * nmat * 4 + 1024 < 80 * 1024
               ? 80 * 1024
               : spc * nmat * kSpTileBytes + spc * sp_rows(T) * 128 + 128 * sp_tpad(T) * nmat * 4 + 1024;
}

struct SpArgs {
    int mts, ks;              // 128-row tiles, K stages of 64 columns
    int ksplit;               // CTAs of a cluster (ranks), a divisor of 128
    int rows, cols, T;
    const float *x;           // [T, cols] (row stride x_stride)
    int x_stride;
    float *out;               // [T, rows] (row stride out_stride)
    int out_stride;
    int32_t *status;
};

__device__ __forceinline__ void set_status(int32_t *status, int code) {
    if (status) atomicCAS(status, 0, int32_t(code));
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t *bar, uint32_t parity, uint32_t limit) {
    for (uint32_t i = 0; i < limit; ++i) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok) : "r"(tc::smem_u32(bar)), "r"(parity) : "memory");
        if (ok) return true;
    }
    return false;
}

// BF16 (round to nearest even) of a finite f32, as the 16 high bits of its pattern.
__device__ __forceinline__ uint32_t bf16_rn(float v) {
    const uint32_t u = __float_as_uint(v);
    return (u + 0x7FFFu + ((u >> 16) & 1u)) >> 16;
}

__device__ __forceinline__ float silu_ieee(float v) { return v / (1.0f + expf(-v)); }

// NMAT = 2: gated MLP (map1 gate, map2 up; output h = silu(gate) * up).  NMAT = 1: product.
// The tensor maps are kernel parameters (the TMA unit reads them from the parameter space).
template <int NMAT>
__global__ void __launch_bounds__(kSpThreads, 1)
    k_split_bf16(SpArgs a, const __grid_constant__ CUtensorMap map1, const __grid_constant__ CUtensorMap map2) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ __align__(8) uint64_t a_full[kSpMaxStages], acc_full[2], mma_done[2], red_full;
    __shared__ uint32_t tmem_base;
    __shared__ int abort_flag, never;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kq = blockIdx.x, nq = a.ksplit;  // rank in the cluster (cluster dims (ksplit, 1, 1))
    const int mt = blockIdx.y;
    const int s0 = int((long long)kq * a.ks / nq), s1 = int((long long)(kq + 1) * a.ks / nq);
    const int S = s1 - s0;
    const int spc = (a.ks + nq - 1) / nq;
    const int T = a.T, NB = sp_rows(T), TP = sp_tpad(T), RPR = 128 / nq;
    uint8_t *wbox = smem;                                           // [spc][NMAT][16 KB]
    uint8_t *act = smem + size_t(spc) * NMAT * kSpTileBytes;       // [spc][NB rows][128 B]
    float *red = reinterpret_cast<float *>(act + size_t(spc) * NB * 128);  // [nq][RPR][NMAT][TP]

    if (warp == 0) {
        if (lane == 0) {
            for (int s = 0; s < kSpMaxStages; ++s) tc::mbar_init(&a_full[s], 1);
            for (int i = 0; i < 2; ++i) {
                tc::mbar_init(&acc_full[i], 1);
                tc::mbar_init(&mma_done[i], 1);
            }
            tc::mbar_init(&red_full, 1);
            tc::mbar_fence_init();
            abort_flag = 0;
            never = 0;
            // The weights need nothing from earlier kernels: every box of the CTA goes out now.
            for (int s = 0; s < S; ++s) {
                tc::mbar_arrive_expect_tx(&a_full[s], uint32_t(NMAT * kSpTileBytes));
                for (int m = 0; m < NMAT; ++m)
                    tc::tma_load_2d(wbox + size_t(s * NMAT + m) * kSpTileBytes, m ? &map2 : &map1,
                                    (s0 + s) * kSpStageCols, mt * 128, &a_full[s]);
            }
            // The cluster's partial sums of this rank's rows: RPR rows x NMAT x TP floats from
            // each of the nq ranks.
            tc::mbar_arrive_expect_tx(&red_full, uint32_t(nq * RPR * NMAT * TP * 4));
        }
        __syncwarp();
    } else if (warp == 1) {
        tc::tmem_alloc(&tmem_base, 256);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    // Peers store into this CTA's shared memory only after every rank has passed this point.
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
    pdl_launch_dependents();
    const uint32_t tbase = tmem_base;
    volatile int *abortp = &abort_flag;
    auto fail = [&]() {
        *abortp = 1;
        set_status(a.status, URB_ERR_TIMEOUT);
    };

    // x (possibly written by the kernel ahead) as three BF16 terms: item = (token, stage,
    // 16-byte chunk of 8 columns).
    pdl_wait();
    bool bad = false;
    for (int it = threadIdx.x; it < T * S * 8; it += kSpThreads) {
        const int ch = it & 7, s = (it >> 3) % S, t = (it >> 3) / S;
        const int c0 = (s0 + s) * kSpStageCols + ch * 8;
        const float *xp = a.x + size_t(t) * a.x_stride + c0;
        float r[8];
        if (c0 + 8 <= a.cols && (a.x_stride & 3) == 0) {
            const float4 v0 = __ldg(reinterpret_cast<const float4 *>(xp));
            const float4 v1 = __ldg(reinterpret_cast<const float4 *>(xp + 4));
            r[0] = v0.x; r[1] = v0.y; r[2] = v0.z; r[3] = v0.w;
            r[4] = v1.x; r[5] = v1.y; r[6] = v1.z; r[7] = v1.w;
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) r[i] = c0 + i < a.cols ? __ldg(xp + i) : 0.0f;
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            if (!isfinite(r[i])) {
                bad = true;
                r[i] = 0.0f;
            }
        }
        uint8_t *stage = act + size_t(s) * NB * 128;
#pragma unroll
        for (int j = 0; j < 3; ++j) {
            uint32_t q[4];
#pragma unroll
            for (int i = 0; i < 8; i += 2) {
                const uint32_t b0 = bf16_rn(r[i]), b1 = bf16_rn(r[i + 1]);
                r[i] -= __uint_as_float(b0 << 16);
                r[i + 1] -= __uint_as_float(b1 << 16);
                q[i >> 1] = b0 | (b1 << 16);
            }
            const int R = 3 * t + j;
            *reinterpret_cast<uint4 *>(stage + (R >> 3) * 1024 + (R & 7) * 128 + ((ch ^ (R & 7)) << 4)) =
                make_uint4(q[0], q[1], q[2], q[3]);
        }
    }
    if (bad) set_status(a.status, URB_ERR_NONFINITE);
    // The tensor cores (async proxy) read what the threads just wrote.
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");

    // Issuers: gated MLP: issuer i runs matrix i over every stage; product: issuer i runs
    // stages i, i + 2, ...  Accumulator i at TMEM column 128 i.
    if ((warp == 1 || warp == 2) && lane == 0) {
        const int me = warp - 1;
        const uint32_t acc = tbase + uint32_t(me) * kSpAccStride;
        bool any = false, ok = true;
        for (int s = NMAT == 2 ? 0 : me; s < S; s += NMAT == 2 ? 1 : 2) {
            if (!tc::mbar_wait(&a_full[s], 0, abortp)) { ok = false; break; }
            tc::fence_after_sync();
            const int m = NMAT == 2 ? me : 0;
            const uint64_t adesc = tc::sdesc_sw128(tc::smem_u32(wbox + size_t(s * NMAT + m) * kSpTileBytes));
            const uint64_t bdesc = tc::sdesc_sw128(tc::smem_u32(act + size_t(s) * NB * 128));
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
                tc::mma_bf16(acc, adesc + 2 * kk, bdesc + 2 * kk, tc::idesc_bf16(NB), any || kk > 0);
            any = true;
        }
        if (!ok) fail();
        if (any) tc::mma_commit(&acc_full[me]);
        tc::mma_commit(&mma_done[me]);
        tc::mbar_wait(&mma_done[me], 0, &never);
    }
    __syncwarp();

    // Epilogue, every warp: row 32 qtr + lane of the tile; warps 0-3 take tokens 0..15 (term
    // columns 0..47), warps 4-7 tokens 16..31 (columns 48..95).  part[m][i] = token 16 h + i's
    // term columns of accumulator m (product: both accumulators, issuer 0's first).
    {
        const int qtr = warp & 3, h = warp >> 2;
        const uint32_t lane_base = uint32_t(32 * qtr) << 16;
        const int used = NMAT == 2 ? (S > 0 ? 2 : 0) : min(S, 2);
        bool ok = true;
        for (int i = 0; i < used && ok; ++i)
            if (!tc::mbar_wait(&acc_full[i], 0, abortp)) { fail(); ok = false; }
        float part[NMAT][16];
#pragma unroll
        for (int m = 0; m < NMAT; ++m)
#pragma unroll
            for (int t = 0; t < 16; ++t) part[m][t] = 0.0f;
        const int nch = min(3, max(0, (NB - 48 * h) / 16));  // this half's 16-column chunks
        if (ok && used > 0 && nch > 0) {
            tc::fence_after_sync();
            uint32_t v[2][3][16];
#pragma unroll
            for (int i = 0; i < 2; ++i)
#pragma unroll
                for (int k = 0; k < 3; ++k)
                    if (i < used && k < nch)
                        tc::tmem_ld16(tbase + lane_base + uint32_t(i) * kSpAccStride + uint32_t(48 * h + 16 * k), v[i][k]);
            tc::wait_ld();
#pragma unroll
            for (int k = 0; k < 3; ++k) {
                if (k >= nch) break;
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    const int t = (16 * k + e) / 3;
                    part[0][t] += __uint_as_float(v[0][k][e]);
                    if (NMAT == 2) part[NMAT - 1][t] += __uint_as_float(v[1][k][e]);
                }
                if (NMAT == 1 && used > 1) {
#pragma unroll
                    for (int e = 0; e < 16; ++e) part[0][(16 * k + e) / 3] += __uint_as_float(v[1][k][e]);
                }
            }
        }
        // Scatter this row's partial sums (tokens 16 h + 4 t4 .. + 3) to the rank that owns the
        // row.  Every thread stores on every path, so every owner's wait completes.
        const int row = 32 * qtr + lane;
        const int owner = row / RPR, r = row - owner * RPR;
        uint32_t dst, bar;
        const float *slot = red + (size_t(kq) * RPR + r) * NMAT * TP;
        asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(dst) : "r"(tc::smem_u32(slot)), "r"(owner));
        asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(bar) : "r"(tc::smem_u32(&red_full)), "r"(owner));
#pragma unroll
        for (int m = 0; m < NMAT; ++m)
#pragma unroll
            for (int t4 = 0; t4 < 4; ++t4) {
                const int t = 16 * h + 4 * t4;
                if (t >= TP) break;
                asm volatile(
                    "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];"
                    ::"r"(dst + uint32_t((m * TP + t) * 4)), "f"(part[m][4 * t4]), "f"(part[m][4 * t4 + 1]),
                      "f"(part[m][4 * t4 + 2]), "f"(part[m][4 * t4 + 3]), "r"(bar)
                    : "memory");
            }
    }

    // Owners: this rank's rows [kq * RPR, +RPR) of the tile, the partials added in rank order.
    if (!mbar_wait_cluster(&red_full, 0, 1u << 26)) fail();
    for (int it = threadIdx.x; it < RPR * T; it += kSpThreads) {
        const int r = it / T, t = it - r * T;
        float v[NMAT];
#pragma unroll
        for (int m = 0; m < NMAT; ++m) {
            float s = 0.0f;
            for (int q = 0; q < nq; ++q) s += red[((size_t(q) * RPR + r) * NMAT + m) * TP + t];
            v[m] = s;
        }
        const long long grow = (long long)mt * 128 + kq * RPR + r;
        if (grow < a.rows)
            a.out[size_t(t) * a.out_stride + grow] = NMAT == 2 ? silu_ieee(v[0]) * v[NMAT - 1] : v[0];
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tbase, 256);
    }
}

// Clusters of `ksplit` CTAs of this kernel that can be resident at once on the current device.
template <typename K>
int resident_clusters(K kern, int ksplit, int smem) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ksplit, 1, 1);
    cfg.blockDim = dim3(kSpThreads);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = ksplit;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

constexpr int kSpMaxDevices = 64;
std::atomic<bool> g_sp_attrs[kSpMaxDevices][2];
std::atomic<int> g_sp_resident[kSpMaxDevices][2][5][kSpMaxStages + 1][kSpMaxTok / 4 + 1];

// One launch over rows [0, rows) of T tokens.  K split: the largest cluster (16, 8, ... ranks,
// divisors of 128) that keeps every rank at least one stage, holds at most kSpMaxStages stages
// per CTA in shared memory, and keeps all the launch's clusters resident at once.
template <int NMAT>
int launch_split(Ctx *ctx, const Mat *m1, const Mat *m2, int mts, int ks, int rows, int cols,
                 const float *d_x, int x_stride, int T, float *d_out, int out_stride,
                 int32_t *d_status, cudaStream_t st) {
    auto kern = k_split_bf16<NMAT>;
    const int dev = ctx->device;
    const bool cached = dev >= 0 && dev < kSpMaxDevices;
    if (!cached || !g_sp_attrs[dev][NMAT - 1].load()) {
        URB_CUDA(ctx, cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSpSmemMax));
        URB_CUDA(ctx, cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
        if (cached) g_sp_attrs[dev][NMAT - 1].store(true);
    }
    int chosen = 0;
    for (int li = 0, ksp = 16; ksp >= 1; ksp >>= 1, ++li) {
        if (ksp > ks) continue;
        const int spc = (ks + ksp - 1) / ksp;
        if (spc > kSpMaxStages || sp_smem(spc, NMAT, T) > kSpSmemMax) break;
        int res;
        if (cached) {
            std::atomic<int> &c = g_sp_resident[dev][NMAT - 1][li][spc][(T + 3) / 4];
            res = c.load(std::memory_order_relaxed);
            if (res <= 0) {
                res = resident_clusters(kern, ksp, sp_smem(spc, NMAT, T));
                c.store(res, std::memory_order_relaxed);
            }
        } else {
            res = resident_clusters(kern, ksp, sp_smem(spc, NMAT, T));
        }
        if (res >= mts) {
            chosen = ksp;
            break;
        }
    }
    if (!chosen) return URB_ERR_UNSUPPORTED;
    const int spc = (ks + chosen - 1) / chosen;
    SpArgs a{};
    a.mts = mts;
    a.ks = ks;
    a.ksplit = chosen;
    a.rows = rows;
    a.cols = cols;
    a.T = T;
    a.x = d_x;
    a.x_stride = x_stride;
    a.out = d_out;
    a.out_stride = out_stride;
    a.status = d_status;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = chosen;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cm = {};
    cm.gridDim = dim3(unsigned(chosen), unsigned(mts), 1);
    cm.blockDim = dim3(kSpThreads);
    cm.dynamicSmemBytes = sp_smem(spc, NMAT, T);
    cm.stream = st;
    cm.attrs = at;
    cm.numAttrs = 2;
    CUtensorMap t1, t2;
    std::memcpy(&t1, m1->tc_map_host, sizeof(t1));
    std::memcpy(&t2, (m2 ? m2 : m1)->tc_map_host, sizeof(t2));
    URB_CUDA(ctx, cudaLaunchKernelEx(&cm, kern, a, t1, t2));
    return URB_OK;
}

bool split_ok(const Mat *m) { return m->format == URB_FMT_BF16 && m->tc_map; }

}  // namespace

bool split_tc_applies(const Mat *m, size_t T) { return split_ok(m) && T >= 1 && T <= size_t(kSpMaxTok); }

int split_tc_product(Ctx *ctx, const Mat *m, const float *d_x, int T, float *d_y, int32_t *d_status,
                     cudaStream_t st) {
    if (!split_tc_applies(m, size_t(T))) return URB_ERR_UNSUPPORTED;
    prof_begin(ctx, URB_K_PRODUCT, st);
    const int rc = launch_split<1>(ctx, m, nullptr, m->tc_mts, m->tc_ks, int(m->rows), int(m->cols),
                                   d_x, int(m->cols), T, d_y, int(m->rows), d_status, st);
    prof_end(ctx, st);
    return rc;
}

int split_tc_mlp(Ctx *ctx, const Mat *g, const Mat *u, const Mat *d, const float *d_x, int T,
                 float *d_h, float *d_out, int32_t *d_status, cudaStream_t st) {
    if (!split_tc_applies(g, size_t(T)) || !split_ok(u) || !split_ok(d) || u->rows != g->rows ||
        u->cols != g->cols || d->cols != g->rows)
        return URB_ERR_UNSUPPORTED;
    prof_begin(ctx, URB_K_GATE_UP, st);
    int rc = launch_split<2>(ctx, g, u, g->tc_mts, g->tc_ks, int(g->rows), int(g->cols),
                             d_x, int(g->cols), T, d_h, int(g->rows), d_status, st);
    prof_end(ctx, st);
    if (rc) return rc;
    prof_begin(ctx, URB_K_DOWN, st);
    rc = launch_split<1>(ctx, d, nullptr, d->tc_mts, d->tc_ks, int(d->rows), int(d->cols), d_h,
                         int(d->cols), T, d_out, int(d->rows), d_status, st);
    prof_end(ctx, st);
    return rc;
}

}  // namespace urb
