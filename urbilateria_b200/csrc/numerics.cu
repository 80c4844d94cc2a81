// numerics.cu — checkpoint numerics as standalone device operations: the E4M3 activation
// simulations (simulate_e4m3_activation, src/math/mxfp.rs:82-115, and the fine-grained
// simulate_finegrained_e4m3_activation, :122-149; one thread per block of `block` values) and
// the Qwen3.6 BF16 linear (qwen3_8/math.rs:10-26 over src/model/bf16.rs:591-613).
#include <cmath>

#include "numerics.cuh"
#include "urb_internal.cuh"

namespace urb {
namespace {

__global__ void k_sim_e4m3(const float *x, size_t n, size_t block, float *out, int fine) {
    const size_t b = blockIdx.x * size_t(blockDim.x) + threadIdx.x;
    const size_t begin = b * block;
    if (begin >= n) return;
    const size_t end = begin + block < n ? begin + block : n;
    float m = 0.0f;
    for (size_t i = begin; i < end; ++i) m = fmaxf(m, fabsf(x[i]));
    if (fine) {
        for (size_t i = begin; i < end; ++i) out[i] = num_e4m3_sim_fine(x[i], m);
        return;
    }
    const float scale = num_e4m3_scale(m);
    for (size_t i = begin; i < end; ++i) out[i] = num_e4m3_sim(x[i], scale);
}

int simulate(urb_ctx *ctx, const float *x, size_t n, size_t block, float *out, int fine) {
    if (!ctx || (n && (!x || !out))) return URB_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    cudaSetDevice(ctx->device);
    // Validation order of mxfp.rs:95-101 and :126-132: shape, then finiteness.
    if (n == 0 || block == 0)
        return set_error(ctx, URB_ERR_SHAPE, "activation and block size must be non-zero");
    for (size_t i = 0; i < n; ++i)
        if (!std::isfinite(x[i])) return set_error(ctx, URB_ERR_NONFINITE, "activation is not finite");
    cudaStream_t st = ctx->stream;
    float *d = nullptr;
    URB_CUDA(ctx, cudaMallocAsync(&d, 2 * n * sizeof(float), st));
    URB_CUDA(ctx, cudaMemcpyAsync(d, x, n * sizeof(float), cudaMemcpyDefault, st));
    const size_t blocks = (n + block - 1) / block;
    k_sim_e4m3<<<unsigned((blocks + 255) / 256), 256, 0, st>>>(d, n, block, d + n, fine);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaMemcpyAsync(out, d + n, n * sizeof(float), cudaMemcpyDefault, st);
    cudaFreeAsync(d, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "simulate_e4m3_activation");
    return URB_OK;
}

}  // namespace
}  // namespace urb

using namespace urb;

extern "C" int urb_simulate_e4m3_activation(urb_ctx *ctx, const float *x, size_t n, size_t block,
                                            float *out) {
    return simulate(ctx, x, n, block, out, 0);
}

extern "C" int urb_simulate_finegrained_e4m3_activation(urb_ctx *ctx, const float *x, size_t n,
                                                        size_t block, float *out) {
    return simulate(ctx, x, n, block, out, 1);
}

extern "C" int urb_linear_bf16_fp32_lanes(urb_ctx *ctx, const urb_mat *m, const float *x,
                                          size_t tokens, float *out) {
    if (!ctx || !m || (tokens && (!x || !out))) return URB_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    cudaSetDevice(ctx->device);
    if (m->format != URB_FMT_BF16 || !m->raw_values)
        return set_error(ctx, URB_ERR_UNSUPPORTED, "the FP32-lane linear takes a BF16 matrix");
    if (tokens == 0) return URB_OK;
    const size_t R = m->rows, C = m->cols;
    cudaStream_t st = ctx->stream;
    float *d = nullptr;
    URB_CUDA(ctx, cudaMemsetAsync(ctx->d_status, 0, 4, st));
    URB_CUDA(ctx, cudaMallocAsync(&d, (tokens * C + tokens * R) * sizeof(float), st));
    URB_CUDA(ctx, cudaMemcpyAsync(d, x, tokens * C * sizeof(float), cudaMemcpyDefault, st));
    int rc = launch_router_bf16_lanes(static_cast<const uint16_t *>(m->raw_values), int(R), nullptr,
                                      d, int(tokens), int(C), d + tokens * C, nullptr,
                                      ctx->d_status, st);
    int32_t status = 0;
    cudaError_t e = rc ? cudaGetLastError() : cudaSuccess;
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(out, d + tokens * C, tokens * R * sizeof(float), cudaMemcpyDefault, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(&status, ctx->d_status, 4, cudaMemcpyDeviceToHost, st);
    cudaFreeAsync(d, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (rc || e != cudaSuccess) return cuda_fail(ctx, e, "BF16 linear");
    if (status) return set_error(ctx, status, "BF16 linear output is not finite");
    return URB_OK;
}
