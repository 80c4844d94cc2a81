// numerics.cu — the E4M3 activation simulation as a standalone device operation
// (simulate_e4m3_activation, src/math/mxfp.rs:82-115): one thread per block of `block` values.
#include <cmath>

#include "numerics.cuh"
#include "urb_internal.cuh"

namespace urb {
namespace {

__global__ void k_sim_e4m3(const float *x, size_t n, size_t block, float *out) {
    const size_t b = blockIdx.x * size_t(blockDim.x) + threadIdx.x;
    const size_t begin = b * block;
    if (begin >= n) return;
    const size_t end = begin + block < n ? begin + block : n;
    float m = 0.0f;
    for (size_t i = begin; i < end; ++i) m = fmaxf(m, fabsf(x[i]));
    const float scale = num_e4m3_scale(m);
    for (size_t i = begin; i < end; ++i) out[i] = num_e4m3_sim(x[i], scale);
}

}  // namespace
}  // namespace urb

using namespace urb;

extern "C" int urb_simulate_e4m3_activation(urb_ctx *ctx, const float *x, size_t n, size_t block,
                                            float *out) {
    if (!ctx || (n && (!x || !out))) return URB_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    cudaSetDevice(ctx->device);
    // Validation order of mxfp.rs:95-101: shape, then finiteness.
    if (n == 0 || block == 0)
        return set_error(ctx, URB_ERR_SHAPE, "activation and block size must be non-zero");
    for (size_t i = 0; i < n; ++i)
        if (!std::isfinite(x[i])) return set_error(ctx, URB_ERR_NONFINITE, "activation is not finite");
    cudaStream_t st = ctx->stream;
    float *d = nullptr;
    URB_CUDA(ctx, cudaMallocAsync(&d, 2 * n * sizeof(float), st));
    URB_CUDA(ctx, cudaMemcpyAsync(d, x, n * sizeof(float), cudaMemcpyDefault, st));
    const size_t blocks = (n + block - 1) / block;
    k_sim_e4m3<<<unsigned((blocks + 255) / 256), 256, 0, st>>>(d, n, block, d + n);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaMemcpyAsync(out, d + n, n * sizeof(float), cudaMemcpyDefault, st);
    cudaFreeAsync(d, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "simulate_e4m3_activation");
    return URB_OK;
}
