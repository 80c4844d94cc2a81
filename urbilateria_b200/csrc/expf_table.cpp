// expf_table.cpp — embeds the libm-expf exception table generated at build time by
// gen_expf_table.c (URB_EXPF_TABLE_PATH) and uploads it, with its 16-bit bucket index, to
// the device of a context.
#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

#include "urb_internal.cuh"

#ifndef URB_EXPF_TABLE_PATH
#error "URB_EXPF_TABLE_PATH must name the generated expf table"
#endif

#define URB_STR2(x) #x
#define URB_STR(x) URB_STR2(x)

__asm__(".section .rodata\n"
        ".balign 16\n"
        ".global urb_expf_table_begin\n"
        "urb_expf_table_begin:\n"
        ".incbin \"" URB_STR(URB_EXPF_TABLE_PATH) "\"\n"
        ".global urb_expf_table_end\n"
        "urb_expf_table_end:\n"
        ".previous\n");

extern "C" const uint32_t urb_expf_table_begin[];
extern "C" const uint32_t urb_expf_table_end[];

namespace urb {

int expf_table_init(Ctx *ctx) {
    size_t words = size_t(urb_expf_table_end - urb_expf_table_begin);
    size_t n = words / 2;
    constexpr uint32_t kBuckets = 1u << 20;  // top 20 bits of the input
    std::vector<uint32_t> keys(n), vals(n), index(kBuckets + 1, 0);
    for (size_t i = 0; i < n; ++i) {
        keys[i] = urb_expf_table_begin[2 * i];
        vals[i] = urb_expf_table_begin[2 * i + 1];
    }
    // index[b] = first entry whose key >> 12 >= b.
    size_t j = 0;
    for (uint32_t b = 0; b <= kBuckets; ++b) {
        while (j < n && (keys[j] >> 12) < b) ++j;
        index[b] = uint32_t(j);
    }
    uint32_t *d = nullptr;
    size_t bytes = (2 * n + kBuckets + 1) * sizeof(uint32_t);
    URB_CUDA(ctx, cudaMalloc(&d, bytes));
    URB_CUDA(ctx, cudaMemcpy(d, keys.data(), n * 4, cudaMemcpyHostToDevice));
    URB_CUDA(ctx, cudaMemcpy(d + n, vals.data(), n * 4, cudaMemcpyHostToDevice));
    URB_CUDA(ctx, cudaMemcpy(d + 2 * n, index.data(), (kBuckets + 1) * 4, cudaMemcpyHostToDevice));
    ctx->expf_keys = d;
    ctx->expf_vals = d + n;
    ctx->expf_index = d + 2 * n;
    ctx->expf_count = int(n);
    return URB_OK;
}

}  // namespace urb
