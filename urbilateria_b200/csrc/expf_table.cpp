// expf_table.cpp — embeds the libm exception tables generated at build time by
// gen_expf_table.c (URB_EXPF_TABLE_PATH) and gen_log1pf_table.c (URB_LOG1PF_TABLE_PATH) and
// uploads them, each with its bucket index over the top 20 input bits, to the device of a
// context.
#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

#include "urb_internal.cuh"

#ifndef URB_EXPF_TABLE_PATH
#error "URB_EXPF_TABLE_PATH must name the generated expf table"
#endif
#ifndef URB_LOG1PF_TABLE_PATH
#error "URB_LOG1PF_TABLE_PATH must name the generated log1pf table"
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
        ".balign 16\n"
        ".global urb_log1pf_table_begin\n"
        "urb_log1pf_table_begin:\n"
        ".incbin \"" URB_STR(URB_LOG1PF_TABLE_PATH) "\"\n"
        ".global urb_log1pf_table_end\n"
        "urb_log1pf_table_end:\n"
        ".previous\n");

extern "C" const uint32_t urb_expf_table_begin[];
extern "C" const uint32_t urb_expf_table_end[];
extern "C" const uint32_t urb_log1pf_table_begin[];
extern "C" const uint32_t urb_log1pf_table_end[];

namespace urb {
namespace {

// Uploads one (key, value) table with its bucket index; *base receives the allocation
// (keys at +0, values at +n, index at +2n).
int upload_table(Ctx *ctx, const uint32_t *begin, const uint32_t *end, uint32_t **base,
                 int *count) {
    size_t words = size_t(end - begin);
    size_t n = words / 2;
    constexpr uint32_t kBuckets = 1u << 20;  // top 20 bits of the input
    std::vector<uint32_t> keys(n), vals(n), index(kBuckets + 1, 0);
    for (size_t i = 0; i < n; ++i) {
        keys[i] = begin[2 * i];
        vals[i] = begin[2 * i + 1];
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
    *base = d;
    *count = int(n);
    return URB_OK;
}

}  // namespace

int expf_table_init(Ctx *ctx) {
    uint32_t *d = nullptr;
    int n = 0;
    int rc = upload_table(ctx, urb_expf_table_begin, urb_expf_table_end, &d, &n);
    if (rc) return rc;
    ctx->expf_keys = d;
    ctx->expf_vals = d + n;
    ctx->expf_index = d + 2 * size_t(n);
    ctx->expf_count = n;
    rc = upload_table(ctx, urb_log1pf_table_begin, urb_log1pf_table_end, &d, &n);
    if (rc) return rc;
    ctx->log1pf_keys = d;
    ctx->log1pf_vals = d + n;
    ctx->log1pf_index = d + 2 * size_t(n);
    return URB_OK;
}

}  // namespace urb
