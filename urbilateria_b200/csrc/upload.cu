// upload.cu — device residency for weight matrices: payload validation (the checks of the
// reference constructors) and the repack into the tiled layout described in urb_internal.cuh.
#include <cuda.h>

#include <cstring>
#include <mutex>

#include "urb_internal.cuh"
#include "urb_tc.cuh"

namespace urb {
namespace {

// Flags written by the validation kernels.
constexpr int kFlagInvalidScale = 1;  // an E8M0 0xFF byte (mxfp.rs:1431-1435, :422-424)
constexpr int kFlagNanE4m3 = 2;       // an E4M3 NaN code 0x7F/0xFF (mxfp.rs:419-421)
constexpr int kFlagWide = 4;          // a row's scales span more than f16 can hold exactly
constexpr int kFlagBadF32Scale = 8;   // an INT scale that is not finite and positive (quant.rs:119-123, 384-389)

__global__ void k_scan_fscales(const float *scales, size_t n, int *flags) {
    size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x;
    size_t stride = size_t(gridDim.x) * blockDim.x;
    bool bad = false;
    for (; i < n; i += stride) bad |= !(isfinite(scales[i]) && scales[i] > 0.0f);
    if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) atomicOr(flags, kFlagBadF32Scale);
}

// Largest decoded magnitude exponent (relative to scale 2^0) and the f16 window per format:
// MXFP4 values 0.5..6 -> need 2^(s-127-E0) in [2^-23, 2^13];
// MXFP8 values 2^-9..448 -> need 2^(s-127-E0) in [2^-15, 2^7].
__host__ __device__ constexpr int fmt_top(int fmt) { return fmt == URB_FMT_MXFP4 ? 13 : 7; }
__host__ __device__ constexpr int fmt_window(int fmt) { return fmt == URB_FMT_MXFP4 ? 36 : 22; }

__global__ void k_scan_e4m3(const uint8_t *values, size_t n, int *flags) {
    size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x;
    size_t stride = size_t(gridDim.x) * blockDim.x;
    bool bad = false;
    for (; i < n; i += stride) bad |= (values[i] & 0x7f) == 0x7f;
    if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) atomicOr(flags, kFlagNanE4m3);
}

// One warp per (padded) row: scale range of the row -> row exponent offset, 0xFF detection.
__global__ void k_scan_scales(const uint8_t *scales, int fmt, size_t rows, size_t rows_pad,
                              size_t scale_cols, size_t block_rows, int8_t *row_exp,
                              int *flags) {
    size_t row = blockIdx.x * size_t(blockDim.x / 32) + threadIdx.x / 32;
    int lane = threadIdx.x & 31;
    if (row >= rows_pad) return;
    if (row >= rows) {
        if (lane == 0) row_exp[row] = 0;
        return;
    }
    const uint8_t *s = scales + (row / block_rows) * scale_cols;
    int smax = 0, smin = 255;
    bool bad = false;
    for (size_t c = lane; c < scale_cols; c += 32) {
        int v = s[c];
        bad |= v == 0xff;
        smax = max(smax, v);
        smin = min(smin, v);
    }
    for (int o = 16; o > 0; o >>= 1) {
        smax = max(smax, __shfl_xor_sync(0xffffffffu, smax, o));
        smin = min(smin, __shfl_xor_sync(0xffffffffu, smin, o));
    }
    bad = __any_sync(0xffffffffu, bad);
    if (lane == 0) {
        int e0 = smax - 127 - fmt_top(fmt);
        row_exp[row] = int8_t(max(-128, min(127, e0)));
        int f = 0;
        if (bad) f |= kFlagInvalidScale;
        if (smax - smin > fmt_window(fmt) || e0 < -128 || e0 > 127) f |= kFlagWide;
        if (f) atomicOr(flags, f);
    }
}

// One thread per (row block, slice, lane): writes that lane's slot of the tile.
template <int FMT>
__global__ void k_repack(const uint8_t *values, const uint8_t *scales, size_t rows, size_t cols,
                         size_t scale_cols, size_t block_rows, size_t block_cols, int rbs,
                         int kslices, uint8_t *tiles) {
    size_t id = blockIdx.x * size_t(blockDim.x) + threadIdx.x;
    size_t total = size_t(rbs) * kslices * 32;
    if (id >= total) return;
    int lane = int(id & 31);
    size_t tile = id >> 5;
    int s = int(tile % kslices);
    size_t rb = tile / kslices;
    int g = lane >> 2, q = lane & 3;
    size_t col0 = size_t(s) * 128 + size_t(q) * 32;  // first column of this lane's group
    uint8_t *dst = tiles + tile * tile_bytes(FMT);
    constexpr int half = tile_payload_bytes(FMT) / 64;  // bytes per row per lane
    for (int h = 0; h < 2; ++h) {
        size_t row = rb * 16 + g + 8 * h;
        uint8_t buf[half];
        for (int i = 0; i < half; ++i) buf[i] = 0;
        uint8_t scale = 127;
        if (row < rows) {
            if (FMT == URB_FMT_MXFP4) {
                size_t row_bytes = (cols + 1) / 2;
                const uint8_t *src = values + row * row_bytes;
                for (int i = 0; i < 16; ++i) {
                    size_t c = col0 + 2 * i;  // low nibble column
                    uint8_t lo = c < cols ? (src[c / 2] & 0x0f) : 0;
                    uint8_t hi = c + 1 < cols ? (src[c / 2] >> 4) : 0;
                    buf[i] = uint8_t(lo | (hi << 4));
                }
                if (col0 < cols) scale = scales[row * scale_cols + col0 / 32];
            } else if (FMT == URB_FMT_MXFP8) {
                const uint8_t *src = values + row * cols;
                for (int i = 0; i < 32; ++i) {
                    size_t c = col0 + i;
                    buf[i] = c < cols ? src[c] : 0;
                }
                if (col0 < cols) scale = scales[(row / block_rows) * scale_cols + col0 / block_cols];
            } else {  // BF16: two bytes per element
                const uint16_t *src = reinterpret_cast<const uint16_t *>(values) + row * cols;
                for (int i = 0; i < 32; ++i) {
                    size_t c = col0 + i;
                    uint16_t v = c < cols ? src[c] : 0;
                    buf[2 * i] = uint8_t(v & 0xff);
                    buf[2 * i + 1] = uint8_t(v >> 8);
                }
            }
        }
        uint8_t *d = dst + lane * (2 * half) + h * half;
        for (int i = 0; i < half; ++i) d[i] = buf[i];
        if (FMT == URB_FMT_MXFP4 || FMT == URB_FMT_MXFP8)
            dst[tile_payload_bytes(FMT) + 2 * lane + h] = scale;
    }
}

// The mma.sync tiles of an MX matrix from its tcgen05 tiles (every byte the same as k_repack
// writes from the reference layout, padding included): one thread per (tile, lane).
template <int FMT>
__global__ void k_bs_to_mma(const uint8_t *bs, int mts, int rbs, int kslices, uint8_t *tiles) {
    const size_t id = blockIdx.x * size_t(blockDim.x) + threadIdx.x;
    if (id >= size_t(rbs) * kslices * 32) return;
    const int lane = int(id & 31);
    const size_t tile = id >> 5;
    const int s = int(tile % kslices);
    const size_t rb = tile / kslices;
    const int g = lane >> 2, q = lane & 3;
    const int col0 = s * 128 + q * 32;                       // the lane's 32-column group
    constexpr int SC = bs_stage_cols(FMT), TB = bs_tile_bytes(FMT);
    constexpr int half = tile_payload_bytes(FMT) / 64;       // bytes per row per lane
    uint8_t *dst = tiles + tile * tile_bytes(FMT);
    for (int h = 0; h < 2; ++h) {
        const size_t row = rb * 16 + g + 8 * h;
        const int rr = int(row & 127), kb = (col0 % SC) / 32;
        const uint8_t *t = bs + (size_t(col0 / SC) * mts + row / 128) * TB;
        const uint8_t *rowp = t + (rr >> 3) * 1024 + (rr & 7) * 128;
        uint8_t *d = dst + lane * (2 * half) + h * half;
        if (FMT == URB_FMT_MXFP4) {
            *reinterpret_cast<uint4 *>(d) = *reinterpret_cast<const uint4 *>(rowp + ((kb ^ (rr & 7)) << 4));
        } else {
            *reinterpret_cast<uint4 *>(d) = *reinterpret_cast<const uint4 *>(rowp + (((2 * kb) ^ (rr & 7)) << 4));
            *reinterpret_cast<uint4 *>(d + 16) =
                *reinterpret_cast<const uint4 *>(rowp + (((2 * kb + 1) ^ (rr & 7)) << 4));
        }
        dst[tile_payload_bytes(FMT) + 2 * lane + h] =
            t[16384 + 512 * (kb >> 2) + 16 * (rr & 31) + 4 * (rr >> 5) + (kb & 3)];
    }
}

size_t div_ceil(size_t a, size_t b) { return (a + b - 1) / b; }

std::mutex g_mma_tiles_mu;

// cuTensorMapEncodeTiled from the driver, resolved once through the runtime.
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled() {
    static const EncodeTiledFn fn = [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<EncodeTiledFn>(p);
    }();
    return fn;
}

// The BF16 matrix's tensor map for the grouped tcgen05 passes: 2-D [rows, cols] bf16 over the
// row-major copy, boxes of 64 columns (128 bytes, the swizzle span) x 128 rows, 128-byte
// swizzle (the canonical K-major layout the MMA descriptors name), zero fill past the edges.
// The row pitch must be a multiple of 16 bytes (cols % 8 == 0); other shapes keep no map.
int make_bf16_tile_map(Ctx *ctx, Mat *m, cudaStream_t st) {
    if (m->cols % 8 != 0 || m->rows == 0 || m->cols == 0) return URB_OK;
    const EncodeTiledFn enc = encode_tiled();
    if (!enc) return URB_OK;
    CUtensorMap map;
    const cuuint64_t dims[2] = {cuuint64_t(m->cols), cuuint64_t(m->rows)};
    const cuuint64_t strides[1] = {cuuint64_t(m->cols) * 2};
    const cuuint32_t box[2] = {64, 128};
    const cuuint32_t elem[2] = {1, 1};
    if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, m->raw_values, dims, strides, box, elem,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return URB_OK;
    static_assert(sizeof(CUtensorMap) == sizeof(m->tc_map_host), "tensor map size");
    std::memcpy(m->tc_map_host, &map, sizeof(CUtensorMap));
    URB_CUDA(ctx, cudaMallocAsync(&m->tc_map, sizeof(CUtensorMap), st));
    URB_CUDA(ctx, cudaMemcpyAsync(m->tc_map, &map, sizeof(CUtensorMap), cudaMemcpyHostToDevice, st));
    m->tc_mts = int(div_ceil(m->rows, 128));
    m->tc_ks = int(div_ceil(m->cols, size_t(bs_stage_cols(URB_FMT_BF16))));
    return URB_OK;
}

}  // namespace

int ensure_mma_tiles(Ctx *ctx, const Mat *cm, cudaStream_t st) {
    Mat *m = const_cast<Mat *>(cm);
    std::lock_guard<std::mutex> lk(g_mma_tiles_mu);
    if (m->tiles || !m->tiled) return URB_OK;
    if (!m->tc_tiles || (m->format != URB_FMT_MXFP4 && m->format != URB_FMT_MXFP8))
        return set_error(ctx, URB_ERR_UNSUPPORTED, "no tiles to build the mma.sync layout from");
    uint8_t *t = nullptr;
    const size_t total = size_t(m->rbs) * m->kslices * tile_bytes(m->format);
    URB_CUDA(ctx, cudaMallocAsync((void **)&t, total, st));
    const size_t threads = size_t(m->rbs) * m->kslices * 32;
    const unsigned blocks = unsigned(div_ceil(threads, 256));
    if (m->format == URB_FMT_MXFP4)
        k_bs_to_mma<URB_FMT_MXFP4><<<blocks, 256, 0, st>>>(m->tc_tiles, m->tc_mts, m->rbs, m->kslices, t);
    else
        k_bs_to_mma<URB_FMT_MXFP8><<<blocks, 256, 0, st>>>(m->tc_tiles, m->tc_mts, m->rbs, m->kslices, t);
    URB_CUDA(ctx, cudaGetLastError());
    // Other streams may read the tiles next: they are complete before the pointer is published.
    URB_CUDA(ctx, cudaStreamSynchronize(st));
    m->tiles = t;
    return URB_OK;
}

int upload_matrix(Ctx *ctx, Mat *m, const void *values, const uint8_t *scales) {
    cudaStream_t st = ctx->stream;
    size_t value_bytes = 0, scale_bytes = 0, scale_cols = 0;
    switch (m->format) {
    case URB_FMT_MXFP4:
        value_bytes = m->rows * div_ceil(m->cols, 2);
        scale_cols = div_ceil(m->cols, m->group_size);
        scale_bytes = m->rows * scale_cols;
        break;
    case URB_FMT_MXFP8:
        value_bytes = m->rows * m->cols;
        scale_cols = div_ceil(m->cols, m->block_cols);
        scale_bytes = div_ceil(m->rows, m->block_rows) * scale_cols;
        break;
    case URB_FMT_BF16:
        value_bytes = m->rows * m->cols * 2;
        break;
    case URB_FMT_F32:
        value_bytes = m->rows * m->cols * 4;
        break;
    case URB_FMT_INT8:  // quant.rs:555-559 resident_bytes: payload + 4 bytes per scale
        value_bytes = m->rows * m->cols;
        scale_bytes = m->rows * sizeof(float);
        break;
    case URB_FMT_INT4:  // quant.rs:285-289
        value_bytes = m->rows * div_ceil(m->cols, 2);
        scale_bytes = m->rows * div_ceil(m->cols, m->group_size) * sizeof(float);
        break;
    }
    m->resident_bytes = value_bytes + scale_bytes;

    // Stage the reference-layout payload on the device (host or device source pointers).
    URB_CUDA(ctx, cudaMallocAsync(&m->raw_values, value_bytes, st));
    URB_CUDA(ctx, cudaMemcpyAsync(m->raw_values, values, value_bytes, cudaMemcpyDefault, st));
    if (scale_bytes) {
        URB_CUDA(ctx, cudaMallocAsync((void **)&m->raw_scales, scale_bytes, st));
        URB_CUDA(ctx, cudaMemcpyAsync(m->raw_scales, scales, scale_bytes, cudaMemcpyDefault, st));
    }

    int *d_flags = nullptr;
    URB_CUDA(ctx, cudaMallocAsync((void **)&d_flags, sizeof(int), st));
    URB_CUDA(ctx, cudaMemsetAsync(d_flags, 0, sizeof(int), st));

    bool mx = m->format == URB_FMT_MXFP4 || m->format == URB_FMT_MXFP8;
    // Tiled fast path eligibility by shape: MXFP4 with 32-column groups; MXFP8 whose scale
    // blocks are whole 32-column groups; BF16 always.  F32 stays on the generic path.
    bool tiled_shape = (m->format == URB_FMT_MXFP4 && m->group_size == 32) ||
                       (m->format == URB_FMT_MXFP8 && m->block_cols % 32 == 0) ||
                       (m->format == URB_FMT_BF16);
    m->rbs = int(div_ceil(m->rows, 16));
    m->kslices = int(div_ceil(m->cols, 128));
    // Row exponents cover both layouts: 16-row tiles (mma.sync) and 128-row tiles (tcgen05).
    size_t rows_pad = div_ceil(m->rows, 128) * 128;

    if (is_int_format(m->format))
        k_scan_fscales<<<256, 256, 0, st>>>(reinterpret_cast<const float *>(m->raw_scales),
                                            scale_bytes / sizeof(float), d_flags);
    if (m->format == URB_FMT_MXFP8) {
        k_scan_e4m3<<<1024, 256, 0, st>>>(static_cast<const uint8_t *>(m->raw_values),
                                          value_bytes, d_flags);
    }
    if (mx) {
        URB_CUDA(ctx, cudaMallocAsync((void **)&m->row_exp, rows_pad, st));
        size_t block_rows = m->format == URB_FMT_MXFP8 ? m->block_rows : 1;
        int warps = 8;
        k_scan_scales<<<unsigned(div_ceil(rows_pad, warps)), warps * 32, 0, st>>>(
            m->raw_scales, m->format, m->rows, rows_pad, scale_cols, block_rows, m->row_exp,
            d_flags);
    } else if (m->format == URB_FMT_BF16) {
        URB_CUDA(ctx, cudaMallocAsync((void **)&m->row_exp, rows_pad, st));
        URB_CUDA(ctx, cudaMemsetAsync(m->row_exp, 0, rows_pad, st));
    }
    URB_CUDA(ctx, cudaGetLastError());
    int flags = 0;
    URB_CUDA(ctx, cudaMemcpyAsync(&flags, d_flags, sizeof(int), cudaMemcpyDeviceToHost, st));
    URB_CUDA(ctx, cudaStreamSynchronize(st));
    URB_CUDA(ctx, cudaFreeAsync(d_flags, st));
    // Reference validation order: E4M3 NaN before scales (mxfp.rs:419-424).
    if (flags & kFlagNanE4m3) return set_error(ctx, URB_ERR_NONFINITE, "E4M3 payload contains NaN codes");
    if (flags & kFlagInvalidScale) return set_error(ctx, URB_ERR_INVALID_SCALE, "E8M0 scale byte 0xff is NaN");
    if (flags & kFlagBadF32Scale) return set_error(ctx, URB_ERR_NONFINITE, "INT scale is not finite and positive");

    // Block-scaled tensor-core layout: any MX matrix whose scale blocks are 32-column groups
    // (the tensor core applies the E8M0 scales itself, so no exponent window applies).
    if (mx) {
        int rc = repack_tc(ctx, m, st);
        if (rc) return rc;
    }
    m->tiled = tiled_shape && !(flags & kFlagWide);
    // MX matrices keep only the tcgen05 tiles (the mma.sync layout is built on first use, from
    // them); BF16 keeps its row-major upload and the mma.sync tiles.
    if (m->tiled && !mx) {
        size_t total = size_t(m->rbs) * m->kslices * tile_bytes(m->format);
        URB_CUDA(ctx, cudaMallocAsync((void **)&m->tiles, total, st));
        size_t threads = size_t(m->rbs) * m->kslices * 32;
        unsigned blocks = unsigned(div_ceil(threads, 256));
        const uint8_t *v = static_cast<const uint8_t *>(m->raw_values);
        size_t br = m->format == URB_FMT_MXFP8 ? m->block_rows : 1;
        size_t bc = m->format == URB_FMT_MXFP8 ? m->block_cols : 32;
        switch (m->format) {
        case URB_FMT_MXFP4:
            k_repack<URB_FMT_MXFP4><<<blocks, 256, 0, st>>>(v, m->raw_scales, m->rows, m->cols,
                                                            scale_cols, br, bc, m->rbs,
                                                            m->kslices, m->tiles);
            break;
        case URB_FMT_MXFP8:
            k_repack<URB_FMT_MXFP8><<<blocks, 256, 0, st>>>(v, m->raw_scales, m->rows, m->cols,
                                                            scale_cols, br, bc, m->rbs,
                                                            m->kslices, m->tiles);
            break;
        default:
            k_repack<URB_FMT_BF16><<<blocks, 256, 0, st>>>(v, nullptr, m->rows, m->cols, 0, 1,
                                                           32, m->rbs, m->kslices, m->tiles);
        }
        URB_CUDA(ctx, cudaGetLastError());
        // BF16 keeps its row-major copy as well: the bit-exact router reads whole rows in
        // column order.
    }
    if (m->format == URB_FMT_BF16) {
        int rc = make_bf16_tile_map(ctx, m, st);
        if (rc) return rc;
    }
    if (mx && m->tc_tiles) {
        // The tcgen05 tiles hold every weight and scale: the reference layout goes.
        URB_CUDA(ctx, cudaFreeAsync(m->raw_values, st));
        m->raw_values = nullptr;
        if (m->raw_scales) URB_CUDA(ctx, cudaFreeAsync(m->raw_scales, st));
        m->raw_scales = nullptr;
    }
    URB_CUDA(ctx, cudaStreamSynchronize(st));
    return URB_OK;
}

}  // namespace urb
