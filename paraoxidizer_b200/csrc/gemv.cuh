// gemv.cuh -- launch interface and device-layout definitions of the GEMV / re-tiling /
// dequantization kernels (gemv.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace pox {

enum { kKindI4 = 0, kKindI8 = 1, kKindF16 = 2 };

constexpr int kTileBytesL = 1024;  // one tile: 16 rows x one k-block
constexpr int kChunkTiles = 8;     // k-blocks per chunk (one streamed item = one row tile x one chunk)
constexpr int kMaxBatch = 8;       // batch rows per launch of the streaming kernel

__host__ __device__ inline int kind_kblock(int kind) { return kind == kKindI4 ? 128 : (kind == kKindI8 ? 64 : 32); }

// Device layout of a re-tiled weight matrix. The matrix is cut into items: one row tile (16
// rows) x one chunk of kChunkTiles k-blocks. Items are ordered chunk-major (item = c * nT + T)
// and stored as uniform blobs, so a CTA streaming a contiguous item range reads one contiguous
// byte range and touches at most a couple of chunks of x:
//   INT4 blob = [scales: 8 k-blocks x 16 rows x (f16 scale | f16 min << 16), 512 B][8 tiles]
//   INT8/F16 blob = [8 tiles]
// A tile (16 rows x one k-block) is 1 KiB: bytes [s*512 + lane*16, +16) hold lane's 16 bytes of
// row g + 8s (g = lane/4) in MMA fragment order. The last chunk of a row may hold fewer than
// kChunkTiles k-blocks; its blobs keep the full stride.
struct TileLayout {
    int N, K, KB, nT, nkb, nchunks, scale_bytes;
    size_t stride;
    __host__ __device__ TileLayout(int kind, int N_, int K_) : N(N_), K(K_) {
        KB = kind_kblock(kind);
        nT = (N + 15) / 16;
        nkb = K / KB;
        nchunks = (nkb + kChunkTiles - 1) / kChunkTiles;
        scale_bytes = kind == kKindI4 ? kChunkTiles * 64 : 0;
        stride = (size_t)scale_bytes + (size_t)kChunkTiles * kTileBytesL;
    }
    __host__ __device__ int kch(int c) const {
        const int r = nkb - c * kChunkTiles;
        return r < kChunkTiles ? r : kChunkTiles;
    }
    __host__ __device__ int items() const { return nT * nchunks; }
    __host__ __device__ size_t bytes() const { return (size_t)items() * stride; }
    // byte offset of tile (row tile T, k-block kb) and of its 16 scale words (INT4)
    __host__ __device__ size_t tile_off(int T, int kb) const {
        const size_t item = (size_t)(kb / kChunkTiles) * nT + T;
        return item * stride + scale_bytes + (size_t)(kb % kChunkTiles) * kTileBytesL;
    }
    __host__ __device__ size_t scale_off(int T, int kb) const {
        const size_t item = (size_t)(kb / kChunkTiles) * nT + T;
        return item * stride + (size_t)(kb % kChunkTiles) * 64;
    }
};

struct StreamArgs {
    const unsigned char* blobs;  // re-tiled weights (item blobs, see TileLayout)
    float i8_scale;              // INT8 per-tensor scale
    const uint32_t* item_ptr;    // outlier CSR by item [items+1] (nullptr if none)
    const uint2* entries;        // (col << 4 | row % 16, f32 bits of v - dequant(q))
    const float* x;              // [B][K] device, 16-byte aligned
    float* y;                    // [B][N] device
    float* partial;              // scratch [nT][nchunks][16][kMaxBatch]
    unsigned* counters;          // scratch [nT], zero between launches
    int* err;                    // error flag (host-mapped)
    int N, K, B;
    int ring;                    // smem ring stages
    int span;                    // max chunks of x a CTA stages
};

// Row-per-warp GEMV over the raw .pox layout (any even group size, any cols).
struct GemvGenericArgs {
    const uint8_t* raw;
    const uint8_t* raw_scales;
    float i8_scale;
    const uint32_t* row_ptr;
    const uint2* entries;
    const float* x;
    float* y;
    int N, K, B, gs, groups;
};

enum { kErrTimeoutFull = 1, kErrTimeoutEmpty = 2 };

// Scratch bytes the streaming kernel needs for a tensor (partials + counters).
size_t stream_scratch_bytes(int kind, int N, int K);
// Plans and launches the streaming GEMV (B <= kMaxBatch). Returns cudaErrorInvalidConfiguration
// when the shape does not fit the kernel's shared-memory plan. pdl enables programmatic
// dependent launch (the weight stream may start before the previous kernel in the stream ends).
cudaError_t launch_gemv_stream(int kind, const StreamArgs& a, bool pdl, cudaStream_t st);
cudaError_t launch_gemv_generic(int kind, const GemvGenericArgs& a, cudaStream_t st);
cudaError_t launch_repack(int kind, const uint8_t* src, uint8_t* blobs, int N, int K, cudaStream_t st);
cudaError_t launch_repack_i4_scales(const uint8_t* src, uint8_t* blobs, int N, int K, int gs, cudaStream_t st);
cudaError_t launch_dequant_i4(bool tiled, const void* w, const void* raw_scales, float* out, int N, int K,
                              int groups, int gs, cudaStream_t st);
cudaError_t launch_dequant_i8(bool tiled, const void* w, float scale, float* out, int N, int K, cudaStream_t st);
cudaError_t launch_apply_outliers(const uint32_t* row_ptr, const uint2* entries, const uint16_t* vals, float* out,
                                  int N, int K, cudaStream_t st);
cudaError_t launch_apply_outliers_items(const uint32_t* item_ptr, const uint2* entries, const uint16_t* vals,
                                        float* out, int N, int K, cudaStream_t st);

}  // namespace pox
