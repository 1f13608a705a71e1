// gemv.cuh -- launch interface and device layout of the weight-only quantized GEMV, the x
// preparation, re-tiling and dequantization kernels (gemv.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace pox {

enum { kKindI4 = 0, kKindI8 = 1, kKindF16 = 2 };

constexpr int kTileBytes = 1024;  // one tile: 16 rows x one k-block
constexpr int kMaxBatch = 8;      // batch rows per launch of the tensor-core GEMV
constexpr int kXBlock = 128;      // k per x quantization block
constexpr int kXLimbMax = 16383;  // |X| bound of the 15-bit x quantization

enum { kErrWaitRing = 1, kErrWaitX = 2, kErrWaitEnt = 4 };  // bits of the kernel error flag

__host__ __device__ inline int kind_kblock(int kind) { return kind == kKindI4 ? 128 : (kind == kKindI8 ? 64 : 32); }

// Device layout of a re-tiled weight matrix [N][K].
// Tiles are 16 rows x one k-block (INT4 128 k, INT8 64 k, F16 32 k) = 1 KiB, stored row-tile
// major: tile (T, kb) at byte (T * nkb + kb) * 1024, so the k-blocks of one row tile are one
// contiguous stream. Inside a tile, lane l = 4g + t of a warp owns the 16 bytes at
// s * 512 + l * 16 (s = 0, 1): row 16T + g + 8s, k sub-range t of the block:
//   INT4: word w (4 bytes) of the 16: byte i = q[k0 + 8w + i] | q[k0 + 8w + 4 + i] << 4,
//         k0 = 128 kb + 32 t (low nibbles and high nibbles each cover 4 consecutive k)
//   INT8: byte j = q[64 kb + 16 t + j]
//   F16 : half j = w[32 kb + 8 t + j]
// so that a tile is read with two fully coalesced 512-byte warp loads and every lane's bytes
// are directly the A fragments of m16n8k32 (u8/s8) or m16n8k16 (f16) MMAs.
// INT4 tiles carry their scales: the 1 KiB of nibbles is followed by 16 u32 words
// (f16 scale | f16 min << 16), word 2g + s for row 16T + g + 8s, so one blob is 1088 bytes and a
// run of consecutive tiles is one contiguous copy.
__host__ __device__ inline int kind_tile_bytes(int kind) { return kTileBytes + (kind == kKindI4 ? 64 : 0); }
struct TileLayout {
    int N, K, KB, nT, nkb, tb;
    __host__ __device__ TileLayout(int kind, int N_, int K_) : N(N_), K(K_) {
        KB = kind_kblock(kind);
        nT = (N + 15) / 16;
        nkb = K / KB;
        tb = kind_tile_bytes(kind);
    }
    __host__ __device__ size_t tiles() const { return (size_t)nT * nkb; }
    __host__ __device__ size_t bytes() const { return tiles() * tb; }
};

// Prepared activations ("x prep"): x [B][K] f32 becomes, per batch row b, two columns
// 2b (hi) and 2b+1 (lo) of Kp = ceil(K / 128) * 128 elements each:
//   INT4 / INT8 weights: per 128-k block, X = rint(x * 16383 / max|x|) split into exact int8
//     limbs X = 128 * hi + lo (hi in [-128, 127], lo in [0, 127]); meta[b][blk] = (max|x| /
//     16383, sum of x over the block)
//   F16 weights: hi = f16(x), lo = f16(x - hi) (22 significant bits of x)
struct XPrep {
    void* cols;      // [2B][Kp] bytes (INT) or halves (F16)
    float2* meta;    // [B][nxbs]: nxbs = Kp / 128 rounded up to even (16-byte aligned rows)
    int Kp, nxb, nxbs;
};

// Operation fused into the x preparation of a GEMV (decode step): the GEMV input row b is
// op(x + b * ld_x), element-wise after the row's RMSNorm scale where that applies.
enum { kPrepNone = 0, kPrepNorm = 1, kPrepSwiGLU = 2 };
struct PrepOp {
    int mode = kPrepNone;
    const uint16_t* norm_w = nullptr;  // kPrepNorm: [K] f16 weight (nullptr: none)
    float eps = 1e-5f;                 // kPrepNorm
    const float* up = nullptr;         // kPrepSwiGLU: up rows (x holds the gate rows)
    int ld_x = 0, ld_up = 0;           // row strides in elements (0: K)
};

struct GemvArgs {
    const uint8_t* w;        // tile blobs (TileLayout)
    float i8_scale;          // INT8 per-tensor scale
    const uint32_t* row_ptr; // outlier CSR by row [N+1] (nullptr if none)
    const uint2* ent;        // (col, f32 bits of v - dequant(q))
    const void* xq;          // prepared x columns
    const float2* xm;        // prepared x meta
    const float* x;          // original x [B][K] f32 (outlier correction)
    float* y;                // [B][N]
    const float* resid;      // nullptr, or [B][N] added to the result (y may alias it)
    int* err;                // kernel error flag (a bounded wait expired)
    int N, K, Kp, B, nxb, nxbs;
    int nT, nkb, S;          // row tiles, k-blocks, k-splits (cluster size)
};

// Scratch bytes of the prepared x for a tensor of `K` columns at up to kMaxBatch rows.
size_t xprep_bytes(int kind, int K);
XPrep xprep_view(void* scratch, int kind, int K);

cudaError_t launch_xprep(int kind, const float* x, int B, int K, const XPrep& xp, const PrepOp& op, bool pdl,
                         cudaStream_t st);
// Plans and launches the tensor-core GEMV (B <= kMaxBatch). pdl lets the weight stream start
// before the previous kernel in the stream (the x preparation) has finished.
cudaError_t launch_gemv_tc(int kind, const GemvArgs& a, bool pdl, cudaStream_t st);

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
cudaError_t launch_gemv_generic(int kind, const GemvGenericArgs& a, cudaStream_t st);

cudaError_t launch_repack(int kind, const uint8_t* src, uint8_t* tiles, int N, int K, cudaStream_t st);
cudaError_t launch_repack_i4_scales(const uint8_t* src, uint8_t* tiles, int N, int K, int gs, cudaStream_t st);
cudaError_t launch_dequant_i4(bool tiled, const void* w, const void* scales, float* out, int N, int K, int groups,
                              int gs, cudaStream_t st);
cudaError_t launch_dequant_i8(bool tiled, const void* w, float scale, float* out, int N, int K, cudaStream_t st);
cudaError_t launch_apply_outliers(const uint32_t* row_ptr, const uint2* entries, const uint16_t* vals, float* out,
                                  int N, int K, cudaStream_t st);


// ---- small-M path (tcgen05): batch 9 .. 128 rows of x per launch (gemm_tc05.cu) ----
struct TcArgs {
    const uint8_t* w;          // tile blobs (TileLayout of the kind; K % 128 == 0)
    const uint32_t* tile_ptr;  // INT4 outliers by (row tile, 128-k block): [nT * nkb + 1] (nullptr if none)
    const uint32_t* tile_ent;  // (row % 16) | (col % 128) << 4 | f16 value << 16, in tile_ptr order
    uint32_t nnz;
    const uint8_t* xs;         // prepared x: [K / 128][2][Bp][128 B], swizzled
    const float* xscale;       // [Bp] power-of-two scale of each x row
    float wscale;              // INT8 per-tensor scale (1 otherwise)
    float* y;                  // [B][Nout]
    const float* resid;        // nullptr, or [B][Nout] added (may alias y)
    float* ws;                 // k-split partials [S][Bp][Nout]
    int* tickets;              // [row blocks] zero-initialised, self-resetting
    int* err;
    int Nout, K, nkb, nT, B, Bp, S;
};
int tc05_pad(int B);                      // padded batch (MMA N): 16, 32, 64 or 128
size_t tc05_x_bytes(int K, int Bp);       // prepared-x bytes
int tc05_splits(int nrb, int nkb, int sms);
cudaError_t launch_tc05(int kind, const TcArgs& a, cudaStream_t st);
cudaError_t launch_xprep_tc05(const float* x, int B, int Bp, int K, const PrepOp& op, uint8_t* xs, float* xscale,
                              cudaStream_t st);

}  // namespace pox
