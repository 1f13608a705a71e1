// gemv.cuh -- launch interface and device layout of the weight-only quantized GEMV, the x
// preparation, re-tiling and dequantization kernels (gemv.cu).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace pox {

enum { kKindI4 = 0, kKindI8 = 1, kKindF16 = 2 };

constexpr int kTileBytes = 1024;  // one tile: 16 rows x one k-block
constexpr int kMaxBatch = 8;      // batch rows per launch of the tensor-core GEMV
constexpr int kXBlock = 128;      // k per x quantization block
constexpr int kXLimbMax = 16383;  // |X| bound of the 15-bit x quantization

enum { kErrWaitRing = 1, kErrWaitX = 2, kErrWaitEnt = 4 };  // bits of the kernel error flag
enum { kErrPersist = 256 };  // the persistent decode kernel: a grid-barrier or ring wait expired
// Bits for invalid input found on the device (reported as POX_ERR_INVALID rather than a timeout): a
// decode position at or beyond 16 x max_blocks_per_seq, a block-table entry outside [0, kv_blocks).
enum { kErrAttnPos = 64, kErrAttnPage = 128, kErrInputMask = kErrAttnPos | kErrAttnPage };

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

#ifdef __CUDACC__
// Element k of batch row b of the GEMV input, after the fused pre-op: x itself, RMSNorm
// (crates/paraoxidizer-runtime/src/engine.rs:294-350: x * (1 / sqrt(sum x^2 / n + eps)) then * w),
// or SwiGLU (engine.rs:671-677: g / (1 + exp(-g)) * u).
struct PrepRow {
    const float* x;
    const float* up;
    float inv;  // RMSNorm scale of this row
};
__device__ __forceinline__ float prep_elem(const PrepOp& op, const PrepRow& r, int k, float v) {
    if (op.mode == kPrepNorm) {
        const float t = v * r.inv;
        return op.norm_w ? t * half_bits_to_float(op.norm_w[k]) : t;
    }
    if (op.mode == kPrepSwiGLU) {
        const float u = r.up[k];
        return v / (1.0f + expf(-v)) * u;
    }
    return v;
}
// RMSNorm scale 1 / sqrt(sum x^2 / K + eps) of rows b0 .. b1, computed by the whole block (every
// thread must call it): each thread sums squares of k = 4 t + 4 nthreads j in order (its loads of
// four j issued together), then warps in a butterfly and the block in warp order.
__device__ __forceinline__ void block_rms_inv(const float* x, int ldx, int K, float eps, int b0, int b1,
                                              float* s_inv) {
    __shared__ float red[32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    const int step = 4 * blockDim.x;
    for (int b = b0; b <= b1; b++) {
        const float* xr = x + (size_t)b * ldx;
        float s = 0.f;
        for (int k0 = 4 * tid; k0 < K; k0 += 4 * step) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; u++)
                v[u] = k0 + u * step < K ? *reinterpret_cast<const float4*>(xr + k0 + u * step)
                                         : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int u = 0; u < 4; u++) {
                s = fmaf(v[u].x, v[u].x, s);
                s = fmaf(v[u].y, v[u].y, s);
                s = fmaf(v[u].z, v[u].z, s);
                s = fmaf(v[u].w, v[u].w, s);
            }
        }
        s = warp_sum(s);
        if (lane == 0) red[warp] = s;
        __syncthreads();
        if (tid == 0) {
            float t = 0.f;
            for (int w = 0; w < nw; w++) t += red[w];
            s_inv[b - b0] = 1.0f / sqrtf(t / (float)K + eps);
        }
        __syncthreads();
    }
}

#endif

struct GemvArgs {
    const uint8_t* w;        // tile blobs (TileLayout)
    float i8_scale;          // INT8 per-tensor scale
    const float* row_scale;  // INT8 per-output-channel scales [N] (nullptr: i8_scale)
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
    const float* row_scale;  // INT8 per-output-channel scales [N] (nullptr: i8_scale)
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
cudaError_t launch_dequant_i8(bool tiled, const void* w, float scale, const float* row_scale, float* out, int N, int K,
                              cudaStream_t st);
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
    const float* row_scale;    // INT8 per-output-channel scales [Nout] (nullptr: wscale)
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

// ---- small-M path on the integer tensor cores (tcgen05 kind::i8): INT4 without outliers and
// INT8, padded batch 16 .. 64 (gemm_tcq.cu) ----
struct TqArgs {
    const uint8_t* w;     // tile blobs (TileLayout of the kind; K % 128 == 0)
    const uint8_t* xl;    // x limbs [K / 128][2 Bp][128 B], 128-byte swizzled (row 2b: hi, 2b + 1: lo)
    const float2* xm;     // [K / 128][Bp]: (max|x| / 16383, sum x) of each 128-k block of each x row
    float wscale;         // INT8 per-tensor scale (1 otherwise)
    const float* row_scale;  // INT8 per-output-channel scales [Nout] (nullptr: wscale)
    float* y;             // [B][Nout]
    const float* resid;   // nullptr, or [B][Nout] added (may alias y)
    float* ws;            // k-split partials [S][Bp][Nout]
    int* tickets;         // [row blocks] zero-initialised, self-resetting
    int* err;
    int Nout, K, nkb, nT, B, Bp, S;  // nkb: 128-k blocks
};
bool tq_supported(int kind, bool outliers, int Bp);
size_t tq_x_bytes(int K, int Bp);  // limbs, then (256-byte aligned) the block meta
cudaError_t launch_xprep_tq(const float* x, int B, int Bp, int K, const PrepOp& op, uint8_t* xl, float2* xm,
                            cudaStream_t st);
cudaError_t launch_tq(int kind, const TqArgs& a, cudaStream_t st);

}  // namespace pox
