// quantize.cu -- group-wise INT4 quantizer on the GPU, bit-exact with the reference's
// quantize_int4_group (crates/paraoxidizer-quant/src/kernels.rs:26-82):
//   per group: min / max by a sequential scan that keeps the first of equal values and skips NaN,
//   max = min + 1e-4 when |max - min| < 1e-8, scale = (max - min) / 15 (f32), stored as f16 scale
//   and f16 min (IEEE round-to-nearest-even, crate half 2.7.1), q = round((w - min) / scale)
//   (half away from zero) clamped to [0, 15] (NaN -> 0), two q per byte, low nibble first.
// One warp per group. The first-occurrence rule only matters for +0 / -0 ties: the reduction
// carries (value, index) pairs and prefers the smaller index on equal values.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/pox_cuda.h"
#include "api_internal.h"

namespace pox {

__device__ __forceinline__ void better(float& v, int& i, float ov, int oi, bool want_min) {
    const bool take = want_min ? (ov < v || (ov == v && oi < i)) : (ov > v || (ov == v && oi < i));
    if (take) {
        v = ov;
        i = oi;
    }
}

__global__ void quantize_i4_kernel(const float* __restrict__ w, size_t groups, int gs, uint8_t* __restrict__ packed,
                                   uint8_t* __restrict__ scales) {
    const size_t g = (size_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (g >= groups) return;
    const float* gw = w + g * gs;
    float mn = INFINITY, mx = -INFINITY;
    int imn = 0x7fffffff, imx = 0x7fffffff;
    for (int i = lane; i < gs; i += 32) {  // each lane scans its elements in order: first of equals kept
        const float v = gw[i];
        if (v < mn) {
            mn = v;
            imn = i;
        }
        if (v > mx) {
            mx = v;
            imx = i;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        better(mn, imn, __shfl_xor_sync(0xffffffffu, mn, o), __shfl_xor_sync(0xffffffffu, imn, o), true);
        better(mx, imx, __shfl_xor_sync(0xffffffffu, mx, o), __shfl_xor_sync(0xffffffffu, imx, o), false);
    }
    if (fabsf(__fsub_rn(mx, mn)) < 1e-8f) mx = __fadd_rn(mn, 1e-4f);
    const float scale = __fdiv_rn(__fsub_rn(mx, mn), 15.0f);
    if (lane == 0) {  // f16 scale then f16 min, little-endian (kernels.rs:57-62)
        const uint32_t sb = __half_as_ushort(__float2half_rn(scale));
        const uint32_t mb = __half_as_ushort(__float2half_rn(mn));
        *reinterpret_cast<uint32_t*>(scales + g * 4) = sb | (mb << 16);
    }
    auto q_of = [&](float v) -> uint32_t {
        const float r = roundf(__fdiv_rn(__fsub_rn(v, mn), scale));
        if (isnan(r)) return 0u;
        return (uint32_t)fminf(fmaxf(r, 0.0f), 15.0f);
    };
    uint8_t* gp = packed + g * (gs / 2);
    for (int j = lane; j < gs / 2; j += 32) gp[j] = (uint8_t)(q_of(gw[2 * j]) | (q_of(gw[2 * j + 1]) << 4));
}

// ---------------------------------------------------------------------------------------------
// extract_and_zero_outliers (crates/paraoxidizer-quant/src/outlier.rs:57-85), bit-exact.
// The reference's f32 sums are left folds in index order, so one thread adds the elements in that
// order (IEEE adds, the square a separate multiply: no contraction) while the block's other threads
// stage the next chunk; the per-element threshold test, the ascending-index compaction (integer
// prefix sums) and the zeroing are parallel and exact.
// ---------------------------------------------------------------------------------------------
constexpr int kStatChunk = 4096;  // floats per staged chunk (two buffers)

// stats[0] = mean, stats[1] = threshold = sigma * sqrt(var_sum / n)
__global__ void __launch_bounds__(256) outlier_stats_kernel(const float* __restrict__ w, size_t n, float sigma,
                                                            float* __restrict__ stats) {
    __shared__ float buf[2][kStatChunk];
    const int tid = threadIdx.x;
    const size_t nch = (n + kStatChunk - 1) / kStatChunk;
    const float nf = (float)n;  // weights.len() as f32
    float mean = 0.f;
    for (int pass = 0; pass < 2; pass++) {
        float acc = -0.0f;  // the fold's start value, as the oracle restates it
        // chunk c is staged into buf[c & 1] by every thread while thread 0 sums chunk c - 1
        for (size_t c = 0; c <= nch; c++) {
            if (c < nch) {
                const size_t base = c * kStatChunk;
                for (int i = tid; i < kStatChunk; i += blockDim.x)
                    buf[c & 1][i] = base + i < n ? w[base + i] : 0.f;
            }
            if (c > 0 && tid == 0) {
                const size_t base = (c - 1) * kStatChunk, m = min((size_t)kStatChunk, n - base);
                const float* b = buf[(c - 1) & 1];
                if (pass == 0) {
                    for (size_t i = 0; i < m; i++) acc = __fadd_rn(acc, b[i]);
                } else {
                    for (size_t i = 0; i < m; i++) {
                        const float d = __fsub_rn(b[i], mean);
                        acc = __fadd_rn(acc, __fmul_rn(d, d));  // powi(2) = d * d
                    }
                }
            }
            __syncthreads();
        }
        if (tid == 0) {
            if (pass == 0) {
                mean = __fdiv_rn(acc, nf);
                stats[0] = mean;
            } else {
                stats[1] = __fmul_rn(sigma, __fsqrt_rn(__fdiv_rn(acc, nf)));
            }
        }
        __syncthreads();
        mean = stats[0];  // every thread (visible after the barrier; the block wrote it)
        __syncthreads();
    }
}

__device__ __forceinline__ bool is_outlier(float v, float mean, float thr) { return fabsf(__fsub_rn(v, mean)) > thr; }

// Elements [1024 blk, 1024 blk + 1024): thread t takes 4 t .. 4 t + 3.
__global__ void __launch_bounds__(256) outlier_count_kernel(const float* __restrict__ w, size_t n,
                                                            const float* __restrict__ stats, uint32_t* __restrict__ counts) {
    const float mean = stats[0], thr = stats[1];
    const size_t base = (size_t)blockIdx.x * 1024 + 4 * threadIdx.x;
    uint32_t c = 0;
#pragma unroll
    for (int j = 0; j < 4; j++)
        if (base + j < n && is_outlier(w[base + j], mean, thr)) c++;
    __shared__ uint32_t red[8];
    for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = c;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t t = 0;
        for (int i = 0; i < 8; i++) t += red[i];
        counts[blockIdx.x] = t;
    }
}

// Exclusive prefix sum of counts[0 .. nb) in place; counts[nb] = total. One block of 1024 threads.
__global__ void __launch_bounds__(1024) outlier_scan_kernel(uint32_t* __restrict__ counts, size_t nb) {
    __shared__ uint32_t part[1024];
    const int tid = threadIdx.x;
    const size_t per = (nb + 1023) / 1024, s0 = (size_t)tid * per, s1 = min(nb, s0 + per);
    uint32_t sum = 0;
    for (size_t i = s0; i < s1; i++) sum += counts[i];
    part[tid] = sum;
    __syncthreads();
    if (tid == 0) {
        uint32_t run = 0;
        for (int i = 0; i < 1024; i++) {
            const uint32_t v = part[i];
            part[i] = run;
            run += v;
        }
        counts[nb] = run;
    }
    __syncthreads();
    uint32_t run = part[tid];
    for (size_t i = s0; i < s1; i++) {
        const uint32_t v = counts[i];
        counts[i] = run;
        run += v;
    }
}

// Writes the table (count | indices | f16 values, ascending index) and zeroes the extracted weights.
__global__ void __launch_bounds__(256) outlier_write_kernel(float* __restrict__ w, size_t n,
                                                            const float* __restrict__ stats,
                                                            const uint32_t* __restrict__ offs, uint32_t count,
                                                            uint8_t* __restrict__ table) {
    const float mean = stats[0], thr = stats[1];
    const size_t base = (size_t)blockIdx.x * 1024 + 4 * threadIdx.x;
    bool f[4];
    uint32_t c = 0;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        f[j] = base + j < n && is_outlier(w[base + j], mean, thr);
        c += f[j];
    }
    // exclusive prefix of c over the block in thread order
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t incl = c;
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    __shared__ uint32_t wsum[8];
    if (lane == 31) wsum[warp] = incl;
    __syncthreads();
    uint32_t before = 0;
    for (int i = 0; i < warp; i++) before += wsum[i];
    uint32_t pos = offs[blockIdx.x] + before + incl - c;
    uint32_t* idx = reinterpret_cast<uint32_t*>(table + 4);
    __half* val = reinterpret_cast<__half*>(table + 4 + 4 * (size_t)count);
#pragma unroll
    for (int j = 0; j < 4; j++) {
        if (f[j]) {
            idx[pos] = (uint32_t)(base + j);
            val[pos] = __float2half_rn(w[base + j]);  // f16::from_f32: round to nearest even
            w[base + j] = 0.0f;
            pos++;
        }
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) *reinterpret_cast<uint32_t*>(table) = count;
}

}  // namespace pox

using namespace pox;

extern "C" int pox_cuda_extract_outliers(pox_cuda_ctx* ctx, float* w_dev, size_t n, float sigma, uint8_t* table,
                                         size_t table_cap, size_t* table_len) {
    if (!ctx || !table_len) return set_error(POX_ERR_INVALID, "NULL argument");
    *table_len = 0;
    if (n == 0) return POX_OK;  // empty weights: None (outlier.rs:59-61)
    if (!w_dev) return set_error(POX_ERR_INVALID, "w is NULL");
    if (n > 0xFFFFFFFFull) return set_error(POX_ERR_UNSUPPORTED, "outlier indices are u32: at most 2^32 elements");
    std::lock_guard<std::mutex> lk(ctx->mu);
    cudaError_t e = cudaSetDevice(ctx->device);
    if (e != cudaSuccess) return cuda_error(e, "cudaSetDevice");
    cudaStream_t st = ctx->stream;
    const size_t nb = (n + 1023) / 1024;
    float* stats = nullptr;
    uint32_t* counts = nullptr;
    uint8_t* dtab = nullptr;
    auto done = [&](int rc) {
        cudaStreamSynchronize(st);
        cudaFree(stats);
        cudaFree(counts);
        cudaFree(dtab);
        return rc;
    };
    e = cudaMalloc(&stats, 2 * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&counts, (nb + 1) * sizeof(uint32_t));
    if (e != cudaSuccess) return done(cuda_error(e, "cudaMalloc(outlier scratch)"));
    outlier_stats_kernel<<<1, 256, 0, st>>>(w_dev, n, sigma, stats);
    outlier_count_kernel<<<(unsigned)nb, 256, 0, st>>>(w_dev, n, stats, counts);
    outlier_scan_kernel<<<1, 1024, 0, st>>>(counts, nb);
    uint32_t count = 0;
    e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaMemcpyAsync(&count, counts + nb, sizeof(uint32_t), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return done(cuda_error(e, "outlier statistics"));
    if (count == 0) return done(POX_OK);  // None
    const size_t bytes = 4 + 6 * (size_t)count;
    *table_len = bytes;
    if (!table || table_cap < bytes)
        return done(set_error(POX_ERR_LAYOUT, "outlier table needs %zu bytes, buffer holds %zu (nothing modified)", bytes,
                              table_cap));
    e = cudaMalloc(&dtab, bytes);
    if (e != cudaSuccess) return done(cuda_error(e, "cudaMalloc(outlier table)"));
    outlier_write_kernel<<<(unsigned)nb, 256, 0, st>>>(w_dev, n, stats, counts, count, dtab);
    e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaMemcpyAsync(table, dtab, bytes, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return done(cuda_error(e, "outlier table"));
    return done(POX_OK);
}

extern "C" int pox_cuda_quantize_int4(pox_cuda_ctx* ctx, const float* w_dev, size_t numel, size_t group_size,
                                      uint8_t* packed_dev, uint8_t* scales_dev, void* stream) {
    if (!ctx) return set_error(POX_ERR_INVALID, "ctx is NULL");
    if (numel == 0) return POX_OK;
    if (!w_dev || !packed_dev || !scales_dev) return set_error(POX_ERR_INVALID, "NULL buffer");
    if (group_size == 0 || group_size % 2 || numel % group_size || group_size > (1u << 20))
        return set_error(POX_ERR_UNSUPPORTED, "numel must be a multiple of an even group size");
    cudaError_t e = cudaSetDevice(ctx->device);
    if (e != cudaSuccess) return cuda_error(e, "cudaSetDevice");
    const size_t groups = numel / group_size;
    const unsigned blocks = (unsigned)((groups + 7) / 8);
    quantize_i4_kernel<<<blocks, 256, 0, stream ? (cudaStream_t)stream : ctx->stream>>>(w_dev, groups, (int)group_size,
                                                                                       packed_dev, scales_dev);
    e = cudaGetLastError();
    return e == cudaSuccess ? POX_OK : cuda_error(e, "quantize_int4 launch");
}
