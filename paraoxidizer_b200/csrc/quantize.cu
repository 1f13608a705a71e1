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

}  // namespace pox

using namespace pox;

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
