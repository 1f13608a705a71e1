// api_internal.h -- host-side structures shared by the C ABI translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <unordered_map>
#include <vector>

#include "../../include/pox_cuda.h"

struct pox_tensor {
    int dtype = POX_I4;
    size_t rows = 0, cols = 0, gs = 0;
    int groups = 0;
    bool tiled = false;        // re-tiled device layout (tensor-core GEMV) vs raw .pox layout
    void* w = nullptr;         // tiles or raw payload
    void* scales_dev = nullptr;   // tiled INT4: scale words per tile; raw INT4: the .pox scale bytes
    float i8_scale = 0.f;
    float* row_scales = nullptr;  // INT8 per-output-channel scales [rows] (f32 of the f16 table), or nullptr
    uint32_t* row_ptr = nullptr;  // outlier CSR by row [rows+1]
    uint2* entries = nullptr;     // (col, f32 bits of v - dequant(q))
    uint16_t* vals = nullptr;     // f16 outlier values (dequantization path)
    uint32_t* tile_ptr = nullptr; // tiled INT4: outliers ordered by (row tile, 128-k block) [nT * nkb + 1]
    uint32_t* tile_ent = nullptr; //   (row % 16) | (col % 128) << 4 | f16 value << 16
    size_t nnz = 0;
    void* scratch = nullptr;      // prepared x of the tiled GEMV (up to 8 batch rows)
    size_t scratch_bytes = 0;
    // host-slice calls: the launches of the last (batch, staging buffers) as one CUDA graph
    cudaGraphExec_t host_graph = nullptr;
    size_t host_graph_batch = 0;
    const void* host_graph_x = nullptr;
    const void* host_graph_y = nullptr;
    size_t bytes = 0;
    // host slices the tensor was uploaded from (registry key of the host-slice entry points)
    const uint8_t* h_data = nullptr;
    size_t h_data_len = 0;
    const uint8_t* h_scales = nullptr;
    size_t h_scale_len = 0;
    const uint8_t* h_outliers = nullptr;
    size_t h_outlier_len = 0;
};

struct pox_cuda_ctx {
    int device = 0;
    int num_sms = 148;
    cudaStream_t stream = nullptr;
    std::mutex mu;
    std::vector<pox_tensor*> tensors;
    // resident tensors by the host address of their weight payload (the key of the host-slice calls)
    std::unordered_multimap<const void*, pox_tensor*> by_host;
    // host-slice calls on tiled tensors: pinned, device-mapped staging for x and y (the x preparation
    // reads x over PCIe and the GEMV writes y there: no DMA copies)
    float* pin_x = nullptr;
    float* pin_x_dev = nullptr;
    size_t pin_x_bytes = 0;
    float* pin_y = nullptr;
    float* pin_y_dev = nullptr;
    size_t pin_y_bytes = 0;
    void* scratch_x = nullptr;
    size_t scratch_x_bytes = 0;
    void* scratch_y = nullptr;
    size_t scratch_y_bytes = 0;
    void* tc_scratch = nullptr;  // small-M path: prepared x, row scales, k-split partials
    size_t tc_scratch_bytes = 0;
    int* tc_tickets = nullptr;   // small-M path: per row block split counters (zeroed, self-resetting)
    size_t tc_tickets_n = 0;
    void* attn_scratch = nullptr;  // kernel-level paged attention: split partials
    size_t attn_scratch_bytes = 0;
    int* err_host = nullptr;  // kernel error flag (host-mapped); nonzero = a bounded wait expired or bad input
    int* err_dev = nullptr;
    std::vector<pox_model*> models;  // decode models created on this context (destroyed with it)
};

namespace pox {
int set_error(int code, const char* fmt, ...);
int cuda_error(cudaError_t e, const char* what);
int ensure_scratch(pox_cuda_ctx* ctx, size_t xbytes, size_t ybytes);
int upload_tensor_locked(pox_cuda_ctx* ctx, const pox_tensor_desc* d, pox_tensor** out, bool keep);
struct PrepOp;
// GEMV of a resident tensor on device pointers; op fuses RMSNorm / SwiGLU into the x preparation
// and resid (same shape as y, may alias it) is added to the result (tiled tensors only).
// prepared = the x preparation was already written by the caller (gemv_x_target), x itself is
// still passed (the GEMV's outlier correction reads it).
int gemv_launch(pox_cuda_ctx* ctx, const pox_tensor* t, const float* x, size_t batch, float* y, cudaStream_t st,
                const PrepOp* op = nullptr, const float* resid = nullptr, bool prepared = false);
// Where a kernel that produces the input of an INT4 tiled tensor's GEMV can write it prepared
// (batch <= 8: the two-limb fixed point + meta; small-M path: swizzled f16 + row scales).
struct XTarget {
    uint8_t* cols = nullptr;
    float2* meta = nullptr;
    int Kp = 0, nxbs = 0;
    uint8_t* xs = nullptr;
    float* xscale = nullptr;
    uint8_t* xl = nullptr;   // integer small-M path: limbs [K/128][2 Bp][128 B] (swizzled), then
    float2* xm = nullptr;    // (max|x|/16383, sum x) [K/128][Bp]
    int Bp = 0;
};
int gemv_x_target(pox_cuda_ctx* ctx, const pox_tensor* t, size_t batch, cudaStream_t st, XTarget* out);
bool gemv_uses_small_m(const pox_tensor* t, size_t batch);
void destroy_ctx_extras(pox_cuda_ctx* ctx);
// Small-M path scratch for a tensor of rows x cols at `batch` rows of x (grown outside stream
// capture only; a captured graph keeps the buffers it was captured with).
int ensure_tc_scratch(pox_cuda_ctx* ctx, size_t rows, size_t cols, size_t batch, cudaStream_t st);
// After a synchronize: turns a raised kernel error flag into POX_ERR_TIMEOUT, or POX_ERR_INVALID for
// input rejected on the device (and clears it).
int take_kernel_error(pox_cuda_ctx* ctx);
// Drops the cached device address of the no-allocation GEMV's scratch array for `device`.
void noalloc_forget_device(int device);
}  // namespace pox
