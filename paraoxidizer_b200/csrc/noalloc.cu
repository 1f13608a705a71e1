// noalloc.cu -- the GEMV entry point that allocates nothing (pox_cuda_tensor_gemv_noalloc).
//
// Some callers cannot call cudaMalloc once they are running: a serving process that reserved its
// HBM for weights and paged KV blocks at start-up and treats any later allocation as a failure,
// or a host runtime that hands this library only the device buffers it owns. For them this entry
// point runs the same x preparation and tensor-core GEMV as pox_cuda_tensor_gemv, but the
// prepared-x scratch those kernels need lives in the file-scope device array below instead of the
// tensor's own buffer, and nothing is allocated or freed by the call.
//
// The array is kNoAllocScratchBytes (1 MiB + 16 KiB) on every GPU that loads this library, held
// until the process exits. It fits the prepared x of up to kMaxBatch rows of K <= 32768 columns;
// larger K is rejected with POX_ERR_UNSUPPORTED. All calls on one device share it and it keeps
// the last call's contents: two calls whose kernels overlap on the GPU (different streams or
// contexts on the same device) race on it, so callers serialize them. Nothing in it has to start
// at zero: every byte a call uses is written earlier in the same call by the x preparation (an
// alignment pad entry of the block metadata is copied but never used).
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>

#include "../../include/pox_cuda.h"
#include "api_internal.h"
#include "gemv.cuh"

namespace {

constexpr size_t kNoAllocMaxK = 32768;
constexpr size_t kNoAllocScratchBytes = (size_t)1 << 20 | (size_t)16 << 10;  // 1 MiB + 16 KiB

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch per device, looked up once (the symbol's host-side name is
// only a stand-in; a kernel must be given the address cudaGetSymbolAddress returns). Destroying a
// context of a device forgets that device's address, so a context created after a device reset looks
// it up again instead of using a stale one.
std::mutex g_mu;
void* g_addr[64] = {};

int scratch_address(int device, void** out) {
    if (device < 0 || device >= 64) return pox::set_error(POX_ERR_INVALID, "device %d out of range", device);
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_addr[device]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);  // device is current
        if (e != cudaSuccess) return pox::cuda_error(e, "cudaGetSymbolAddress(no-alloc scratch)");
        g_addr[device] = p;
    }
    *out = g_addr[device];
    return POX_OK;
}

}  // namespace

void pox::noalloc_forget_device(int device) {
    if (device < 0 || device >= 64) return;
    std::lock_guard<std::mutex> lk(g_mu);
    g_addr[device] = nullptr;
}

extern "C" int pox_cuda_tensor_gemv_noalloc(pox_cuda_ctx* ctx, const pox_tensor* t, const float* x_dev,
                                            size_t batch, float* y_dev, void* stream) {
    using namespace pox;
    if (!ctx || !t) return set_error(POX_ERR_INVALID, "ctx/tensor is NULL");
    if (batch && (!x_dev || !y_dev)) return set_error(POX_ERR_INVALID, "x/y is NULL");
    const cudaError_t se = cudaSetDevice(ctx->device);
    if (se != cudaSuccess) return cuda_error(se, "cudaSetDevice");
    // The call returns before its kernels finish, so a bounded wait that ran out in an earlier call's
    // kernels (this entry point's or another on the context) is reported here, before new work.
    const int prev = take_kernel_error(ctx);
    if (prev) return prev;
    if (t->rows == 0 || t->cols == 0 || batch == 0) return POX_OK;
    if (((uintptr_t)x_dev & 15) != 0) return set_error(POX_ERR_INVALID, "x must be 16-byte aligned");
    cudaStream_t st = stream ? (cudaStream_t)stream : ctx->stream;
    const int kind = t->dtype == POX_I4 ? kKindI4 : (t->dtype == POX_I8 ? kKindI8 : kKindF16);
    const int N = (int)t->rows, K = (int)t->cols;
    void* scratch = nullptr;
    if (t->tiled) {
        const size_t need = xprep_bytes(kind, K);
        if ((size_t)K > kNoAllocMaxK || need > kNoAllocScratchBytes)
            return set_error(POX_ERR_UNSUPPORTED,
                             "no-alloc GEMV: cols %d needs %zu scratch bytes; the static scratch holds %zu "
                             "(cols <= %zu)",
                             K, need, kNoAllocScratchBytes, kNoAllocMaxK);
        const int rc = scratch_address(ctx->device, &scratch);
        if (rc) return rc;
    }
    for (size_t done = 0; done < batch;) {
        const int b = (int)std::min<size_t>(batch - done, kMaxBatch);
        const float* xb = x_dev + done * t->cols;
        float* yb = y_dev + done * t->rows;
        cudaError_t e;
        if (t->tiled) {
            const TileLayout TL(kind, N, K);
            const XPrep xp = xprep_view(scratch, kind, K);
            e = launch_xprep(kind, xb, b, K, xp, PrepOp(), true, st);
            if (e != cudaSuccess) return cuda_error(e, "x preparation launch");
            GemvArgs a = {};
            a.w = (const uint8_t*)t->w;
            a.i8_scale = t->i8_scale;
            a.row_scale = t->row_scales;
            a.row_ptr = kind == kKindI4 ? t->row_ptr : nullptr;
            a.ent = t->entries;
            a.xq = xp.cols;
            a.xm = xp.meta;
            a.x = xb;
            a.y = yb;
            a.err = ctx->err_dev;
            a.N = N;
            a.K = K;
            a.Kp = xp.Kp;
            a.B = b;
            a.nxb = xp.nxb;
            a.nxbs = xp.nxbs;
            a.nT = TL.nT;
            a.nkb = TL.nkb;
            a.S = 1;
            e = launch_gemv_tc(kind, a, true, st);
        } else {
            // the raw-layout kernels use no scratch
            GemvGenericArgs a;
            a.raw = (const uint8_t*)t->w;
            a.raw_scales = (const uint8_t*)t->scales_dev;
            a.i8_scale = t->i8_scale;
            a.row_scale = t->row_scales;
            a.row_ptr = t->row_ptr;
            a.entries = t->entries;
            a.x = xb;
            a.y = yb;
            a.N = N;
            a.K = K;
            a.B = b;
            a.gs = (int)t->gs;
            a.groups = t->groups;
            e = launch_gemv_generic(kind, a, st);
        }
        if (e != cudaSuccess) return cuda_error(e, "gemv launch");
        done += (size_t)b;
    }
    return POX_OK;
}
