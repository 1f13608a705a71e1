// comm.cu -- exchanges of tensor-parallel decode (NCCL and one-shot peer-memory kernels); the
// design and the buffer-reuse argument are in comm.cuh.
#include <cuda_runtime.h>

#include <cstring>

#include "../../include/pox_cuda.h"
#include "api_internal.h"
#include "comm.cuh"
#include "common.cuh"

#ifdef POX_HAVE_NCCL
#include <nccl.h>
#endif

namespace pox {

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ float4 ld_volatile_f4(const float* p) {
    float4 v;
    asm volatile("ld.volatile.global.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p)
                 : "memory");
    return v;
}
__device__ __forceinline__ float2 ld_volatile_f2(const float* p) {
    float2 v;
    asm volatile("ld.volatile.global.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "l"(p) : "memory");
    return v;
}

// Arrival handshake of one exchange: block 0 stores this rank's epoch into every rank's flag
// array; in every block, thread p < tp waits (bounded) until rank p's flag here reached the epoch.
// Returns false (error flag raised) if a rank did not arrive in time; no peer data is read then.
// Once a wait has expired, later exchanges skip waiting (a sticky local abort word, cleared by
// comm_reset), so a missing rank costs one timeout, not one per exchange.
__device__ bool peer_handshake(const PeerView& v, unsigned long long epoch) {
    __shared__ int ok;
    if (threadIdx.x == 0) ok = 1;
    if (blockIdx.x == 0 && threadIdx.x < v.tp) st_release_sys(v.flags[threadIdx.x] + v.rank, epoch);
    __syncthreads();
    if (threadIdx.x < v.tp) {
        const unsigned long long* f = v.flags[v.rank] + threadIdx.x;
        if (*(volatile int*)v.abort) {
            ok = 0;
        } else {
            const long long t0 = clock64();
            while (ld_acquire_sys(f) < epoch) {
                if (clock64() - t0 > kWaitCycles) {
                    atomicOr(v.err, kErrWaitPeer);
                    *(volatile int*)v.abort = 1;
                    ok = 0;
                    break;
                }
                __nanosleep(32);
            }
        }
    }
    __syncthreads();
    return ok != 0;
}

// out[i] = sum over ranks p = 0 .. tp-1 (in order) of slot s of rank p, n4 float4 elements.
__global__ void __launch_bounds__(256) peer_allreduce_kernel(PeerView v, int call, int cps, int s, int n4,
                                                             float* __restrict__ out) {
    const unsigned long long epoch = *v.step * (unsigned long long)cps + (unsigned long long)call + 1ull;
    if (!peer_handshake(v, epoch)) return;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += gridDim.x * blockDim.x) {
        float4 acc = ld_volatile_f4(v.slot[0][s] + 4 * (size_t)i);
        for (int p = 1; p < v.tp; p++) {
            const float4 t = ld_volatile_f4(v.slot[p][s] + 4 * (size_t)i);
            acc.x += t.x;
            acc.y += t.y;
            acc.z += t.z;
            acc.w += t.w;
        }
        reinterpret_cast<float4*>(out)[i] = acc;
    }
}

// The better of two (logit, token) pairs: larger logit, then the smaller token (first maximum).
__device__ __forceinline__ void better_pair(float2& a, float2 b) {
    const int ai = __float_as_int(a.y), bi = __float_as_int(b.y);
    if (b.x > a.x || (b.x == a.x && bi < ai)) a = b;
}

// Greedy pick over the ranks' pairs; then the step counter advances (single block).
__global__ void __launch_bounds__(256) peer_pick_kernel(PeerView v, int call, int cps, int B, uint32_t* next) {
    const unsigned long long epoch = *v.step * (unsigned long long)cps + (unsigned long long)call + 1ull;
    const bool ok = peer_handshake(v, epoch);
    if (ok) {
        for (int b = threadIdx.x; b < B; b += blockDim.x) {
            float2 best = ld_volatile_f2(v.slot[0][2] + 2 * (size_t)b);
            for (int p = 1; p < v.tp; p++) better_pair(best, ld_volatile_f2(v.slot[p][2] + 2 * (size_t)b));
            const int idx = __float_as_int(best.y);
            next[b] = idx < 0 ? 0u : (uint32_t)idx;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) *v.step += 1ull;
}

// NCCL variant of the pick: gathered [tp][B] pairs in local memory.
__global__ void gathered_pick_kernel(const float2* __restrict__ g, int tp, int B, uint32_t* next,
                                     unsigned long long* step) {
    for (int b = threadIdx.x; b < B; b += blockDim.x) {
        float2 best = g[b];
        for (int p = 1; p < tp; p++) better_pair(best, g[(size_t)p * B + b]);
        const int idx = __float_as_int(best.y);
        next[b] = idx < 0 ? 0u : (uint32_t)idx;
    }
    __syncthreads();
    if (threadIdx.x == 0) *step += 1ull;
}

static size_t align256(size_t n) { return (n + 255) & ~(size_t)255; }

int comm_alloc(TpComm& c, int rank, int tp, size_t max_batch, size_t hidden, int* err_dev) {
    c.rank = rank;
    c.tp = tp;
    c.slot_bytes = align256(max_batch * hidden * sizeof(float));
    c.pair_bytes = align256(max_batch * sizeof(float2));
    const size_t bytes = 256 + 2 * c.slot_bytes + c.pair_bytes;
    cudaError_t e = cudaMalloc(&c.buf, bytes);
    if (e == cudaSuccess) e = cudaMemset(c.buf, 0, bytes);
    if (e == cudaSuccess) e = cudaMalloc(&c.step, sizeof(unsigned long long));
    if (e == cudaSuccess) e = cudaMemset(c.step, 0, sizeof(unsigned long long));
    if (e == cudaSuccess) e = cudaMalloc(&c.gathered, (size_t)tp * max_batch * sizeof(float2));
    if (e != cudaSuccess) return cuda_error(e, "cudaMalloc(exchange buffers)");
    c.pairs = reinterpret_cast<float2*>(c.buf + 256 + 2 * c.slot_bytes);
    std::memset(&c.view, 0, sizeof(c.view));
    c.view.rank = rank;
    c.view.tp = tp;
    c.view.step = c.step;
    c.view.err = err_dev;
    c.view.abort = reinterpret_cast<int*>(c.buf + 128);  // local only; peers never touch it
    return POX_OK;
}

void comm_free(TpComm& c) {
#ifdef POX_HAVE_NCCL
    if (c.nccl) ncclCommDestroy((ncclComm_t)c.nccl);
#endif
    c.nccl = nullptr;
    for (int p = 0; p < kMaxTP; p++)
        if (c.mapped[p]) cudaIpcCloseMemHandle(c.mapped[p]);
    cudaFree(c.buf);
    cudaFree(c.step);
    cudaFree(c.gathered);
    c = TpComm();
}

int comm_init_nccl(TpComm& c, const uint8_t id[128]) {
#ifdef POX_HAVE_NCCL
    static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
    if (c.nccl) return POX_OK;
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof(uid));
    ncclComm_t comm;
    const ncclResult_t r = ncclCommInitRank(&comm, c.tp, uid, c.rank);
    if (r != ncclSuccess) return set_error(POX_ERR_NCCL, "ncclCommInitRank: %s", ncclGetErrorString(r));
    c.nccl = comm;
    if (!c.mode) c.mode = POX_COMM_NCCL;
    return POX_OK;
#else
    (void)c;
    (void)id;
    return set_error(POX_ERR_UNSUPPORTED, "built without NCCL");
#endif
}

int comm_ipc_handle(TpComm& c, uint8_t handle[64]) {
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "cudaIpcMemHandle_t is 64 bytes");
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, c.buf);
    if (e != cudaSuccess) return cuda_error(e, "cudaIpcGetMemHandle");
    std::memcpy(handle, &h, sizeof(h));
    return POX_OK;
}

int comm_open_peers(TpComm& c, const uint8_t* handles) {
    if (c.peer_ready) return POX_OK;
    char* base[kMaxTP] = {};
    for (int p = 0; p < c.tp; p++) {
        if (p == c.rank) {
            base[p] = c.buf;
            continue;
        }
        cudaIpcMemHandle_t h;
        std::memcpy(&h, handles + 64 * (size_t)p, sizeof(h));
        void* ptr = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) return cuda_error(e, "cudaIpcOpenMemHandle");
        c.mapped[p] = ptr;
        base[p] = static_cast<char*>(ptr);
    }
    for (int p = 0; p < c.tp; p++) {
        c.view.flags[p] = reinterpret_cast<unsigned long long*>(base[p]);
        c.view.slot[p][0] = reinterpret_cast<float*>(base[p] + 256);
        c.view.slot[p][1] = reinterpret_cast<float*>(base[p] + 256 + c.slot_bytes);
        c.view.slot[p][2] = reinterpret_cast<float*>(base[p] + 256 + 2 * c.slot_bytes);
    }
    c.peer_ready = true;
    if (!c.mode) c.mode = POX_COMM_PEER;
    return POX_OK;
}

int comm_reset(TpComm& c, cudaStream_t st) {
    if (!c.buf) return POX_OK;
    const cudaError_t e = cudaMemsetAsync(c.buf + 128, 0, sizeof(int), st);
    return e == cudaSuccess ? POX_OK : cuda_error(e, "cudaMemsetAsync(abort word)");
}

float* comm_partial(TpComm& c, int call, float* x) {
    if (c.mode == POX_COMM_PEER) return c.view.slot[c.rank][call & 1];
    return x;
}

int comm_allreduce(TpComm& c, int call, int cps, float* x, size_t n, cudaStream_t st) {
    if (c.mode == POX_COMM_PEER) {
        const int n4 = (int)(n / 4);  // n = batch x hidden, hidden % 128 == 0
        const int blocks = std::max(1, std::min(148, (n4 + 255) / 256));
        peer_allreduce_kernel<<<blocks, 256, 0, st>>>(c.view, call, cps, call & 1, n4, x);
        const cudaError_t e = cudaGetLastError();
        return e == cudaSuccess ? POX_OK : cuda_error(e, "peer allreduce launch");
    }
#ifdef POX_HAVE_NCCL
    if (c.mode == POX_COMM_NCCL) {
        const ncclResult_t r = ncclAllReduce(x, x, n, ncclFloat, ncclSum, (ncclComm_t)c.nccl, st);
        return r == ncclSuccess ? POX_OK : set_error(POX_ERR_NCCL, "ncclAllReduce: %s", ncclGetErrorString(r));
    }
#endif
    return set_error(POX_ERR_INVALID, "tensor-parallel exchange not set up");
}

int comm_pick(TpComm& c, int call, int cps, int B, uint32_t* next, cudaStream_t st) {
    if (c.mode == POX_COMM_PEER) {
        peer_pick_kernel<<<1, 256, 0, st>>>(c.view, call, cps, B, next);
        const cudaError_t e = cudaGetLastError();
        return e == cudaSuccess ? POX_OK : cuda_error(e, "peer pick launch");
    }
#ifdef POX_HAVE_NCCL
    if (c.mode == POX_COMM_NCCL) {
        const ncclResult_t r =
            ncclAllGather(c.pairs, c.gathered, 2 * (size_t)B, ncclFloat, (ncclComm_t)c.nccl, st);
        if (r != ncclSuccess) return set_error(POX_ERR_NCCL, "ncclAllGather: %s", ncclGetErrorString(r));
        gathered_pick_kernel<<<1, 256, 0, st>>>(c.gathered, c.tp, B, next, c.step);
        const cudaError_t e = cudaGetLastError();
        return e == cudaSuccess ? POX_OK : cuda_error(e, "pick launch");
    }
#endif
    return set_error(POX_ERR_INVALID, "tensor-parallel exchange not set up");
}

}  // namespace pox

extern "C" int pox_cuda_comm_check_missing_rank(pox_cuda_ctx* ctx, double* wait_seconds) {
    using namespace pox;
    if (!ctx) return set_error(POX_ERR_INVALID, "ctx is NULL");
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (cudaSetDevice(ctx->device) != cudaSuccess) return set_error(POX_ERR_CUDA, "cudaSetDevice");
    if (cudaStreamSynchronize(ctx->stream) != cudaSuccess) return set_error(POX_ERR_CUDA, "cudaStreamSynchronize");
    int rc = take_kernel_error(ctx);  // an earlier call's error is reported first
    if (rc) return rc;
    TpComm c;
    rc = comm_alloc(c, 0, 2, 1, 128, ctx->err_dev);
    char* absent = nullptr;  // exchange buffer of the rank that never arrives: same layout, never written
    float* out = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    const size_t bytes = 256 + 2 * c.slot_bytes + c.pair_bytes;
    cudaError_t e = rc ? cudaErrorUnknown : cudaMalloc(&absent, bytes);
    if (e == cudaSuccess) e = cudaMemset(absent, 0, bytes);
    if (e == cudaSuccess) e = cudaMalloc(&out, 128 * sizeof(float));
    if (e == cudaSuccess) e = cudaEventCreate(&e0);
    if (e == cudaSuccess) e = cudaEventCreate(&e1);
    int abort_word = 0;
    float ms = 0.f;
    if (e == cudaSuccess) {
        char* base[2] = {c.buf, absent};
        for (int p = 0; p < 2; p++) {
            c.view.flags[p] = reinterpret_cast<unsigned long long*>(base[p]);
            for (int s = 0; s < 3; s++) c.view.slot[p][s] = reinterpret_cast<float*>(base[p] + 256 + s * c.slot_bytes);
        }
        cudaEventRecord(e0, ctx->stream);
        peer_allreduce_kernel<<<1, 256, 0, ctx->stream>>>(c.view, 0, 3, 0, 32, out);
        e = cudaGetLastError();
        cudaEventRecord(e1, ctx->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
        if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, e0, e1);
        if (e == cudaSuccess) e = cudaMemcpy(&abort_word, c.buf + 128, sizeof(int), cudaMemcpyDeviceToHost);
    }
    const int flag = *(volatile int*)ctx->err_host;
    *(volatile int*)ctx->err_host = 0;
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    cudaFree(out);
    cudaFree(absent);
    comm_free(c);
    if (rc) return rc;
    if (e != cudaSuccess) return cuda_error(e, "missing-rank check");
    if (wait_seconds) *wait_seconds = ms * 1e-3;
    if (!(flag & kErrWaitPeer) || abort_word != 1)
        return set_error(POX_ERR_CUDA, "the exchange did not report the missing rank (flag 0x%x, abort %d)", flag,
                         abort_word);
    return POX_OK;
}

