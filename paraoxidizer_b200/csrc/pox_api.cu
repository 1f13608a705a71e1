// pox_api.cu -- the C ABI of include/pox_cuda.h: contexts, resident tensors (upload once, device
// re-tiling, outlier CSR), and the reference-shaped GEMV / dequantization entry points.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/pox_cuda.h"
#include "api_internal.h"
#include "common.cuh"
#include "gemv.cuh"

using namespace pox;

// ------------------------------------------------------------------------------------------
// errors
// ------------------------------------------------------------------------------------------
static thread_local std::string t_last_error;

int pox::set_error(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    t_last_error = buf;
    return code;
}

int pox::cuda_error(cudaError_t e, const char* what) {
    if (e == cudaErrorMemoryAllocation)
        return set_error(POX_ERR_OOM, "%s: %s", what, cudaGetErrorString(e));
    return set_error(POX_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define CK(call, what)                               \
    do {                                             \
        cudaError_t _e = (call);                     \
        if (_e != cudaSuccess) return cuda_error(_e, what); \
    } while (0)

extern "C" const char* pox_cuda_last_error(void) { return t_last_error.c_str(); }
extern "C" const char* pox_cuda_version(void) { return "pox_cuda 0.1.0 (sm_100a)"; }

extern "C" int pox_cuda_device_count(int* out) {
    if (!out) return set_error(POX_ERR_INVALID, "out is NULL");
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) {
        cudaGetLastError();
        n = 0;
    }
    *out = n;
    return POX_OK;
}

// ------------------------------------------------------------------------------------------
// context
// ------------------------------------------------------------------------------------------
extern "C" int pox_cuda_create(int device, pox_cuda_ctx** out) {
    if (!out) return set_error(POX_ERR_INVALID, "out is NULL");
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        return set_error(POX_ERR_UNSUPPORTED, "no CUDA device available");
    }
    if (device < 0 || device >= n) return set_error(POX_ERR_INVALID, "device %d out of range (%d devices)", device, n);
    CK(cudaSetDevice(device), "cudaSetDevice");
    cudaDeviceProp prop;
    CK(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
    if (prop.major != 10)
        return set_error(POX_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a", device,
                         prop.major, prop.minor);
    auto* c = new pox_cuda_ctx();
    c->device = device;
    c->num_sms = prop.multiProcessorCount;
    cudaError_t e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        delete c;
        return cuda_error(e, "cudaStreamCreate");
    }
    // kernel error flag (bounded waits that expired), mapped so the host reads it without a copy
    e = cudaHostAlloc((void**)&c->err_host, sizeof(int), cudaHostAllocMapped);
    if (e == cudaSuccess) e = cudaHostGetDevicePointer((void**)&c->err_dev, c->err_host, 0);
    if (e != cudaSuccess) {
        cudaStreamDestroy(c->stream);
        delete c;
        return cuda_error(e, "cudaHostAlloc(error flag)");
    }
    *c->err_host = 0;
    *out = c;
    return POX_OK;
}

static void free_tensor_mem(pox_tensor* t) {
    if (!t) return;
    if (t->host_graph) cudaGraphExecDestroy(t->host_graph);
    t->host_graph = nullptr;
    cudaFree(t->w);
    cudaFree(t->scales_dev);
    cudaFree(t->row_ptr);
    cudaFree(t->entries);
    cudaFree(t->vals);
    cudaFree(t->tile_ptr);
    cudaFree(t->tile_ent);
    cudaFree(t->scratch);
    cudaFree(t->row_scales);
    t->scratch = nullptr;
    t->row_scales = nullptr;
    t->w = t->scales_dev = nullptr;
    t->row_ptr = nullptr;
    t->entries = nullptr;
    t->vals = nullptr;
    t->tile_ptr = nullptr;
    t->tile_ent = nullptr;
}

extern "C" void pox_cuda_destroy(pox_cuda_ctx* ctx) {
    if (!ctx) return;
    pox::destroy_ctx_extras(ctx);  // models still alive (they own resident tensors of this context)
    {
        std::lock_guard<std::mutex> lk(ctx->mu);
        cudaSetDevice(ctx->device);
        cudaStreamSynchronize(ctx->stream);
        for (pox_tensor* t : ctx->tensors) {
            free_tensor_mem(t);
            delete t;
        }
        ctx->tensors.clear();
        ctx->by_host.clear();
        cudaFreeHost(ctx->pin_x);
        cudaFreeHost(ctx->pin_y);
        cudaFree(ctx->scratch_x);
        cudaFree(ctx->scratch_y);
        cudaFree(ctx->tc_scratch);
        cudaFree(ctx->tc_tickets);
        cudaFree(ctx->attn_scratch);
        cudaFreeHost(ctx->err_host);
        cudaStreamDestroy(ctx->stream);
    }
    pox::noalloc_forget_device(ctx->device);
    delete ctx;
}

int pox::take_kernel_error(pox_cuda_ctx* ctx) {
    const int f = *(volatile int*)ctx->err_host;
    if (f == 0) return POX_OK;
    *(volatile int*)ctx->err_host = 0;
    if ((f & ~kErrInputMask) == 0)
        return set_error(POX_ERR_INVALID, "attention input rejected on the device (flag 0x%x:%s%s); results of that call "
                         "are invalid", f, (f & kErrAttnPos) ? " a position beyond its block table" : "",
                         (f & kErrAttnPage) ? " a block-table entry outside [0, kv_blocks)" : "");
    return set_error(POX_ERR_TIMEOUT, "a kernel's bounded wait expired (flag 0x%x); results of that call are invalid", f);
}

extern "C" int pox_cuda_synchronize(pox_cuda_ctx* ctx) {
    if (!ctx) return set_error(POX_ERR_INVALID, "ctx is NULL");
    CK(cudaSetDevice(ctx->device), "cudaSetDevice");
    CK(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
    return take_kernel_error(ctx);
}

extern "C" void* pox_cuda_stream(pox_cuda_ctx* ctx) { return ctx ? (void*)ctx->stream : nullptr; }

int pox::ensure_scratch(pox_cuda_ctx* ctx, size_t xbytes, size_t ybytes) {
    if (xbytes > ctx->scratch_x_bytes) {
        cudaFree(ctx->scratch_x);
        ctx->scratch_x = nullptr;
        ctx->scratch_x_bytes = 0;
        CK(cudaMalloc(&ctx->scratch_x, xbytes), "cudaMalloc(x scratch)");
        ctx->scratch_x_bytes = xbytes;
    }
    if (ybytes > ctx->scratch_y_bytes) {
        cudaFree(ctx->scratch_y);
        ctx->scratch_y = nullptr;
        ctx->scratch_y_bytes = 0;
        CK(cudaMalloc(&ctx->scratch_y, ybytes), "cudaMalloc(y scratch)");
        ctx->scratch_y_bytes = ybytes;
    }
    return POX_OK;
}

// ------------------------------------------------------------------------------------------
// tensors
// ------------------------------------------------------------------------------------------
static inline size_t div_ceil(size_t a, size_t b) { return (a + b - 1) / b; }

static float h2f(uint16_t b) {
    __half_raw r;
    r.x = b;
    return __half2float(__half(r));
}

// Validation shared by the upload and the host-slice entry points (metal_backend.rs:95-108,
// kernels.rs:237-241).
static int validate_desc(const pox_tensor_desc* d) {
    if (!d) return set_error(POX_ERR_INVALID, "desc is NULL");
    if (d->rows == 0 || d->cols == 0) return POX_OK;
    if (!d->data) return set_error(POX_ERR_INVALID, "data is NULL");
    if (d->rows > 0x7FFFFFFF || d->cols > 0x7FFFFFFF)
        return set_error(POX_ERR_UNSUPPORTED, "dimension beyond 2^31");
    switch (d->dtype) {
        case POX_I4: {
            if (d->group_size == 0) return set_error(POX_ERR_LAYOUT, "INT4 group_size is 0");
            if (d->group_size % 2 != 0)
                return set_error(POX_ERR_UNSUPPORTED, "odd INT4 group size %zu", d->group_size);
            const size_t req_s = d->rows * div_ceil(d->cols, d->group_size) * 4;
            const size_t req_w = d->rows * div_ceil(d->cols, 2);
            if (d->scale_len < req_s || d->data_len < req_w || (!d->scales && req_s))
                return set_error(POX_ERR_LAYOUT, "Buffer layout incompatible with 2D GEMV (need %zu weight bytes, %zu "
                                 "scale bytes; got %zu, %zu)", req_w, req_s, d->data_len, d->scale_len);
            return POX_OK;
        }
        case POX_I8:
            if (d->group_size > 1)
                return set_error(POX_ERR_UNSUPPORTED, "INT8 group_size %zu: 0 (per-tensor f32 scale) or 1 (f16 scale "
                                 "per row)", d->group_size);
            if (d->data_len < d->rows * d->cols || !d->scales || d->scale_len < (d->group_size == 1 ? 2 * d->rows : 4))
                return set_error(POX_ERR_LAYOUT, "GEMV INT8 dimension mismatch");
            return POX_OK;
        case POX_F16:
            if (d->data_len < d->rows * d->cols * 2) return set_error(POX_ERR_LAYOUT, "F16 weight buffer too small");
            return POX_OK;
        default:
            return set_error(POX_ERR_UNSUPPORTED, "dtype %d not supported", d->dtype);
    }
}

// Builds the per-row CSR of an INT4 outlier table. Entries are applied in table order by the
// reference (kernels.rs:211-219), so for a repeated slot the last entry wins. The stored
// correction is v - dequant(q): adding corr * x to the tiled GEMV reproduces "replace".
static bool is_device_memory(const void* p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice;
}

static int build_outlier_csr(const pox_tensor_desc* d, std::vector<uint32_t>& row_ptr, std::vector<uint32_t>& cols,
                             std::vector<float>& corr, std::vector<uint16_t>& vals) {
    row_ptr.assign(d->rows + 1, 0);
    cols.clear();
    corr.clear();
    vals.clear();
    if (!d->outliers || d->outlier_len < 4) return POX_OK;  // outlier.rs:113-115
    if (is_device_memory(d->outliers) || is_device_memory(d->data) || is_device_memory(d->scales))
        return set_error(POX_ERR_UNSUPPORTED, "a tensor with an outlier table needs its payloads in host memory");
    const uint8_t* b = d->outliers;
    const uint64_t count = (uint64_t)b[0] | ((uint64_t)b[1] << 8) | ((uint64_t)b[2] << 16) | ((uint64_t)b[3] << 24);
    if (4 + 6 * count > d->outlier_len)
        return set_error(POX_ERR_LAYOUT, "outlier table truncated: %llu entries need %llu bytes, have %zu",
                         (unsigned long long)count, (unsigned long long)(4 + 6 * count), d->outlier_len);
    const uint64_t numel = (uint64_t)d->rows * d->cols;
    if (numel > 0xFFFFFFFFull && count)
        return set_error(POX_ERR_UNSUPPORTED, "outlier indices of a tensor beyond 2^32 elements");
    struct E { uint32_t row, col, order; uint16_t val; };
    std::vector<E> es;
    es.reserve(count);
    for (uint64_t i = 0; i < count; i++) {
        const uint8_t* p = b + 4 + 4 * i;
        const uint32_t idx = (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
        const uint8_t* pv = b + 4 + 4 * count + 2 * i;
        const uint16_t v = (uint16_t)(pv[0] | (pv[1] << 8));
        if ((uint64_t)idx >= numel) continue;
        es.push_back({(uint32_t)(idx / d->cols), (uint32_t)(idx % d->cols), (uint32_t)i, v});
    }
    std::sort(es.begin(), es.end(), [](const E& a, const E& b) {
        if (a.row != b.row) return a.row < b.row;
        if (a.col != b.col) return a.col < b.col;
        return a.order < b.order;
    });
    const size_t row_bytes = div_ceil(d->cols, 2);
    const size_t gpr = div_ceil(d->cols, d->group_size);
    for (size_t i = 0; i < es.size(); i++) {
        if (i + 1 < es.size() && es[i + 1].row == es[i].row && es[i + 1].col == es[i].col) continue;  // last wins
        const E& e = es[i];
        const uint8_t byte = d->data[(size_t)e.row * row_bytes + e.col / 2];
        const uint32_t q = (e.col & 1) ? (byte >> 4) : (byte & 15u);
        const uint8_t* sp = d->scales + ((size_t)e.row * gpr + e.col / d->group_size) * 4;
        const float sc = h2f((uint16_t)(sp[0] | (sp[1] << 8)));
        const float mn = h2f((uint16_t)(sp[2] | (sp[3] << 8)));
        volatile float t = (float)q * sc;  // dequantize_int4_group: mul, then add (kernels.rs:118)
        const float deq = mn + t;
        row_ptr[e.row + 1]++;
        cols.push_back(e.col);
        corr.push_back(h2f(e.val) - deq);
        vals.push_back(e.val);
    }
    for (size_t r = 0; r < d->rows; r++) row_ptr[r + 1] += row_ptr[r];
    return POX_OK;
}

template <class T>
static int upload_vec(const std::vector<T>& v, void** dst, size_t* bytes, cudaStream_t st) {
    if (v.empty()) return POX_OK;
    CK(cudaMalloc(dst, v.size() * sizeof(T)), "cudaMalloc(outliers)");
    CK(cudaMemcpyAsync(*dst, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice, st), "cudaMemcpy(outliers)");
    *bytes += v.size() * sizeof(T);
    return POX_OK;
}

int pox::upload_tensor_locked(pox_cuda_ctx* ctx, const pox_tensor_desc* d, pox_tensor** out, bool keep) {
    int rc = validate_desc(d);
    if (rc) return rc;
    auto* t = new pox_tensor();
    t->dtype = d->dtype;
    t->rows = d->rows;
    t->cols = d->cols;
    t->gs = d->group_size;
    t->h_data = d->data;
    t->h_data_len = d->data_len;
    t->h_scales = d->scales;
    t->h_scale_len = d->scale_len;
    t->h_outliers = d->outliers;
    t->h_outlier_len = d->outlier_len;
    if (d->rows == 0 || d->cols == 0) {
        if (keep) {
            ctx->tensors.push_back(t);
            ctx->by_host.emplace(t->h_data, t);
        }
        *out = t;
        return POX_OK;
    }
    cudaStream_t st = ctx->stream;
    const int N = (int)d->rows, K = (int)d->cols;
    void* tmp = nullptr;
    void* tmp_s = nullptr;
    auto fail = [&](int code) {
        cudaStreamSynchronize(st);
        cudaFree(tmp);
        cudaFree(tmp_s);
        free_tensor_mem(t);
        delete t;
        return code;
    };
#define CKF(call, what)                                          \
    do {                                                         \
        cudaError_t _e = (call);                                 \
        if (_e != cudaSuccess) return fail(cuda_error(_e, what)); \
    } while (0)

    if (d->dtype == POX_I4) {
        const size_t raw_bytes = d->rows * div_ceil(d->cols, 2);
        const size_t groups = div_ceil(d->cols, d->group_size);
        const size_t sbytes = d->rows * groups * 4;
        t->groups = (int)groups;
        t->tiled = (K % 128 == 0) && (d->group_size % 128 == 0);
        CKF(cudaMalloc(&tmp, raw_bytes), "cudaMalloc(raw)");
        CKF(cudaMemcpyAsync(tmp, d->data, raw_bytes, cudaMemcpyDefault, st), "cudaMemcpy(raw)");
        if (t->tiled) {
            const TileLayout TL(kKindI4, N, K);
            CKF(cudaMalloc(&t->w, TL.bytes()), "cudaMalloc(tiles)");
            CKF(launch_repack(kKindI4, (const uint8_t*)tmp, (uint8_t*)t->w, N, K, st), "repack_i4");
            CKF(cudaMalloc(&tmp_s, sbytes), "cudaMalloc(raw scales)");
            CKF(cudaMemcpyAsync(tmp_s, d->scales, sbytes, cudaMemcpyDefault, st), "cudaMemcpy(scales)");
            CKF(launch_repack_i4_scales((const uint8_t*)tmp_s, (uint8_t*)t->w, N, K, (int)d->group_size, st),
                "repack_i4_scales");
            t->bytes += TL.bytes();
        } else {
            t->w = tmp;
            tmp = nullptr;
            t->bytes += raw_bytes;
            CKF(cudaMalloc(&t->scales_dev, sbytes), "cudaMalloc(scales)");
            CKF(cudaMemcpyAsync(t->scales_dev, d->scales, sbytes, cudaMemcpyDefault, st), "cudaMemcpy(scales)");
            t->bytes += sbytes;
        }
        std::vector<uint32_t> rp, cols;
        std::vector<float> corr;
        std::vector<uint16_t> vals;
        rc = build_outlier_csr(d, rp, cols, corr, vals);
        if (rc) return fail(rc);
        if (!cols.empty()) {
            std::vector<uint2> ent(cols.size());
            for (size_t i = 0; i < cols.size(); i++) {
                uint32_t cb;
                std::memcpy(&cb, &corr[i], 4);
                ent[i] = make_uint2(cols[i], cb);
            }
            t->nnz = cols.size();
            if ((rc = upload_vec(rp, (void**)&t->row_ptr, &t->bytes, st))) return fail(rc);
            if ((rc = upload_vec(vals, (void**)&t->vals, &t->bytes, st))) return fail(rc);
            ent.push_back(make_uint2(0u, 0u));  // padding: the GEMV copies entries in 16-byte pairs
            ent.push_back(make_uint2(0u, 0u));
            if ((rc = upload_vec(ent, (void**)&t->entries, &t->bytes, st))) return fail(rc);
            std::vector<uint32_t> tptr, tent;
            if (t->tiled) {  // the same entries by (row tile, 128-k block), for the small-M path
                const size_t nT = div_ceil(N, 16), nkb = K / 128;
                tptr.assign(nT * nkb + 1, 0);
                for (size_t r = 0; r < (size_t)N; r++)
                    for (uint32_t e = rp[r]; e < rp[r + 1]; e++) tptr[(r / 16) * nkb + cols[e] / 128 + 1]++;
                for (size_t i = 0; i + 1 < tptr.size(); i++) tptr[i + 1] += tptr[i];
                tent.resize(cols.size());
                std::vector<uint32_t> fill(tptr.begin(), tptr.end() - 1);
                for (size_t r = 0; r < (size_t)N; r++)
                    for (uint32_t e = rp[r]; e < rp[r + 1]; e++)
                        tent[fill[(r / 16) * nkb + cols[e] / 128]++] =
                            (uint32_t)(r & 15) | ((cols[e] & 127u) << 4) | ((uint32_t)vals[e] << 16);
                if ((rc = upload_vec(tptr, (void**)&t->tile_ptr, &t->bytes, st))) return fail(rc);
                if ((rc = upload_vec(tent, (void**)&t->tile_ent, &t->bytes, st))) return fail(rc);
            }
            // the host vectors must outlive the async copies
            CKF(cudaStreamSynchronize(st), "cudaStreamSynchronize(upload)");
        }
    } else if (d->dtype == POX_I8) {
        if (d->group_size == 1) {  // f16 scale per output row (the per-channel extension)
            std::vector<uint16_t> sh(d->rows);
            std::vector<float> sf(d->rows);
            CKF(cudaMemcpy(sh.data(), d->scales, 2 * d->rows, cudaMemcpyDefault), "cudaMemcpy(int8 row scales)");
            for (size_t r = 0; r < d->rows; r++) sf[r] = h2f(sh[r]);
            CKF(cudaMalloc(&t->row_scales, d->rows * sizeof(float)), "cudaMalloc(int8 row scales)");
            CKF(cudaMemcpy(t->row_scales, sf.data(), d->rows * sizeof(float), cudaMemcpyHostToDevice),
                "cudaMemcpy(int8 row scales)");
            t->bytes += d->rows * sizeof(float);
            t->i8_scale = 1.0f;
        } else {
            CKF(cudaMemcpy(&t->i8_scale, d->scales, 4, cudaMemcpyDefault), "cudaMemcpy(int8 scale)");  // one f32 LE (kernels.rs:150-151)
        }
        const size_t raw_bytes = d->rows * d->cols;
        t->tiled = (K % 64 == 0);
        CKF(cudaMalloc(&tmp, raw_bytes), "cudaMalloc(raw)");
        CKF(cudaMemcpyAsync(tmp, d->data, raw_bytes, cudaMemcpyDefault, st), "cudaMemcpy(raw)");
        if (t->tiled) {
            const size_t tiles_bytes = TileLayout(kKindI8, N, K).bytes();
            CKF(cudaMalloc(&t->w, tiles_bytes), "cudaMalloc(tiles)");
            CKF(launch_repack(kKindI8, (const uint8_t*)tmp, (uint8_t*)t->w, N, K, st), "repack_i8");
            t->bytes += tiles_bytes;
        } else {
            t->w = tmp;
            tmp = nullptr;
            t->bytes += raw_bytes;
        }
    } else {  // F16
        const size_t raw_bytes = d->rows * d->cols * 2;
        t->tiled = (K % 32 == 0);
        CKF(cudaMalloc(&tmp, raw_bytes), "cudaMalloc(raw)");
        CKF(cudaMemcpyAsync(tmp, d->data, raw_bytes, cudaMemcpyDefault, st), "cudaMemcpy(raw)");
        if (t->tiled) {
            const size_t tiles_bytes = TileLayout(kKindF16, N, K).bytes();
            CKF(cudaMalloc(&t->w, tiles_bytes), "cudaMalloc(tiles)");
            CKF(launch_repack(kKindF16, (const uint8_t*)tmp, (uint8_t*)t->w, N, K, st), "repack_f16");
            t->bytes += tiles_bytes;
        } else {
            t->w = tmp;
            tmp = nullptr;
            t->bytes += raw_bytes;
        }
    }
    if (t->tiled) {
        const int kind = d->dtype == POX_I4 ? kKindI4 : (d->dtype == POX_I8 ? kKindI8 : kKindF16);
        const size_t sb = xprep_bytes(kind, K);
        CKF(cudaMalloc(&t->scratch, sb), "cudaMalloc(prepared x)");
        t->scratch_bytes = sb;
        t->bytes += sb;
    }
    CKF(cudaStreamSynchronize(st), "cudaStreamSynchronize(upload)");
    cudaFree(tmp);
    cudaFree(tmp_s);
#undef CKF
    if (keep) {
        ctx->tensors.push_back(t);
        ctx->by_host.emplace(t->h_data, t);
    }
    *out = t;
    return POX_OK;
}

extern "C" int pox_cuda_tensor_upload(pox_cuda_ctx* ctx, const pox_tensor_desc* desc, pox_tensor** out) {
    if (!ctx || !out) return set_error(POX_ERR_INVALID, "ctx/out is NULL");
    *out = nullptr;
    std::lock_guard<std::mutex> lk(ctx->mu);
    CK(cudaSetDevice(ctx->device), "cudaSetDevice");
    return upload_tensor_locked(ctx, desc, out, true);
}

extern "C" int pox_cuda_tensor_free(pox_cuda_ctx* ctx, pox_tensor* t) {
    if (!t) return POX_OK;
    if (!ctx) return set_error(POX_ERR_INVALID, "ctx is NULL");
    std::lock_guard<std::mutex> lk(ctx->mu);
    auto it = std::find(ctx->tensors.begin(), ctx->tensors.end(), t);
    if (it == ctx->tensors.end()) return set_error(POX_ERR_INVALID, "tensor does not belong to this context");
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    ctx->tensors.erase(it);
    for (auto r = ctx->by_host.equal_range(t->h_data); r.first != r.second; ++r.first)
        if (r.first->second == t) {
            ctx->by_host.erase(r.first);
            break;
        }
    free_tensor_mem(t);
    delete t;
    return POX_OK;
}

extern "C" int pox_cuda_tensor_info(const pox_tensor* t, size_t* rows, size_t* cols, size_t* outlier_count,
                                    size_t* device_bytes) {
    if (!t) return set_error(POX_ERR_INVALID, "tensor is NULL");
    if (rows) *rows = t->rows;
    if (cols) *cols = t->cols;
    if (outlier_count) *outlier_count = t->nnz;
    if (device_bytes) *device_bytes = t->bytes;
    return POX_OK;
}

extern "C" const char* pox_cuda_tensor_gemv_kernel(const pox_tensor* t, size_t batch) {
    if (!t) return nullptr;
    if (!t->tiled) return "gemv_generic";
    if (batch == 0 || !gemv_uses_small_m(t, batch)) return "gemv_tc_kernel";
    const int kind = t->dtype == POX_I4 ? kKindI4 : (t->dtype == POX_I8 ? kKindI8 : kKindF16);
    return tq_supported(kind, t->nnz > 0, tc05_pad((int)std::min<size_t>(batch, 128))) ? "gemm_tq_kernel"
                                                                                       : "gemm_tc05_kernel";
}

// ------------------------------------------------------------------------------------------
// GEMV
// ------------------------------------------------------------------------------------------
// Small-M scratch: prepared x (the f16 layout or the integer path's limbs and block meta, whichever
// is larger), 256 row scales, then the k-split partials.
static size_t tc_x_region(size_t cols, int Bp) {
    return (std::max(pox::tc05_x_bytes((int)cols, Bp), pox::tq_x_bytes((int)cols, Bp)) + 255) & ~(size_t)255;
}
static size_t tc_bytes(size_t rows, size_t cols, int Bp, int S) {
    return tc_x_region(cols, Bp) + 256 * sizeof(float) + (S > 1 ? (size_t)S * Bp * rows * sizeof(float) : 0);
}

int pox::ensure_tc_scratch(pox_cuda_ctx* ctx, size_t rows, size_t cols, size_t batch, cudaStream_t st) {
    const int Bp = tc05_pad((int)std::min<size_t>(batch, 128));
    const int nrb = (int)((rows + 127) / 128);
    const int S = tc05_splits(nrb, (int)(cols / 128), ctx->num_sms);
    const size_t need = tc_bytes(rows, cols, Bp, S);
    const bool grow = need > ctx->tc_scratch_bytes || (size_t)nrb > ctx->tc_tickets_n;
    if (!grow) return POX_OK;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (st && cudaStreamIsCapturing(st, &cs) == cudaSuccess && cs != cudaStreamCaptureStatusNone)
        return set_error(POX_ERR_INVALID, "small-M scratch must be sized by a call before stream capture");
    CK(cudaStreamSynchronize(st ? st : ctx->stream), "cudaStreamSynchronize");
    if (need > ctx->tc_scratch_bytes) {
        cudaFree(ctx->tc_scratch);
        ctx->tc_scratch = nullptr;
        ctx->tc_scratch_bytes = 0;
        const size_t bytes = std::max(need, (size_t)64 << 20);
        CK(cudaMalloc(&ctx->tc_scratch, bytes), "cudaMalloc(small-M scratch)");
        CK(cudaMemset(ctx->tc_scratch, 0, bytes), "cudaMemset(small-M scratch)");
        ctx->tc_scratch_bytes = bytes;
    }
    if ((size_t)nrb > ctx->tc_tickets_n) {
        cudaFree(ctx->tc_tickets);
        ctx->tc_tickets = nullptr;
        ctx->tc_tickets_n = 0;
        const size_t n = std::max<size_t>(nrb, 4096);
        CK(cudaMalloc(&ctx->tc_tickets, n * sizeof(int)), "cudaMalloc(tickets)");
        CK(cudaMemset(ctx->tc_tickets, 0, n * sizeof(int)), "cudaMemset(tickets)");
        ctx->tc_tickets_n = n;
    }
    return POX_OK;
}

// Small-M path: up to 128 rows of x per launch pair (x preparation + tcgen05 GEMM).
static int tc05_gemv(pox_cuda_ctx* ctx, const pox_tensor* t, int kind, const float* x, size_t batch, float* y,
                     cudaStream_t st, const PrepOp& op, const float* resid, bool prepared) {
    const int N = (int)t->rows, K = (int)t->cols;
    const size_t ldx = op.ld_x ? (size_t)op.ld_x : t->cols;
    int rc = ensure_tc_scratch(ctx, t->rows, t->cols, batch, st);
    if (rc) return rc;
    const int nrb = (N + 127) / 128;
    const int S = tc05_splits(nrb, K / 128, ctx->num_sms);
    size_t done = 0;
    while (done < batch) {
        const int b = (int)std::min<size_t>(batch - done, 128);
        const int Bp = tc05_pad(b);
        uint8_t* xs = static_cast<uint8_t*>(ctx->tc_scratch);
        const size_t xsb = tc_x_region(K, Bp);
        float* xscale = reinterpret_cast<float*>(xs + xsb);
        float* ws = xscale + 256;
        PrepOp opb = op;
        if (opb.up) opb.up += done * (size_t)opb.ld_up;
        cudaError_t e = cudaSuccess;
        if (tq_supported(kind, t->nnz > 0, Bp)) {
            // integer tensor cores: x as exact int8 limbs of 128-k blocks, prepared here or by the
            // caller at gemv_x_target's xl / xm
            float2* xm = reinterpret_cast<float2*>(xs + (((size_t)(K / 128) * 2 * Bp * 128 + 255) & ~(size_t)255));
            if (!prepared) {
                e = launch_xprep_tq(x + done * ldx, b, Bp, K, opb, xs, xm, st);
                if (e != cudaSuccess) return cuda_error(e, "x preparation launch");
            }
            TqArgs q = {};
            q.w = (const uint8_t*)t->w;
            q.xl = xs;
            q.xm = xm;
            q.wscale = kind == kKindI8 ? t->i8_scale : 1.0f;
            q.row_scale = kind == kKindI8 ? t->row_scales : nullptr;
            q.y = y + done * t->rows;
            q.resid = resid ? resid + done * t->rows : nullptr;
            q.ws = ws;
            q.tickets = ctx->tc_tickets;
            q.err = ctx->err_dev;
            q.Nout = N;
            q.K = K;
            q.nkb = K / 128;
            q.nT = (N + 15) / 16;
            q.B = b;
            q.Bp = Bp;
            q.S = S;
            e = launch_tq(kind, q, st);
            if (e != cudaSuccess) return cuda_error(e, "small-M GEMM launch");
            done += b;
            continue;
        }
        if (!prepared) {
            e = launch_xprep_tc05(x + done * ldx, b, Bp, K, opb, xs, xscale, st);
            if (e != cudaSuccess) return cuda_error(e, "x preparation launch");
        }
        TcArgs a = {};
        a.w = (const uint8_t*)t->w;
        a.tile_ptr = kind == kKindI4 ? t->tile_ptr : nullptr;
        a.tile_ent = t->tile_ent;
        a.nnz = (uint32_t)t->nnz;
        a.xs = xs;
        a.xscale = xscale;
        a.wscale = kind == kKindI8 ? t->i8_scale : 1.0f;
        a.row_scale = kind == kKindI8 ? t->row_scales : nullptr;
        a.y = y + done * t->rows;
        a.resid = resid ? resid + done * t->rows : nullptr;
        a.ws = ws;
        a.tickets = ctx->tc_tickets;
        a.err = ctx->err_dev;
        a.Nout = N;
        a.K = K;
        a.nkb = K / 128;
        a.nT = (N + 15) / 16;
        a.B = b;
        a.Bp = Bp;
        a.S = S;
        e = launch_tc05(kind, a, st);
        if (e != cudaSuccess) return cuda_error(e, "small-M GEMM launch");
        done += b;
    }
    return POX_OK;
}

// Batches above this use the small-M tensor-core path (when the tensor qualifies).
static int tc05_min_batch() {
    static const int v = [] {
        const char* s = getenv("POX_TC05_MIN_BATCH");
        return s ? std::max(1, atoi(s)) : kMaxBatch + 1;
    }();
    return v;
}

// Batches <= 8 that the integer small-M kernel (padded to 16 rows) serves faster than the batch
// <= 8 GEMV, measured on B200 (us per call, GEMV vs integer kernel):
//  * INT4 without outliers, K >= 8192, batch >= 6: the GEMV stages 2 K bytes of x per row in shared
//    memory and loses occupancy (4096 x 14336: 27.2 vs 20.8 at batch 6, 26.8 vs 20.9 at 8). With
//    K = 4096 the GEMV keeps up or wins (6144 x 4096 at batch 6: 8.4 vs 13.1).
//  * INT8 with at least 16 M weights, batch >= 2 (14336 x 4096: 20.0 vs 17.9 at batch 2, 30.0 vs
//    18.0 at 8).
static bool tq_below_9(const pox_tensor* t, int kind, size_t batch) {
    if (!tq_supported(kind, t->nnz > 0, 16)) return false;
    if (kind == kKindI4) return batch >= 6 && t->cols >= 8192;
    return batch >= 2 && t->rows * t->cols >= ((size_t)16 << 20);
}

bool pox::gemv_uses_small_m(const pox_tensor* t, size_t batch) {
    // the x preparation stages one row (cols floats) in shared memory
    if (!(t->tiled && t->cols % 128 == 0 && t->cols <= 53248)) return false;
    if (batch >= (size_t)tc05_min_batch()) return true;
    const int kind = t->dtype == POX_I4 ? kKindI4 : (t->dtype == POX_I8 ? kKindI8 : kKindF16);
    return kind != kKindF16 && tq_below_9(t, kind, batch);
}

int pox::gemv_x_target(pox_cuda_ctx* ctx, const pox_tensor* t, size_t batch, cudaStream_t st, XTarget* out) {
    *out = XTarget();
    if (!t->tiled || t->dtype != POX_I4 || t->cols % 128 != 0) return set_error(POX_ERR_UNSUPPORTED, "no prepared-x path");
    if (gemv_uses_small_m(t, batch)) {
        if (batch > 128) return set_error(POX_ERR_UNSUPPORTED, "prepared x holds up to 128 rows");
        int rc = ensure_tc_scratch(ctx, t->rows, t->cols, batch, st);
        if (rc) return rc;
        out->Bp = tc05_pad((int)batch);
        if (tq_supported(kKindI4, t->nnz > 0, out->Bp)) {  // as tc05_gemv's integer branch places them
            out->xl = static_cast<uint8_t*>(ctx->tc_scratch);
            out->xm = reinterpret_cast<float2*>(out->xl + (((t->cols / 128) * 2 * (size_t)out->Bp * 128 + 255) & ~(size_t)255));
            return POX_OK;
        }
        out->xs = static_cast<uint8_t*>(ctx->tc_scratch);
        out->xscale = reinterpret_cast<float*>(out->xs + tc_x_region(t->cols, out->Bp));  // as tc05_gemv places them
        return POX_OK;
    }
    if (batch > (size_t)kMaxBatch) return set_error(POX_ERR_UNSUPPORTED, "prepared x holds up to 8 rows");
    const XPrep xp = xprep_view(t->scratch, kKindI4, (int)t->cols);
    out->cols = static_cast<uint8_t*>(xp.cols);
    out->meta = xp.meta;
    out->Kp = xp.Kp;
    out->nxbs = xp.nxbs;
    return POX_OK;
}

int pox::gemv_launch(pox_cuda_ctx* ctx, const pox_tensor* t, const float* x, size_t batch, float* y,
                     cudaStream_t st, const PrepOp* op_in, const float* resid, bool prepared) {
    if (t->rows == 0 || t->cols == 0 || batch == 0) return POX_OK;
    if (((uintptr_t)x & 15) != 0) return set_error(POX_ERR_INVALID, "x must be 16-byte aligned");
    const PrepOp op = op_in ? *op_in : PrepOp();
    if ((op.mode != kPrepNone || resid) && !t->tiled)
        return set_error(POX_ERR_UNSUPPORTED, "fused pre-ops need a tensor in the tiled layout");
    const int kind = t->dtype == POX_I4 ? kKindI4 : (t->dtype == POX_I8 ? kKindI8 : kKindF16);
    const int N = (int)t->rows, K = (int)t->cols;
    (void)K;
    if (prepared && (op.mode != kPrepNone || batch > (gemv_uses_small_m(t, batch) ? 128u : (size_t)kMaxBatch)))
        return set_error(POX_ERR_INVALID, "prepared x: no pre-op, at most one launch of rows");
    if (gemv_uses_small_m(t, batch)) return tc05_gemv(ctx, t, kind, x, batch, y, st, op, resid, prepared);
    const size_t ldx = op.ld_x ? (size_t)op.ld_x : t->cols;
    size_t done = 0;
    while (done < batch) {
        size_t b = std::min<size_t>(batch - done, 8);
        const float* xb = x + done * ldx;
        float* yb = y + done * t->rows;
        PrepOp opb = op;
        if (opb.up) opb.up += done * (size_t)opb.ld_up;
        cudaError_t e;
        if (t->tiled) {
            const TileLayout TL(kind, N, K);
            const XPrep xp = xprep_view(t->scratch, kind, K);
            if (!prepared) {
                e = launch_xprep(kind, xb, (int)b, K, xp, opb, true, st);
                if (e != cudaSuccess) return cuda_error(e, "x preparation launch");
            }
            GemvArgs a = {};
            a.w = (const uint8_t*)t->w;
            a.i8_scale = t->i8_scale;
            a.row_scale = t->row_scales;
            a.row_ptr = kind == kKindI4 ? t->row_ptr : nullptr;
            a.ent = t->entries;
            a.xq = xp.cols;
            a.xm = xp.meta;
            a.x = xb;
            a.resid = resid ? resid + done * t->rows : nullptr;
            a.y = yb;
            a.N = N;
            a.K = K;
            a.Kp = xp.Kp;
            a.B = (int)b;
            a.nxb = xp.nxb;
            a.nxbs = xp.nxbs;
            a.err = ctx->err_dev;
            a.nT = TL.nT;
            a.nkb = TL.nkb;
            a.S = 1;
            e = launch_gemv_tc(kind, a, true, st);
        } else {
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
            a.B = (int)b;
            a.gs = (int)t->gs;
            a.groups = t->groups;
            e = launch_gemv_generic(kind, a, st);
        }
        if (e != cudaSuccess) return cuda_error(e, "gemv launch");
        done += b;
    }
    return POX_OK;
}

extern "C" int pox_cuda_tensor_gemv(pox_cuda_ctx* ctx, const pox_tensor* t, const float* x_dev, size_t batch,
                                    float* y_dev, void* stream) {
    if (!ctx || !t) return set_error(POX_ERR_INVALID, "ctx/tensor is NULL");
    if (batch && (!x_dev || !y_dev)) return set_error(POX_ERR_INVALID, "x/y is NULL");
    CK(cudaSetDevice(ctx->device), "cudaSetDevice");
    cudaStream_t st = stream ? (cudaStream_t)stream : ctx->stream;
    return gemv_launch(ctx, t, x_dev, batch, y_dev, st);
}

extern "C" int pox_cuda_tensor_gemv_ex(pox_cuda_ctx* ctx, const pox_tensor* t, const float* x_dev, size_t batch,
                                       float* y_dev, const pox_gemv_op* op, const float* resid_dev, void* stream) {
    if (!ctx || !t) return set_error(POX_ERR_INVALID, "ctx/tensor is NULL");
    if (batch && (!x_dev || !y_dev)) return set_error(POX_ERR_INVALID, "x/y is NULL");
    PrepOp p;
    if (op) {
        if (op->mode < POX_OP_NONE || op->mode > POX_OP_SWIGLU) return set_error(POX_ERR_INVALID, "bad op mode");
        if (op->mode == POX_OP_SWIGLU && !op->up) return set_error(POX_ERR_INVALID, "SwiGLU needs up");
        p.mode = op->mode == POX_OP_RMSNORM ? kPrepNorm : (op->mode == POX_OP_SWIGLU ? kPrepSwiGLU : kPrepNone);
        p.norm_w = op->norm_w;
        p.eps = op->eps;
        p.up = op->up;
        p.ld_x = (int)op->ld_x;
        p.ld_up = (int)(op->ld_up ? op->ld_up : (uint32_t)t->cols);
    }
    CK(cudaSetDevice(ctx->device), "cudaSetDevice");
    cudaStream_t st = stream ? (cudaStream_t)stream : ctx->stream;
    return gemv_launch(ctx, t, x_dev, batch, y_dev, st, &p, resid_dev);
}

static int ensure_pinned(float** host, float** dev, size_t* have, size_t need) {
    if (need <= *have) return POX_OK;
    cudaFreeHost(*host);
    *host = *dev = nullptr;
    *have = 0;
    CK(cudaHostAlloc((void**)host, need, cudaHostAllocMapped), "cudaHostAlloc(staging)");
    CK(cudaHostGetDevicePointer((void**)dev, *host, 0), "cudaHostGetDevicePointer(staging)");
    *have = need;
    return POX_OK;
}

// Host x in, host y out, synchronous. Caller holds ctx->mu.
// Tiled tensors: x is copied into pinned, device-mapped staging on the host and read from there over
// PCIe by the x preparation (once; the GEMV kernels read only the prepared x), and the GEMV writes y
// straight into pinned, device-mapped staging (each element once): no DMA copies, one stream sync.
// The raw-layout kernels re-read x for every row, so they get x and y in device memory.
static int gemv_host_locked(pox_cuda_ctx* ctx, const pox_tensor* t, const float* x, size_t batch, float* y) {
    if (t->rows == 0 || t->cols == 0 || batch == 0) return POX_OK;
    const size_t xb = batch * t->cols * sizeof(float), yb = batch * t->rows * sizeof(float);
    if (t->tiled) {
        int rc = ensure_pinned(&ctx->pin_x, &ctx->pin_x_dev, &ctx->pin_x_bytes, xb);
        if (!rc) rc = ensure_pinned(&ctx->pin_y, &ctx->pin_y_dev, &ctx->pin_y_bytes, yb);
        if (rc) return rc;
        std::memcpy(ctx->pin_x, x, xb);
        pox_tensor* tm = const_cast<pox_tensor*>(t);
        const bool cached = t->host_graph && t->host_graph_batch == batch && t->host_graph_x == ctx->pin_x_dev &&
                            t->host_graph_y == ctx->pin_y_dev;
        if (cached) {
            CK(cudaGraphLaunch(t->host_graph, ctx->stream), "cudaGraphLaunch");
        } else {
            rc = gemv_launch(ctx, t, ctx->pin_x_dev, batch, ctx->pin_y_dev, ctx->stream);
            if (rc) return rc;
        }
        CK(cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
        std::memcpy(y, ctx->pin_y, yb);
        rc = take_kernel_error(ctx);
        if (rc || cached || gemv_uses_small_m(t, batch)) return rc;  // (the small-M scratch is shared and regrown)
        // the next call of this batch replays the launches as one graph (captured now that every
        // buffer they use exists: the tensor's own x preparation and the staging; a failed capture
        // only means the next call launches them again)
        if (t->host_graph) cudaGraphExecDestroy(t->host_graph);
        tm->host_graph = nullptr;
        cudaGraph_t g = nullptr;
        if (cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
            const int crc = gemv_launch(ctx, t, ctx->pin_x_dev, batch, ctx->pin_y_dev, ctx->stream);
            const cudaError_t ce = cudaStreamEndCapture(ctx->stream, &g);
            if (!crc && ce == cudaSuccess && g && cudaGraphInstantiate(&tm->host_graph, g, 0) == cudaSuccess) {
                tm->host_graph_batch = batch;
                tm->host_graph_x = ctx->pin_x_dev;
                tm->host_graph_y = ctx->pin_y_dev;
            } else {
                tm->host_graph = nullptr;
            }
            if (g) cudaGraphDestroy(g);
        }
        cudaGetLastError();  // a failed capture leaves no error behind for the next call
        return POX_OK;
    }
    int rc = ensure_scratch(ctx, xb, yb);
    if (rc) return rc;
    CK(cudaMemcpyAsync(ctx->scratch_x, x, xb, cudaMemcpyHostToDevice, ctx->stream), "cudaMemcpy(x)");
    rc = gemv_launch(ctx, t, (const float*)ctx->scratch_x, batch, (float*)ctx->scratch_y, ctx->stream);
    if (rc) return rc;
    CK(cudaMemcpyAsync(y, ctx->scratch_y, yb, cudaMemcpyDeviceToHost, ctx->stream), "cudaMemcpy(y)");
    CK(cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
    return take_kernel_error(ctx);
}

extern "C" int pox_cuda_tensor_gemv_host(pox_cuda_ctx* ctx, const pox_tensor* t, const float* x, size_t batch,
                                         float* y) {
    if (!ctx || !t) return set_error(POX_ERR_INVALID, "ctx/tensor is NULL");
    if (batch && (!x || !y)) return set_error(POX_ERR_INVALID, "x/y is NULL");
    std::lock_guard<std::mutex> lk(ctx->mu);
    CK(cudaSetDevice(ctx->device), "cudaSetDevice");
    return gemv_host_locked(ctx, t, x, batch, y);
}

// The resident tensor uploaded from exactly these host slices (same addresses and lengths, shape,
// dtype, group size), looked up by the weight payload's address.
static pox_tensor* find_registered(pox_cuda_ctx* ctx, const pox_tensor_desc& d) {
    for (auto r = ctx->by_host.equal_range(d.data); r.first != r.second; ++r.first) {
        pox_tensor* t = r.first->second;
        if (t->dtype == d.dtype && t->h_data_len == d.data_len && t->h_scales == d.scales &&
            t->h_scale_len == d.scale_len && t->rows == d.rows && t->cols == d.cols &&
            (d.dtype != POX_I4 || (t->gs == d.group_size && t->h_outliers == d.outliers &&
                                   t->h_outlier_len == d.outlier_len)))
            return t;
    }
    return nullptr;
}

// Shared body of the reference-shaped host-slice entry points.
static int host_slice_gemv(pox_cuda_ctx* ctx, const pox_tensor_desc& d, const float* x, size_t x_len, float* y,
                           size_t y_len) {
    if (!ctx) return set_error(POX_ERR_INVALID, "ctx is NULL");
    if (d.rows == 0 || d.cols == 0) return POX_OK;  // metal_backend.rs:95-97
    int rc = validate_desc(&d);
    if (rc) return rc;
    if (!x || !y) return set_error(POX_ERR_INVALID, "x/y is NULL");
    if (x_len < d.cols || y_len < d.rows)
        return set_error(POX_ERR_LAYOUT, "GEMV dimension mismatch (x %zu < cols %zu or y %zu < rows %zu)", x_len,
                         d.cols, y_len, d.rows);
    std::lock_guard<std::mutex> lk(ctx->mu);
    CK(cudaSetDevice(ctx->device), "cudaSetDevice");
    pox_tensor* t = find_registered(ctx, d);
    if (t) return gemv_host_locked(ctx, t, x, 1, y);
    pox_tensor* tmp = nullptr;
    rc = upload_tensor_locked(ctx, &d, &tmp, false);
    if (rc) return rc;
    rc = gemv_host_locked(ctx, tmp, x, 1, y);
    cudaStreamSynchronize(ctx->stream);
    free_tensor_mem(tmp);
    delete tmp;
    return rc;
}

extern "C" int pox_cuda_gemv_int4(pox_cuda_ctx* ctx, const uint8_t* packed_weights, size_t packed_len,
                                  const uint8_t* scale_data, size_t scale_len, size_t rows, size_t cols,
                                  size_t group_size, const float* x, size_t x_len, float* y, size_t y_len) {
    pox_tensor_desc d = {};
    d.dtype = POX_I4;
    d.rows = rows;
    d.cols = cols;
    d.group_size = group_size;
    d.data = packed_weights;
    d.data_len = packed_len;
    d.scales = scale_data;
    d.scale_len = scale_len;
    return host_slice_gemv(ctx, d, x, x_len, y, y_len);
}

extern "C" int pox_cuda_gemv_int4_outliers(pox_cuda_ctx* ctx, const uint8_t* packed_weights, size_t packed_len,
                                           const uint8_t* scale_data, size_t scale_len, size_t group_size,
                                           size_t rows, size_t cols, const uint8_t* outlier_data, size_t outlier_len,
                                           const float* x, size_t x_len, float* y, size_t y_len) {
    pox_tensor_desc d = {};
    d.dtype = POX_I4;
    d.rows = rows;
    d.cols = cols;
    d.group_size = group_size;
    d.data = packed_weights;
    d.data_len = packed_len;
    d.scales = scale_data;
    d.scale_len = scale_len;
    d.outliers = outlier_data;
    d.outlier_len = outlier_data ? outlier_len : 0;
    return host_slice_gemv(ctx, d, x, x_len, y, y_len);
}

extern "C" int pox_cuda_gemv_int8(pox_cuda_ctx* ctx, const uint8_t* q_weights, size_t q_len,
                                  const uint8_t* scale_data, size_t scale_len, size_t rows, size_t cols,
                                  const float* x, size_t x_len, float* y, size_t y_len) {
    pox_tensor_desc d = {};
    d.dtype = POX_I8;
    d.rows = rows;
    d.cols = cols;
    d.data = q_weights;
    d.data_len = q_len;
    d.scales = scale_data;
    d.scale_len = scale_len;
    if (rows && cols && (x_len < cols || y_len < rows || q_len < rows * cols))
        return set_error(POX_ERR_LAYOUT, "GEMV INT8 dimension mismatch");
    return host_slice_gemv(ctx, d, x, x_len, y, y_len);
}

// ------------------------------------------------------------------------------------------
// dequantization (K0)
// ------------------------------------------------------------------------------------------
static int dequant_launch(const pox_tensor* t, float* out, cudaStream_t st) {
    if (t->rows == 0 || t->cols == 0) return POX_OK;
    const int N = (int)t->rows, K = (int)t->cols;
    cudaError_t e;
    if (t->dtype == POX_I4) {
        e = launch_dequant_i4(t->tiled, t->w, t->scales_dev, out, N, K, t->groups, (int)t->gs, st);
        if (e == cudaSuccess && t->nnz)
            e = launch_apply_outliers(t->row_ptr, t->entries, t->vals, out, N, K, st);
    } else if (t->dtype == POX_I8) {
        e = launch_dequant_i8(t->tiled, t->w, t->i8_scale, t->row_scales, out, N, K, st);
    } else {
        return set_error(POX_ERR_UNSUPPORTED, "dequantization of dtype %d", t->dtype);
    }
    if (e != cudaSuccess) return cuda_error(e, "dequant launch");
    return POX_OK;
}

extern "C" int pox_cuda_tensor_dequant(pox_cuda_ctx* ctx, const pox_tensor* t, float* out_dev, void* stream) {
    if (!ctx || !t || !out_dev) return set_error(POX_ERR_INVALID, "NULL argument");
    CK(cudaSetDevice(ctx->device), "cudaSetDevice");
    return dequant_launch(t, out_dev, stream ? (cudaStream_t)stream : ctx->stream);
}

extern "C" int pox_cuda_tensor_dequant_host(pox_cuda_ctx* ctx, const pox_tensor* t, float* out) {
    if (!ctx || !t || !out) return set_error(POX_ERR_INVALID, "NULL argument");
    std::lock_guard<std::mutex> lk(ctx->mu);
    CK(cudaSetDevice(ctx->device), "cudaSetDevice");
    const size_t n = t->rows * t->cols;
    if (n == 0) return POX_OK;
    float* d = nullptr;
    CK(cudaMalloc(&d, n * sizeof(float)), "cudaMalloc(dequant)");
    int rc = dequant_launch(t, d, ctx->stream);
    if (rc == POX_OK) {
        cudaError_t e = cudaMemcpyAsync(out, d, n * sizeof(float), cudaMemcpyDeviceToHost, ctx->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
        if (e != cudaSuccess) rc = cuda_error(e, "dequant copy");
        else rc = take_kernel_error(ctx);
    }
    cudaStreamSynchronize(ctx->stream);
    cudaFree(d);
    return rc;
}
