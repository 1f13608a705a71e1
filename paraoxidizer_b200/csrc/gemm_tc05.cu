// gemm_tc05.cu -- the small-M path of the weight-only quantized projection: x [B][K] times
// W^T for B = 9 .. 128 rows of x (decode at batch 16-64, chunks of a prefill), on the
// 5th-generation tensor cores (tcgen05.mma kind::f16, accumulator in tensor memory).
//
// Same results contract as quant::gemv_int4 / gemv_int8 (crates/paraoxidizer-quant/src/
// kernels.rs:177-255) and the F16 projection (crates/paraoxidizer-runtime/src/engine.rs:235-250)
// for every row of x, within the GEMV tolerance: the weights enter the MMA as f16 -- INT4 as
// f16(min + q scale) per element (one rounding of the exact affine value), INT8 as the exact
// integer q with the per-tensor scale applied in f32 after the sum, F16 as stored -- and x as f16
// after an exact power-of-two scaling per row that puts max|x| in [2^13, 2^14). Outlier values
// replace their weights in the f16 tile exactly as SparseOutlierTable::apply_to does
// (outlier.rs:88-95; the CSR keeps the last of duplicate entries).
//
// Kernel (one CTA = 128 weight rows x one k-split, 9 warps):
//  * warps 0-7 (producers): warp d owns row tile d (16 rows) of the CTA's 128 rows. Per 128-k
//    block it bulk-copies that tile's packed bytes (INT4: nibbles + scale words, 1088 B; INT8 2 KiB;
//    F16 4 KiB, already contiguous in the re-tiled layout) into a private 4-stage ring, expands
//    them to f16 in the 128-byte-swizzled K-major layout the MMA reads, writes the row tile's
//    outlier values over their slots and arrives on the stage's "full" barrier.
//  * warp 8 (MMA): allocates the accumulator (128 lanes x N columns of TMEM), bulk-copies the
//    stage's x block (pre-swizzled in global memory by the x preparation), and issues 8 MMAs of
//    128 x N x 16 per 128-k block; tcgen05.commit frees the stage.
//  * epilogue (warps 0-3 = TMEM lanes 0-127 = the CTA's rows): y[b][row] = scale_b * D[row][b]
//    (+ resid). With a k-split, each CTA stores its partial and the last CTA of the row block
//    (ticket counter) adds the partials in split order, so results are deterministic.
//  * every wait is bounded (kWaitCycles); a timeout raises the context error flag, drains what is
//    in flight and frees the tensor memory before the CTA exits.
#include <algorithm>

#include "common.cuh"
#include "gemv.cuh"
#include "tc05.cuh"

namespace pox {

constexpr int kTcProd = 8;       // producer warps (row tiles of 16 rows)
constexpr int kTcThreads = (kTcProd + 2) * 32;  // + MMA warp + x loader warp
constexpr int kErrWaitTc = 16;   // bit of the kernel error flag

__host__ __device__ constexpr int tc_wbytes(int kind) { return kind == kKindI4 ? 1088 : kind == kKindI8 ? 2048 : 4096; }
// 128-k blocks per weight copy: a copy costs its warp a fixed overhead whatever its size, so a
// producer moves about 4 KiB at a time (consecutive k-blocks of its row tile are contiguous).
__host__ __device__ constexpr int tc_group(int kind) { return kind == kKindI4 ? 4 : kind == kKindI8 ? 2 : 1; }
// Pipeline depths:
//  A stages: dequantized 128-k weight blocks waiting for / read by the MMAs (32 KiB each); the
//    producers run this many blocks ahead of the MMA completions;
//  weight ring: copies (of tc_group k-blocks) in flight per producer warp (HBM latency);
//  x stages: x blocks in flight (L2 latency).
__host__ __device__ constexpr int tc_ring(int) { return 2; }
__host__ __device__ constexpr int tc_xstages(int N) { return N == 128 ? 2 : 3; }
__host__ __device__ constexpr int tc_smem_bytes(int kind, int N, int A) {
    return A * 32768 + tc_xstages(N) * N * 256 + kTcProd * tc_ring(kind) * tc_group(kind) * tc_wbytes(kind) + 1024;
}
__host__ __device__ constexpr int tc_astages(int kind, int N) {  // the most that fit (at most 4)
    return tc_smem_bytes(kind, N, 4) + 3072 <= 232448 ? 4 : tc_smem_bytes(kind, N, 3) + 3072 <= 232448 ? 3 : 2;
}

struct TcSmem {  // byte offsets in dynamic shared memory (1024-aligned base)
    int a, b, ring, bars, tmem, total;
};
__host__ __device__ inline TcSmem tc_smem(int kind, int N) {
    TcSmem s;
    s.a = 0;                                         // A stages x 2 atoms x 128 rows x 128 B
    s.b = s.a + tc_astages(kind, N) * 32768;         // x stages x 2 atoms x N rows x 128 B
    s.ring = s.b + tc_xstages(N) * N * 256;          // kTcProd x ring x group x wbytes
    s.bars = s.ring + kTcProd * tc_ring(kind) * tc_group(kind) * tc_wbytes(kind);
    // barriers: full[A], empty[A], xfull[X], xempty[X], done, ring[kTcProd][ring]
    s.tmem = s.bars + 8 * (2 * tc_astages(kind, N) + 2 * tc_xstages(N) + 1 + kTcProd * tc_ring(kind));
    s.total = s.tmem + 16;
    return s;
}

__device__ __forceinline__ void sts128(uint32_t a, uint4 v) {
    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ void sts16(uint32_t a, uint16_t v) {
    asm volatile("st.shared.u16 [%0], %1;" ::"r"(a), "h"(v) : "memory");
}

// 8 INT4 nibbles of a re-tiled word (byte i = q[i] | q[4+i] << 4) -> 8 f16 weights min + q scale in k order.
__device__ __forceinline__ uint4 i4_word_to_f16(uint32_t w, uint32_t s2, uint32_t m2) {
    const uint32_t kMagic = 0x64006400u;  // f16 pair (1024, 1024)
    const uint32_t t01 = prmt(w, 0u, 0x4140u), t23 = prmt(w, 0u, 0x4342u);
    uint4 r;
    r.x = hfma2_u32(hsub2_u32(lop3_and_or(t01, 0x000F000Fu, kMagic), kMagic), s2, m2);
    r.y = hfma2_u32(hsub2_u32(lop3_and_or(t23, 0x000F000Fu, kMagic), kMagic), s2, m2);
    r.z = hfma2_u32(hsub2_u32(lop3_and_or(t01 >> 4, 0x000F000Fu, kMagic), kMagic), s2, m2);
    r.w = hfma2_u32(hsub2_u32(lop3_and_or(t23 >> 4, 0x000F000Fu, kMagic), kMagic), s2, m2);
    return r;
}

template <int KIND, int N>
__global__ void __launch_bounds__(kTcThreads, 1) gemm_tc05_kernel(TcArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const TcSmem P = tc_smem(KIND, N);
    constexpr int kTcRing = tc_ring(KIND);
    constexpr int kTcStages = tc_astages(KIND, N);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int rb = blockIdx.x, split = blockIdx.y;
    const int kb0 = (int)((long long)a.nkb * split / a.S), kb1 = (int)((long long)a.nkb * (split + 1) / a.S);
    const int nk = kb1 - kb0;
    const uint32_t sA = smem_u32(smem + P.a), sB = smem_u32(smem + P.b), sRing = smem_u32(smem + P.ring);
    const uint32_t bars = smem_u32(smem + P.bars);
    constexpr int XS = tc_xstages(N);
    auto full = [&](int s) { return bars + 8 * s; };
    auto empty = [&](int s) { return bars + 8 * (kTcStages + s); };
    auto xfull = [&](int s) { return bars + 8 * (2 * kTcStages + s); };
    auto xempty = [&](int s) { return bars + 8 * (2 * kTcStages + XS + s); };
    const uint32_t done = bars + 8 * (2 * kTcStages + 2 * XS);
    auto ringbar = [&](int d, int r) { return bars + 8 * (2 * kTcStages + 2 * XS + 1 + d * kTcRing + r); };
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + P.tmem);
    __shared__ int s_abort;

    if (tid == 0) {
        for (int s = 0; s < kTcStages; s++) {
            mbar_init(full(s), kTcProd);
            mbar_init(empty(s), 1);
        }
        for (int s = 0; s < XS; s++) {
            mbar_init(xfull(s), 1);
            mbar_init(xempty(s), 1);
        }
        mbar_init(done, 1);
        for (int d = 0; d < kTcProd; d++)
            for (int r = 0; r < kTcRing; r++) mbar_init(ringbar(d, r), 1);
        s_abort = 0;
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    __syncthreads();
    pdl_launch_dependents();

    const int TB = tc_wbytes(KIND);
    constexpr int GK = tc_group(KIND);
    const int SBy = GK * TB;  // bytes per ring stage
    if (warp < kTcProd) {
        // ------------------------------ producer warp d ------------------------------
        const int d = warp, T = rb * 8 + d;  // row tile
        const bool live = T < a.nT;
        const uint8_t* wsrc = a.w + ((size_t)T * a.nkb + kb0) * TB;
        const uint32_t ring = sRing + d * kTcRing * SBy;
        auto issue = [&](int gi) {  // lane 0: k-blocks kb0 + GK gi .. (one copy) into ring stage gi % kTcRing
            const uint32_t bar = ringbar(d, gi % kTcRing);
            const uint32_t bytes = (uint32_t)min(GK, nk - gi * GK) * TB;
            mbar_expect_tx(bar, bytes);
            bulk_g2s(ring + (gi % kTcRing) * SBy, wsrc + (size_t)gi * GK * TB, bytes, bar);
        };
        if (live && lane == 0)
            for (int gi = 0; gi < kTcRing && gi * GK < nk; gi++) issue(gi);
        // outliers of (row tile, k-block) kb0 + i: entries [tp[i], tp[i + 1]) of the tile-ordered
        // table, each (row % 16) | (col % 128) << 4 | f16 value << 16; lane j holds entry j of the
        // next k-block, loaded one k-block ahead
        const bool has_out = KIND == kKindI4 && a.tile_ptr != nullptr && live;
        const uint32_t* tp = has_out ? a.tile_ptr + (size_t)T * a.nkb + kb0 : nullptr;
        uint32_t e0 = 0, e1 = 0, ent = 0;
        if (has_out) {
            e0 = __ldg(tp);
            e1 = __ldg(tp + 1);
            ent = e0 + lane < a.nnz ? __ldg(a.tile_ent + e0 + lane) : 0u;
        }
        const int g = lane >> 2, t = lane & 3;
        int i = 0;
        bool ok = true;
        for (; i < nk; i++) {
            const int s = i % kTcStages;
            if (!__all_sync(0xffffffffu, mbar_wait(empty(s), ((i / kTcStages) & 1) ^ 1))) { ok = false; break; }
            const uint32_t stA = sA + s * 32768;
            if (live) {
                const int gi = i / GK, r = gi % kTcRing;
                if (i % GK == 0 &&
                    !__all_sync(0xffffffffu, mbar_wait(ringbar(d, r), (gi / kTcRing) & 1))) { ok = false; break; }
                const uint32_t src = ring + r * SBy + (i % GK) * TB;
#pragma unroll
                for (int hs = 0; hs < 2; hs++) {  // rows g (hs 0) and g + 8 (hs 1) of the tile
                    const uint32_t row = 16 * d + g + 8 * hs;
                    if (KIND == kKindI4) {
                        const uint4 v = lds128(src + hs * 512 + lane * 16);
                        const uint32_t sw = lds32(src + 1024 + 4 * (2 * g + hs));
                        const uint32_t s2 = (sw & 0xFFFFu) * 0x10001u, m2 = (sw >> 16) * 0x10001u;
                        const uint32_t atom = stA + (t >> 1) * 16384;
                        const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
                        // lanes t and t + 2 of a quarter warp share a bank group for equal w: they
                        // take the words in the order w ^ 2, so each quarter-warp store is one wavefront
                        const int rot = t & 2;
#pragma unroll
                        for (int w = 0; w < 4; w++) {
                            const int ww = w ^ rot;
                            const uint32_t wd = rot ? wv[w ^ 2] : wv[w];
                            sts128(atom + sw128_off(row, 4 * (t & 1) + ww), i4_word_to_f16(wd, s2, m2));
                        }
                    } else if (KIND == kKindI8) {
#pragma unroll
                        for (int u = 0; u < 2; u++) {  // 64-k tiles u = atoms u
                            const uint4 v = lds128(src + u * 1024 + hs * 512 + lane * 16);
                            uint4 c0, c1;
                            i8x4_to_f16x4(v.x, c0.x, c0.y);
                            i8x4_to_f16x4(v.y, c0.z, c0.w);
                            i8x4_to_f16x4(v.z, c1.x, c1.y);
                            i8x4_to_f16x4(v.w, c1.z, c1.w);
                            sts128(stA + u * 16384 + sw128_off(row, 2 * t), c0);
                            sts128(stA + u * 16384 + sw128_off(row, 2 * t + 1), c1);
                        }
                    } else {
#pragma unroll
                        for (int u0 = 0; u0 < 4; u0++) {  // 32-k tiles u: atom u / 2, chunks 4 (u % 2) + t
                            const int u = u0 ^ (g & 1);   // rows g, g ^ 1 of a quarter warp: other half of the atom
                            const uint4 v = lds128(src + u * 1024 + hs * 512 + lane * 16);
                            sts128(stA + (u >> 1) * 16384 + sw128_off(row, 4 * (u & 1) + t), v);
                        }
                    }
                }
                if (has_out) {
                    __syncwarp();  // the dequantized tile is written before values replace slots in it
                    uint32_t n1 = 0, nent = 0;
                    if (i + 1 < nk) {  // next k-block's range and first entries, in flight meanwhile
                        n1 = __ldg(tp + i + 2);
                        nent = e1 + lane < a.nnz ? __ldg(a.tile_ent + e1 + lane) : 0u;
                    }
                    for (uint32_t base = e0; base < e1; base += 32) {
                        const uint32_t v = base == e0 ? ent : (base + lane < e1 ? __ldg(a.tile_ent + base + lane) : 0u);
                        if (base + lane < e1) {
                            const uint32_t r = v & 15u, kk = (v >> 4) & 127u;
                            sts16(stA + (kk >> 6) * 16384 + sw128_off(16 * d + r, (kk & 63) >> 3) + 2 * (kk & 7),
                                  (uint16_t)(v >> 16));
                        }
                    }
                    e0 = e1;
                    e1 = n1;
                    ent = nent;
                }
                __syncwarp();
                if (lane == 0 && (i % GK == GK - 1 || i + 1 == nk) && (gi + kTcRing) * GK < nk) {
                    fence_proxy_async_smem();  // reads of the ring stage done before its refill
                    issue(gi + kTcRing);
                }
            } else {
                // rows beyond the tensor: zero weights
#pragma unroll
                for (int hs = 0; hs < 2; hs++)
#pragma unroll
                    for (int c = 0; c < 4; c++)
                        sts128(stA + ((t * 4 + c) >> 3) * 16384 + sw128_off(16 * d + g + 8 * hs, (t * 4 + c) & 7),
                               make_uint4(0u, 0u, 0u, 0u));
            }
            fence_proxy_async_smem();  // generic-proxy writes visible to the tensor core
            __syncwarp();
            if (lane == 0) mbar_arrive(full(s));
        }
        if (!ok) {
            if (lane == 0) {
                atomicOr(a.err, kErrWaitTc);
                atomicExch(&s_abort, 1);
                if (live)  // copies issued but not consumed: wait for them (bounded) before exiting
                    for (int gj = i / GK; gj * GK < nk && gj < i / GK + kTcRing; gj++)
                        mbar_wait(ringbar(d, gj % kTcRing), (gj / kTcRing) & 1);
            }
        }
    } else if (warp == kTcProd + 1) {
        // ------------------------------ x loader ------------------------------
        pdl_wait();  // x is written by the preceding kernel
        if (lane == 0) {
            const uint32_t xb = N * 256;
            int i = 0;
            bool ok = true;
            for (; i < nk; i++) {
                const int s = i % XS;
                if (!mbar_wait(xempty(s), ((i / XS) & 1) ^ 1)) {  // MMAs of k-block i - XS done
                    ok = false;
                    break;
                }
                mbar_expect_tx(xfull(s), xb);
                bulk_g2s(sB + s * xb, a.xs + (size_t)(kb0 + i) * xb, xb, xfull(s));
            }
            if (!ok) {
                atomicOr(a.err, kErrWaitTc);
                atomicExch(&s_abort, 1);
                for (int j = max(0, i - XS); j < i; j++) mbar_wait(xfull(j % XS), (j / XS) & 1);  // in flight
            }
        }
        __syncwarp();
    } else {
        // ------------------------------ MMA warp ------------------------------
        pdl_wait();  // x is written by the preceding kernel; TMEM is taken only after it finished
        tmem_alloc(smem_u32(tmem_slot), N < 32 ? 32 : N);
        tmem_relinquish();
        tc_fence_before();
        __syncwarp();
        tc_fence_after();
        const uint32_t tmem = *tmem_slot;
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_f16(128, N);
            const uint32_t xb = N * 256;  // x bytes per 128-k block
            int i = 0;
            bool ok = true;
            for (; i < nk; i++) {  // never waits on an MMA completion: the loaders do
                const int s = i % kTcStages, xs_ = i % XS;
                if (!mbar_wait(full(s), (i / kTcStages) & 1) || !mbar_wait(xfull(xs_), (i / XS) & 1)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int at = 0; at < 2; at++) {
                    const uint64_t ad = umma_desc_sw128(sA + s * 32768 + at * 16384);
                    const uint64_t bd = umma_desc_sw128(sB + xs_ * xb + at * N * 128);
#pragma unroll
                    for (int k16 = 0; k16 < 4; k16++)
                        umma_f16(tmem, ad + 2 * k16, bd + 2 * k16, idesc, (i | at | k16) != 0);
                }
                umma_commit(empty(s));
                umma_commit(xempty(xs_));
            }
            umma_commit(done);  // arrives when every MMA issued above has completed
            if (!ok) {
                atomicOr(a.err, kErrWaitTc);
                atomicExch(&s_abort, 1);
            }
        }
        __syncwarp();
    }

    // ------------------------------ epilogue ------------------------------
    tc_fence_before();
    __syncthreads();  // the TMEM address and every abort decision of the main loop are visible
    tc_fence_after();
    if (warp < 4) {
        pdl_wait();
        if (!mbar_wait(done, 0)) {
            if (lane == 0) atomicOr(a.err, kErrWaitTc);
            atomicExch(&s_abort, 1);
        }
    }
    __syncthreads();  // one decision for the whole CTA
    const bool go = !*(volatile int*)&s_abort;
    if (go && warp < 4) {
        tc_fence_after();
        const uint32_t tmem = *tmem_slot;
        const int row = rb * 128 + warp * 32 + lane;
        float* dst = a.S > 1 ? a.ws + (size_t)split * a.Bp * a.Nout : a.y;
#pragma unroll
        for (int c0 = 0; c0 < N; c0 += 32) {
            float v[32];
            tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + c0, v);
            if (row < a.Nout) {
#pragma unroll
                for (int j = 0; j < 32; j++) {
                    const int b = c0 + j;
                    if (b < a.B) {
                        if (a.S > 1) {
                            dst[(size_t)b * a.Nout + row] = v[j];
                        } else {
                            float r = v[j] * a.xscale[b] * (a.row_scale ? a.row_scale[row] : a.wscale);
                            if (a.resid) r += a.resid[(size_t)b * a.Nout + row];
                            dst[(size_t)b * a.Nout + row] = r;
                        }
                    }
                }
            }
        }
    }
    if (go && a.S > 1) {
        // the last CTA of the row block adds the S partials in split order (all 320 threads, two
        // items of 4 rows per thread in flight, S loads each)
        __shared__ int s_last;
        __threadfence();
        __syncthreads();
        if (tid == 0) {
            const int prev = atomicAdd(a.tickets + rb, 1);
            s_last = prev == a.S - 1;
            if (s_last) a.tickets[rb] = 0;  // ready for the next launch
        }
        __syncthreads();
        if (s_last) {
            __threadfence();
            const int r0 = rb * 128, nrow = min(128, a.Nout - r0);
            const bool vec = (a.Nout & 3) == 0 && ((uintptr_t)a.y & 15) == 0 && ((uintptr_t)a.resid & 15) == 0;
            const int per_b = vec ? (nrow + 3) / 4 : nrow;  // items per batch row
            const int items = a.B * per_b;
            for (int it = tid; it < items; it += kTcThreads) {
                const int b = it / per_b, q = it % per_b;
                const float sc = a.xscale[b] * a.wscale;  // per-tensor scale; per-row scales below
                if (vec) {
                    const size_t o = (size_t)b * a.Nout + r0 + 4 * q;
                    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
                    float4 part[16];
#pragma unroll
                    for (int sp = 0; sp < 16; sp++)
                        if (sp < a.S) part[sp] = __ldcg(reinterpret_cast<const float4*>(a.ws + (size_t)sp * a.Bp * a.Nout + o));
#pragma unroll
                    for (int sp = 0; sp < 16; sp++)
                        if (sp < a.S) {
                            acc.x += part[sp].x;
                            acc.y += part[sp].y;
                            acc.z += part[sp].z;
                            acc.w += part[sp].w;
                        }
                    float4 r;
                    if (a.row_scale) {
                        const int rw = r0 + 4 * q;
                        const float xs = a.xscale[b];
                        r = make_float4(acc.x * (xs * a.row_scale[rw]), acc.y * (xs * a.row_scale[rw + 1]),
                                        acc.z * (xs * a.row_scale[rw + 2]), acc.w * (xs * a.row_scale[rw + 3]));
                    } else {
                        r = make_float4(acc.x * sc, acc.y * sc, acc.z * sc, acc.w * sc);
                    }
                    if (a.resid) {
                        const float4 rr = *reinterpret_cast<const float4*>(a.resid + o);
                        r.x += rr.x;
                        r.y += rr.y;
                        r.z += rr.z;
                        r.w += rr.w;
                    }
                    *reinterpret_cast<float4*>(a.y + o) = r;
                } else {
                    const size_t o = (size_t)b * a.Nout + r0 + q;
                    float acc = 0.f;
                    for (int sp = 0; sp < a.S; sp++) acc += __ldcg(a.ws + (size_t)sp * a.Bp * a.Nout + o);
                    float r = acc * (a.row_scale ? a.xscale[b] * a.row_scale[r0 + q] : sc);
                    if (a.resid) r += a.resid[o];
                    a.y[o] = r;
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();  // every TMEM read has completed (tcgen05.wait::ld) before the deallocation
    if (warp == kTcProd) {
        tc_fence_after();
        tmem_dealloc(*tmem_slot, N < 32 ? 32 : N);
    }
}

// ------------------------------------------------------------------------------------------
// x preparation: one CTA of 1024 threads per row n < Bp of the padded batch. Row n < B:
// v = op(x_n) is computed once into shared memory together with the row's sum of squares and
// max|v| (RMSNorm: the scale 1/rms is common to the row, so max|x w| gives max|v|); e such that
// max|v| 2^-e lies in [2^13, 2^14) (e = 0 for an all-zero row); writes f16(v 2^-e) into the
// k-block-major, 128-byte-swizzled layout [kb][atom][Bp rows][128 B] and xscale[n] = 2^e. Rows
// B .. Bp-1 are zero.
// ------------------------------------------------------------------------------------------
constexpr int kXpThreads = 1024;
__global__ void __launch_bounds__(kXpThreads) xprep_tc05_kernel(const float* __restrict__ x, int B, int Bp, int K,
                                                                PrepOp op, uint8_t* __restrict__ xs,
                                                                float* __restrict__ xscale) {
    extern __shared__ float vs[];  // [K]
    pdl_launch_dependents();
    pdl_wait();
    const int n = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    __shared__ float red_s[32], red_m[32];
    __shared__ float s_mul;
    if (n < B) {
        const float* xr = x + (size_t)n * op.ld_x;
        const float* ur = op.up ? op.up + (size_t)n * op.ld_up : nullptr;
        float ss = 0.f, m = 0.f;
        for (int k = 4 * tid; k < K; k += 4 * kXpThreads) {  // K % 128 == 0
            float4 v = *reinterpret_cast<const float4*>(xr + k);
            float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int j = 0; j < 4; j++) {
                if (op.mode == kPrepNorm) {
                    ss = fmaf(e[j], e[j], ss);
                    if (op.norm_w) e[j] *= half_bits_to_float(op.norm_w[k + j]);  // x w; 1/rms applied below
                } else if (op.mode == kPrepSwiGLU) {
                    e[j] = e[j] / (1.0f + expf(-e[j])) * ur[k + j];
                }
                m = fmaxf(m, fabsf(e[j]));
            }
            *reinterpret_cast<float4*>(vs + k) = make_float4(e[0], e[1], e[2], e[3]);
        }
        ss = warp_sum(ss);
        m = warp_max(m);
        if (lane == 0) {
            red_s[warp] = ss;
            red_m[warp] = m;
        }
        __syncthreads();
        if (tid == 0) {
            float sst = 0.f, mm = 0.f;
            for (int w = 0; w < kXpThreads / 32; w++) {
                sst += red_s[w];
                mm = fmaxf(mm, red_m[w]);
            }
            float inv = 1.f;
            if (op.mode == kPrepNorm) {
                inv = 1.0f / sqrtf(sst / (float)K + op.eps);
                mm *= inv;
            }
            int e = 0;
            if (mm > 0.f && isfinite(mm)) {
                frexpf(mm, &e);  // mm in [2^(e-1), 2^e)
                e -= 14;
            }
            xscale[n] = ldexpf(1.f, e);
            s_mul = inv * ldexpf(1.f, -e);  // 1/rms (or 1) times the power-of-two scale
        }
        __syncthreads();
    }
    const float mul = n < B ? s_mul : 0.f;
    for (int c = tid; c < K / 8; c += kXpThreads) {  // one 16-byte chunk of 8 consecutive k
        const int k = c * 8, kb = k >> 7, kk = k & 127;
        uint32_t h[4] = {0u, 0u, 0u, 0u};
        if (n < B) {
            const float4 a0 = *reinterpret_cast<const float4*>(vs + k), a1 = *reinterpret_cast<const float4*>(vs + k + 4);
            const __half2 p0 = __floats2half2_rn(a0.x * mul, a0.y * mul), p1 = __floats2half2_rn(a0.z * mul, a0.w * mul);
            const __half2 p2 = __floats2half2_rn(a1.x * mul, a1.y * mul), p3 = __floats2half2_rn(a1.z * mul, a1.w * mul);
            h[0] = *reinterpret_cast<const uint32_t*>(&p0);
            h[1] = *reinterpret_cast<const uint32_t*>(&p1);
            h[2] = *reinterpret_cast<const uint32_t*>(&p2);
            h[3] = *reinterpret_cast<const uint32_t*>(&p3);
        }
        const size_t off = ((size_t)kb * 2 + (kk >> 6)) * (size_t)Bp * 128 + sw128_off(n, (kk & 63) >> 3);
        *reinterpret_cast<uint4*>(xs + off) = make_uint4(h[0], h[1], h[2], h[3]);
    }
}

// ------------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------------
int tc05_pad(int B) { return B <= 16 ? 16 : B <= 32 ? 32 : B <= 64 ? 64 : 128; }

size_t tc05_x_bytes(int K, int Bp) { return (size_t)(K / 128) * Bp * 256; }

// k-split count: waves of CTAs x k-blocks per CTA, plus a fixed cost per CTA and per split reduction.
int tc05_splits(int nrb, int nkb, int sms) {
    int best = 1;
    double best_t = 1e30;
    for (int S = 1; S <= 16 && S <= nkb; S++) {  // at most 16: the reduction holds 16 partials
        const int waves = (nrb * S + sms - 1) / sms;
        const int per = (nkb + S - 1) / S;
        const double t = waves * (per + 3.0) + (S > 1 ? 2.0 : 0.0);
        if (t < best_t - 1e-9) {
            best_t = t;
            best = S;
        }
    }
    return best;
}

template <int KIND, int N>
static cudaError_t launch_tc05_t(const TcArgs& a, cudaStream_t st) {
    const TcSmem P = tc_smem(KIND, N);
    const int bytes = P.total + 1024;
    const cudaError_t e =  // per device and function: set on every launch (host-side, cheap)
        cudaFuncSetAttribute(gemm_tc05_kernel<KIND, N>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((a.Nout + 127) / 128), (unsigned)a.S, 1);
    cfg.blockDim = dim3(kTcThreads, 1, 1);
    cfg.dynamicSmemBytes = bytes;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, gemm_tc05_kernel<KIND, N>, a);
}

template <int KIND>
static cudaError_t launch_tc05_kind(const TcArgs& a, cudaStream_t st) {
    switch (a.Bp) {
        case 16: return launch_tc05_t<KIND, 16>(a, st);
        case 32: return launch_tc05_t<KIND, 32>(a, st);
        case 64: return launch_tc05_t<KIND, 64>(a, st);
        case 128: return launch_tc05_t<KIND, 128>(a, st);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_tc05(int kind, const TcArgs& a, cudaStream_t st) {
    if (kind == kKindI4) return launch_tc05_kind<kKindI4>(a, st);
    if (kind == kKindI8) return launch_tc05_kind<kKindI8>(a, st);
    return launch_tc05_kind<kKindF16>(a, st);
}

cudaError_t launch_xprep_tc05(const float* x, int B, int Bp, int K, const PrepOp& op_in, uint8_t* xs, float* xscale,
                              cudaStream_t st) {
    PrepOp op = op_in;
    if (op.ld_x == 0) op.ld_x = K;
    const size_t smem = (size_t)K * sizeof(float);
    if (smem > 48 * 1024) {
        const cudaError_t e = cudaFuncSetAttribute(xprep_tc05_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   (int)smem);
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)Bp, 1, 1);
    cfg.blockDim = dim3(kXpThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, xprep_tc05_kernel, x, B, Bp, K, op, xs, xscale);
}

}  // namespace pox
