// gemm_tcq.cu -- the small-M projection on the integer tensor cores: x [B][K] times W^T for
// up to 64 rows of x, tcgen05.mma kind::i8, for INT8 weights and INT4 weights without outliers
// (padded batch 16-64; tq_supported).
//
// Same results contract as quant::gemv_int4 / gemv_int8 (crates/paraoxidizer-quant/src/
// kernels.rs:177-255) within the GEMV tolerance, computed the way the batch <= 8 GEMV does:
// the weights enter the MMA as exact unsigned (INT4 q) or signed (INT8 q) 8-bit integers, x as
// the 15-bit fixed point of each 128-k block split into two exact int8 limbs (X = 128 hi + lo),
// so every 128-k block's product sum_k q_k X_k is exact in s32. The affine map of the INT4 group
// is applied once per row and 128-k block, sum_k (min + q s) x_k = s sx sum_k q X + min sum_k x
// (sx = the block's max|x| / 16383); INT8 takes its per-tensor scale at the end.
//
// Kernel (one CTA = 128 weight rows x one k-split):
//  * warps 0-7 (producers): warp d owns row tile d (16 rows). It bulk-copies its tile's bytes,
//    four 128-k blocks per copy (INT4 nibbles + scale words, 1088 B per block; INT8 2 KiB),
//    unpacks them into the 128-byte-swizzled K-major u8 / s8 layout the MMA reads and arrives on
//    the A stage's "full" barrier.
//  * warp 8 (MMA): per 128-k block, 4 MMAs of 128 x 2Bp x 32 into a fresh accumulator slot of
//    tensor memory (slots rotate), then commits the A stage free and the slot full.
//  * warp 9 (x loader): bulk-copies each block's x limbs (pre-swizzled by the x preparation) and
//    its (sx, sum x) per batch row.
//  * warps 10.. (epilogue, 4 or 8): thread = weight row (its TMEM lane), a column range of batch
//    rows; per block it reads the slot, combines the limbs and applies the block's scales to
//    running f32 sums, then frees the slot and the x stage. INT4 scale words are read from the
//    tile in global memory a few blocks ahead.
//  * k-splits: each CTA stores its partial; the last CTA of the row block (ticket counter) adds
//    the partials in split order, so results do not depend on timing.
//  * every wait is bounded (kWaitCycles); a timeout raises the context error flag, drains what is
//    in flight and frees the tensor memory before the CTA exits.
#include <algorithm>

#include "common.cuh"
#include "gemv.cuh"
#include "tc05.cuh"

namespace pox {

constexpr int kTqProd = 8;     // producer warps (row tiles of 16 rows)
constexpr int kTqErr = 32;     // bit of the kernel error flag
constexpr int kTqPf = 4;       // INT4 scale words read this many blocks ahead
__host__ __device__ constexpr int tq_epi(int NP) { return NP >= 64 ? 8 : 4; }              // epilogue warps
__host__ __device__ constexpr int tq_threads(int NP) { return (kTqProd + 2 + tq_epi(NP)) * 32; }
__host__ __device__ constexpr int tq_slots(int NP) { return NP == 128 ? 4 : 8; }            // TMEM slots
__host__ __device__ constexpr int tq_tmem_cols(int NP) { return tq_slots(NP) * NP < 32 ? 32 : tq_slots(NP) * NP; }
__host__ __device__ constexpr int tq_wbytes(int kind) { return kind == kKindI4 ? 1088 : 2048; }  // per 128-k block
__host__ __device__ constexpr int tq_group(int kind) { return kind == kKindI4 ? 4 : 2; }  // blocks per weight copy
constexpr int kTqXs = 4;                                                                    // x stages
__host__ __device__ constexpr int tq_xsb(int NP) { return NP * 128 + 1024; }               // limbs + block meta
__host__ __device__ constexpr int tq_fixed(int kind, int NP) {
    return kTqXs * tq_xsb(NP) + kTqProd * 2 * tq_group(kind) * tq_wbytes(kind) + 1024;
}
__host__ __device__ constexpr int tq_astages(int kind, int NP) {  // 16 KiB A stages: as many as fit, at most 8
    return (226 * 1024 - tq_fixed(kind, NP)) / 16384 > 8 ? 8 : (226 * 1024 - tq_fixed(kind, NP)) / 16384;
}
__host__ __device__ constexpr int tq_smem(int kind, int NP) { return tq_astages(kind, NP) * 16384 + tq_fixed(kind, NP); }

// Where this path beats the f16 tiles of gemm_tc05.cu (us per call with its x preparation, B200,
// f16 tiles vs this kernel): INT8 up to a padded batch of 64; INT4 without outliers up to 64 too
// (4096 x 14336: 28.9 vs 26.6 at batch 32, 34.5 vs 32.0 at 64; 28672 x 4096: 51.9 vs 41.8 and
// 58.3 vs 51.6; 6144 x 4096 and 4096 x 4096 within 6 % either way). At a padded batch of 128 the
// per-block readout of every batch column outweighs the cheaper unpacking.
bool tq_supported(int kind, bool outliers, int Bp) {
    return (kind == kKindI4 && !outliers && Bp <= 64) || (kind == kKindI8 && Bp <= 64);
}
size_t tq_x_bytes(int K, int Bp) {
    const size_t limbs = (size_t)(K / 128) * 2 * Bp * 128;
    return ((limbs + 255) & ~(size_t)255) + (size_t)(K / 128) * Bp * sizeof(float2);
}

// D[tmem] (+)= A[smem] * B[smem]^T, one CTA, A u8 and B s8, s32 accumulator.
__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// kind::i8 instruction descriptor: A u8 or s8, B s8 (both K-major), s32 accumulator, M x N.
__host__ __device__ constexpr uint32_t umma_idesc_i8(int M, int N, int a_signed) {
    return (2u << 4)                          // D format: s32
           | ((uint32_t)a_signed << 7)        // A format: u8 (0) / s8 (1)
           | (1u << 10)                       // B format: s8
           | ((uint32_t)(N >> 3) << 17)       // N / 8
           | ((uint32_t)(M >> 4) << 24);      // M / 16
}
__device__ __forceinline__ void sts128q(uint32_t a, uint4 v) {
    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}

template <int KIND, int NP>
__global__ void __launch_bounds__(tq_threads(NP), 1) gemm_tq_kernel(TqArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    constexpr int AS = tq_astages(KIND, NP), XSB = tq_xsb(NP), NSL = tq_slots(NP), E = tq_epi(NP);
    constexpr int TB = tq_wbytes(KIND), GK = tq_group(KIND), RB = GK * TB;  // ring stage bytes
    constexpr int BP = NP / 2;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int rb = blockIdx.x, split = blockIdx.y;
    const int kb0 = (int)((long long)a.nkb * split / a.S), kb1 = (int)((long long)a.nkb * (split + 1) / a.S);
    const int nk = kb1 - kb0;
    const uint32_t sA = smem_u32(smem), sX = sA + AS * 16384, sRing = sX + kTqXs * XSB;
    const uint32_t bars = sRing + kTqProd * 2 * RB;
    auto full = [&](int s) { return bars + 8 * s; };
    auto empty = [&](int s) { return bars + 8 * (AS + s); };
    auto xfull = [&](int s) { return bars + 8 * (2 * AS + s); };
    auto xempty = [&](int s) { return bars + 8 * (2 * AS + kTqXs + s); };
    auto accfull = [&](int s) { return bars + 8 * (2 * AS + 2 * kTqXs + s); };
    auto accempty = [&](int s) { return bars + 8 * (2 * AS + 2 * kTqXs + NSL + s); };
    auto ringbar = [&](int d, int r) { return bars + 8 * (2 * AS + 2 * kTqXs + 2 * NSL + 2 * d + r); };
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + (bars - sA) + 8 * (2 * AS + 2 * kTqXs + 2 * NSL + 2 * kTqProd));
    __shared__ int s_abort;

    if (tid == 0) {
        for (int s = 0; s < AS; s++) {
            mbar_init(full(s), kTqProd);
            mbar_init(empty(s), 1);
        }
        for (int s = 0; s < kTqXs; s++) {
            mbar_init(xfull(s), 1);
            mbar_init(xempty(s), E);
        }
        for (int s = 0; s < NSL; s++) {
            mbar_init(accfull(s), 1);
            mbar_init(accempty(s), E);
        }
        for (int d = 0; d < kTqProd; d++)
            for (int r = 0; r < 2; r++) mbar_init(ringbar(d, r), 1);
        s_abort = 0;
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    __syncthreads();
    pdl_launch_dependents();

    if (warp < kTqProd) {
        // ------------------------------ producer warp d ------------------------------
        const int d = warp, T = rb * 8 + d;  // row tile
        const bool live = T < a.nT;
        const uint8_t* wsrc = a.w + ((size_t)T * a.nkb + kb0) * TB;
        const uint32_t ring = sRing + d * 2 * RB;
        auto issue = [&](int gi) {  // lane 0: blocks kb0 + GK gi .. (one copy) into ring stage gi % 2
            const uint32_t bar = ringbar(d, gi & 1);
            const uint32_t bytes = (uint32_t)min(GK, nk - gi * GK) * TB;
            mbar_expect_tx(bar, bytes);
            bulk_g2s(ring + (gi & 1) * RB, wsrc + (size_t)gi * GK * TB, bytes, bar);
        };
        if (live && lane == 0)
            for (int gi = 0; gi < 2 && gi * GK < nk; gi++) issue(gi);
        const int g = lane >> 2, t = lane & 3;
        int i = 0;
        bool ok = true;
        for (; i < nk; i++) {
            const int s = i % AS;
            if (!__all_sync(0xffffffffu, mbar_wait(empty(s), ((i / AS) & 1) ^ 1))) { ok = false; break; }
            const uint32_t stA = sA + s * 16384;
            if (live) {
                const int gi = i / GK;
                if (i % GK == 0 &&
                    !__all_sync(0xffffffffu, mbar_wait(ringbar(d, gi & 1), (gi >> 1) & 1))) { ok = false; break; }
                const uint32_t src = ring + (gi & 1) * RB + (i % GK) * TB;
#pragma unroll
                for (int hs = 0; hs < 2; hs++) {  // rows g (hs 0) and g + 8 (hs 1) of the tile
                    const uint32_t row = 16 * d + g + 8 * hs;
                    if (KIND == kKindI4) {
                        // word w of the lane's 16 bytes: 8 consecutive k (32 t + 8 w ..), low nibbles
                        // the first four, high nibbles the next four; each pair of words is one
                        // 16-byte chunk of u8 in k order
                        const uint4 v = lds128(src + hs * 512 + lane * 16);
                        const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
                        uint32_t u[8];
#pragma unroll
                        for (int w = 0; w < 4; w++) {
                            u[2 * w] = wv[w] & 0x0F0F0F0Fu;
                            u[2 * w + 1] = (wv[w] >> 4) & 0x0F0F0F0Fu;
                        }
                        sts128q(stA + sw128_off(row, 2 * t), make_uint4(u[0], u[1], u[2], u[3]));
                        sts128q(stA + sw128_off(row, 2 * t + 1), make_uint4(u[4], u[5], u[6], u[7]));
                    } else {
#pragma unroll
                        for (int uu = 0; uu < 2; uu++) {  // 64-k tiles u; rows g, g ^ 1 of a quarter warp take them in turn
                            const int u = uu ^ (g & 1);
                            const uint4 v = lds128(src + u * 1024 + hs * 512 + lane * 16);
                            sts128q(stA + sw128_off(row, 4 * u + t), v);
                        }
                    }
                }
                __syncwarp();
                if (lane == 0 && (i % GK == GK - 1 || i + 1 == nk) && (gi + 2) * GK < nk) {
                    fence_proxy_async_smem();  // reads of the ring stage done before its refill
                    issue(gi + 2);
                }
            } else {
                // rows beyond the tensor: zero weights (16 rows x 8 chunks = 4 chunks per lane)
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    const int q = lane * 4 + c;
                    sts128q(stA + sw128_off(16 * d + (q >> 3), q & 7), make_uint4(0u, 0u, 0u, 0u));
                }
            }
            fence_proxy_async_smem();  // generic-proxy writes visible to the tensor core
            __syncwarp();
            if (lane == 0) mbar_arrive(full(s));
        }
        if (!ok && lane == 0) {
            atomicOr(a.err, kTqErr);
            atomicExch(&s_abort, 1);
            if (live)  // copies issued but not consumed: wait for them (bounded) before exiting
                for (int gj = i / GK; gj * GK < nk && gj < i / GK + 2; gj++)
                    mbar_wait(ringbar(d, gj & 1), (gj >> 1) & 1);
        }
    } else if (warp == kTqProd + 1) {
        // ------------------------------ x loader ------------------------------
        pdl_wait();  // x is written by the preceding kernel
        if (lane == 0) {
            const uint32_t lb = NP * 128, mb = BP * (uint32_t)sizeof(float2);
            int i = 0;
            bool ok = true;
            for (; i < nk; i++) {
                const int s = i % kTqXs;
                if (!mbar_wait(xempty(s), ((i / kTqXs) & 1) ^ 1)) {  // epilogue done with block i - kTqXs
                    ok = false;
                    break;
                }
                mbar_expect_tx(xfull(s), lb + mb);
                bulk_g2s(sX + s * XSB, a.xl + (size_t)(kb0 + i) * lb, lb, xfull(s));
                bulk_g2s(sX + s * XSB + lb, a.xm + (size_t)(kb0 + i) * BP, mb, xfull(s));
            }
            if (!ok) {
                atomicOr(a.err, kTqErr);
                atomicExch(&s_abort, 1);
                for (int j = max(0, i - kTqXs); j < i; j++) mbar_wait(xfull(j % kTqXs), (j / kTqXs) & 1);  // in flight
            }
        }
        __syncwarp();
    } else if (warp == kTqProd) {
        // ------------------------------ MMA warp ------------------------------
        pdl_wait();  // TMEM is taken only after the preceding kernel finished
        tmem_alloc(smem_u32(tmem_slot), tq_tmem_cols(NP));
        tmem_relinquish();
        tc_fence_before();
        // the allocation is published to the epilogue warps (named barrier 1: MMA warp + epilogue)
        asm volatile("bar.arrive 1, %0;" ::"r"(32 * (1 + E)) : "memory");
        __syncwarp();
        tc_fence_after();
        const uint32_t tmem = *tmem_slot;
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_i8(128, NP, KIND == kKindI8 ? 1 : 0);
            int i = 0;
            bool ok = true;
            for (; i < nk; i++) {
                const int s = i % AS, xs_ = i % kTqXs, sl = i % NSL;
                if (!mbar_wait(full(s), (i / AS) & 1) || !mbar_wait(xfull(xs_), (i / kTqXs) & 1) ||
                    !mbar_wait(accempty(sl), ((i / NSL) & 1) ^ 1)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint64_t ad = umma_desc_sw128(sA + s * 16384);
                const uint64_t bd = umma_desc_sw128(sX + xs_ * XSB);
#pragma unroll
                for (int k32 = 0; k32 < 4; k32++) umma_i8(tmem + sl * NP, ad + 2 * k32, bd + 2 * k32, idesc, k32 != 0);
                umma_commit(empty(s));
                umma_commit(accfull(sl));
            }
            if (!ok) {
                atomicOr(a.err, kTqErr);
                atomicExch(&s_abort, 1);
            }
        }
        __syncwarp();
    } else {
        // ------------------------------ epilogue warps ------------------------------
        constexpr int NC = NP / (E / 4);  // accumulator columns of this warp
        constexpr int NBR = NC / 2;       // batch rows of this warp
        const int e = warp - (kTqProd + 2), q = warp & 3, h = e >> 2;
        const int r = 32 * q + lane, row = rb * 128 + r;
        const int T = rb * 8 + (r >> 4), rr = r & 15;
        const bool rlive = row < a.Nout;
        // INT4 scale word (f16 scale | f16 min << 16) of this row in block kb0 + j
        auto scale_word = [&](int j) -> uint32_t {
            if (KIND != kKindI4 || !rlive || j >= nk) return 0u;
            return __ldg(reinterpret_cast<const uint32_t*>(a.w + ((size_t)T * a.nkb + kb0 + j) * TB + 1024) +
                         2 * (rr & 7) + (rr >> 3));
        };
        uint32_t sq0 = scale_word(0), sq1 = scale_word(1), sq2 = scale_word(2), sq3 = scale_word(3);
        float acc[NBR];
#pragma unroll
        for (int j = 0; j < NBR; j++) acc[j] = 0.f;
        pdl_wait();  // y and resid are touched only after the preceding kernel finished
        asm volatile("bar.sync 1, %0;" ::"r"(32 * (1 + E)) : "memory");  // the TMEM allocation is done
        tc_fence_after();
        const uint32_t tmem = *tmem_slot;
        int i = 0;
        bool ok = true;
        for (; i < nk; i++) {
            const int sl = i % NSL, xs_ = i % kTqXs;
            if (!__all_sync(0xffffffffu, mbar_wait(accfull(sl), (i / NSL) & 1))) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t sw = sq0;
            sq0 = sq1;
            sq1 = sq2;
            sq2 = sq3;
            sq3 = scale_word(i + kTqPf);
            const float2 smn = __half22float2(*reinterpret_cast<const __half2*>(&sw));  // (scale, min)
            const float2* xm = reinterpret_cast<const float2*>(smem + (sX - sA) + xs_ * XSB + NP * 128) + h * NBR;
#pragma unroll
            for (int c0 = 0; c0 < NC; c0 += 32) {
                float v[32];
                tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + sl * NP + h * NC + c0, v);
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    const int S = __float_as_int(v[2 * j]) * 128 + __float_as_int(v[2 * j + 1]);  // exact: |S| < 2^25
                    const float2 m = xm[c0 / 2 + j];
                    if (KIND == kKindI4) acc[c0 / 2 + j] = fmaf(smn.x, (float)S * m.x, fmaf(smn.y, m.y, acc[c0 / 2 + j]));
                    else acc[c0 / 2 + j] = fmaf((float)S, m.x, acc[c0 / 2 + j]);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(accempty(sl));
                mbar_arrive(xempty(xs_));
            }
        }
        if (!ok && lane == 0) {
            atomicOr(a.err, kTqErr);
            atomicExch(&s_abort, 1);
        }
        __syncwarp();
        // results of this CTA: y (one split) or its partial
        if (ok && rlive) {
            float* dst = a.S > 1 ? a.ws + (size_t)split * a.Bp * a.Nout : a.y;
#pragma unroll
            for (int j = 0; j < NBR; j++) {
                const int b = h * NBR + j;
                if (b < a.B) {
                    const size_t o = (size_t)b * a.Nout + row;
                    float v = acc[j] * (a.row_scale ? a.row_scale[row] : a.wscale);
                    if (a.S == 1 && a.resid) v += a.resid[o];
                    dst[o] = v;
                }
            }
        }
    }

    __syncthreads();  // every role is done; the abort decision is visible
    const bool go = !*(volatile int*)&s_abort;
    if (go && a.S > 1) {
        // the last CTA of the row block adds the S partials in split order
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
            // all splits' loads of an item are issued before the sum (one L2 round trip per item),
            // four rows per item when y, resid and the rows are 16-byte aligned
            const int r0 = rb * 128, nrow = min(128, a.Nout - r0);
            const bool vec = (a.Nout & 3) == 0 && ((uintptr_t)a.y & 15) == 0 && ((uintptr_t)a.resid & 15) == 0;
            const int per_b = vec ? (nrow + 3) / 4 : nrow;
            for (int it = tid; it < a.B * per_b; it += blockDim.x) {
                const int b = it / per_b, qq = it % per_b;
                if (vec) {
                    const size_t o = (size_t)b * a.Nout + r0 + 4 * qq;
                    float4 part[16];
#pragma unroll
                    for (int sp = 0; sp < 16; sp++)
                        if (sp < a.S) part[sp] = __ldcg(reinterpret_cast<const float4*>(a.ws + (size_t)sp * a.Bp * a.Nout + o));
                    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                    for (int sp = 0; sp < 16; sp++)
                        if (sp < a.S) {
                            acc.x += part[sp].x;
                            acc.y += part[sp].y;
                            acc.z += part[sp].z;
                            acc.w += part[sp].w;
                        }
                    if (a.resid) {
                        const float4 rv = *reinterpret_cast<const float4*>(a.resid + o);
                        acc.x += rv.x;
                        acc.y += rv.y;
                        acc.z += rv.z;
                        acc.w += rv.w;
                    }
                    *reinterpret_cast<float4*>(a.y + o) = acc;
                } else {
                    const size_t o = (size_t)b * a.Nout + r0 + qq;
                    float part[16];
#pragma unroll
                    for (int sp = 0; sp < 16; sp++)
                        if (sp < a.S) part[sp] = __ldcg(a.ws + (size_t)sp * a.Bp * a.Nout + o);
                    float acc = 0.f;
#pragma unroll
                    for (int sp = 0; sp < 16; sp++)
                        if (sp < a.S) acc += part[sp];
                    if (a.resid) acc += a.resid[o];
                    a.y[o] = acc;
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();  // every TMEM read has completed (tcgen05.wait::ld) before the deallocation
    if (warp == kTqProd) {
        tc_fence_after();
        tmem_dealloc(*tmem_slot, tq_tmem_cols(NP));
    }
}

// x preparation of the integer small-M path: one warp per (padded batch row n < Bp, 128-k block),
// lane l covering k = 4l .. 4l+3, the arithmetic of xprep_int_kernel; the two limbs of row n are
// rows 2n (hi) and 2n + 1 (lo) of the block's 128-byte-swizzled [2Bp][128 B] tile, and (max|x| /
// 16383, sum x) goes to meta[kb][n]. Rows n >= B are zero.
__global__ void __launch_bounds__(256) xprep_tq_kernel(const float* __restrict__ x, int B, int Bp, int K, PrepOp op,
                                                       uint8_t* __restrict__ xl, float2* __restrict__ xm) {
    pdl_launch_dependents();
    pdl_wait();
    const int nkb = K / 128;
    const int nwb = blockDim.x >> 5, wid0 = blockIdx.x * nwb;
    const int wid = wid0 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    __shared__ float s_inv[8];
    const int b0 = wid0 / nkb;
    if (op.mode == kPrepNorm && b0 < B) {
        const int b1 = min(B - 1, min(Bp * nkb - 1, wid0 + nwb - 1) / nkb);
        block_rms_inv(x, op.ld_x, K, op.eps, b0, b1, s_inv);
    }
    if (wid >= Bp * nkb) return;
    const int n = wid / nkb, kb = wid % nkb;
    const int k = kb * 128 + 4 * lane;
    float e[4] = {0.f, 0.f, 0.f, 0.f};
    if (n < B) {
        PrepRow r;
        r.x = x + (size_t)n * op.ld_x;
        r.up = op.up ? op.up + (size_t)n * op.ld_up : nullptr;
        r.inv = op.mode == kPrepNorm ? s_inv[n - b0] : 1.f;
        const float4 v = *reinterpret_cast<const float4*>(r.x + k);  // K % 128 == 0
        e[0] = prep_elem(op, r, k, v.x);
        e[1] = prep_elem(op, r, k + 1, v.y);
        e[2] = prep_elem(op, r, k + 2, v.z);
        e[3] = prep_elem(op, r, k + 3, v.w);
    }
    const float m = warp_max(fmaxf(fmaxf(fabsf(e[0]), fabsf(e[1])), fmaxf(fabsf(e[2]), fabsf(e[3]))));
    const float inv = m > 0.f ? (float)kXLimbMax / m : 0.f;
    uint32_t hi = 0, lo = 0;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int X = max(-kXLimbMax, min(kXLimbMax, __float2int_rn(e[i] * inv)));
        hi |= ((uint32_t)(X >> 7) & 0xFFu) << (8 * i);
        lo |= ((uint32_t)X & 0x7Fu) << (8 * i);
    }
    uint8_t* base = xl + (size_t)kb * (2 * Bp) * 128;
    const uint32_t off = 4u * (lane & 3);  // byte of k inside its 16-byte chunk (chunk = lane / 4)
    *reinterpret_cast<uint32_t*>(base + sw128_off(2 * n, lane >> 2) + off) = hi;
    *reinterpret_cast<uint32_t*>(base + sw128_off(2 * n + 1, lane >> 2) + off) = lo;
    const float s = warp_sum((e[0] + e[1]) + (e[2] + e[3]));
    if (lane == 0) xm[(size_t)kb * Bp + n] = make_float2(m > 0.f ? m / (float)kXLimbMax : 0.f, s);
}

cudaError_t launch_xprep_tq(const float* x, int B, int Bp, int K, const PrepOp& op_in, uint8_t* xl, float2* xm,
                            cudaStream_t st) {
    PrepOp op = op_in;
    if (op.ld_x == 0) op.ld_x = K;
    const int warps = Bp * (K / 128);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((warps + 7) / 8), 1, 1);
    cfg.blockDim = dim3(256, 1, 1);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, xprep_tq_kernel, x, B, Bp, K, op, xl, xm);
}

template <int KIND, int NP>
static cudaError_t launch_tq_t(const TqArgs& a, cudaStream_t st) {
    const int bytes = tq_smem(KIND, NP) + 1024;
    const cudaError_t e = cudaFuncSetAttribute(gemm_tq_kernel<KIND, NP>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((a.Nout + 127) / 128), (unsigned)a.S, 1);
    cfg.blockDim = dim3(tq_threads(NP), 1, 1);
    cfg.dynamicSmemBytes = bytes;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, gemm_tq_kernel<KIND, NP>, a);
}

template <int KIND>
static cudaError_t launch_tq_kind(const TqArgs& a, cudaStream_t st) {
    switch (a.Bp) {
        case 16: return launch_tq_t<KIND, 32>(a, st);
        case 32: return launch_tq_t<KIND, 64>(a, st);
        case 64: return launch_tq_t<KIND, 128>(a, st);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_tq(int kind, const TqArgs& a, cudaStream_t st) {
    if (kind == kKindI4) return launch_tq_kind<kKindI4>(a, st);
    if (kind == kKindI8) return launch_tq_kind<kKindI8>(a, st);
    return cudaErrorInvalidValue;
}

}  // namespace pox
