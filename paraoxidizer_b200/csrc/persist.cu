// persist.cu -- every layer of a decode step in one persistent kernel (batch 1..4, one GPU).
//
// The per-layer path (engine.cu) runs 9 dependent launches per layer; at batch 1 their fixed costs
// (ramp, drain, the launch hop of each link) outweigh the weight stream. Here one cooperative launch
// of one CTA per SM runs the layers of forward_token (crates/paraoxidizer-runtime/src/engine.rs:
// 411-700) stage by stage:
//   A  xq = limbs(rmsnorm(x, attn_norm));  qkv = W_qkv xq
//   B  attention items (sequence, kv head, 64-token split) on the tensor cores, RoPE and the KV
//      append fused; the item that finishes a (sequence, kv head) last combines its splits -> att
//   D  xq = limbs(att);                    x += W_o xq
//   E  xq = limbs(rmsnorm(x, mlp_norm));   gu = W_gu xq
//   F  xq = limbs(silu(g) * u);            x += W_down xq
// with a grid barrier (bounded wait) after A, B, D, E and F. Every CTA prepares the whole input of a
// stage itself (x is at most a few tens of KB); the o and down stages leave per-row-tile sums of
// squares, so an RMSNorm input takes one round trip.
//
// Warps 0-7 consume, warp 8 produces. The weights are the INT4 tiles of the GEMV path (gemv.cuh
// TileLayout; 16 rows x 128 k + 16 scale words, 1088 B, a row tile's k-blocks contiguous). CTA c
// takes the row tiles c, c + grid, ... of each projection; the producer copies each row tile in
// chunks of up to 32 k-blocks (one 34 KB bulk copy each) into a ring of chunk slots, walking the
// CTA's whole sequence across projections, stages and layers, so while the consumers wait at a
// barrier or run attention the next projection's weights are already arriving (they are
// immutable: no dependency). The consumers accumulate with mma.sync m16n8k32 u8 x s8 on the exact
// two-limb x and reduce a row tile's eight warp partials through shared memory in warp order
// (deterministic).
//
// Cross-CTA data (x, qkv, att, gu, the attention partials, the sums of squares) is read with
// ld.global.cg, from L2, never from a possibly stale L1 line.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>

#include "../../include/pox_cuda.h"
#include "api_internal.h"
#include "attn.cuh"
#include "common.cuh"
#include "gemv.cuh"
#include "model.h"
#include "persist.h"

namespace pox {

constexpr int kPCons = 8;                   // consumer warps: preparation, GEMV tiles, attention items
constexpr int kPConsThreads = kPCons * 32;  // 256
constexpr int kPThreads = kPConsThreads + 32;  // + the producer warp (warp 8)
constexpr int kPGroups = 2;     // attention items run by warps 0-3 and 4-7 (named barriers 1 and 2)
constexpr int kConsBar = 3;     // named barrier of the 8 consumer warps
constexpr int kPTile = kTileBytes + 64;     // INT4 tile + its scale words
constexpr int kChunkTiles = 32;             // tiles per weight copy (consecutive k-blocks of one row tile)
constexpr int kChunkBytes = kChunkTiles * kPTile;  // 34816

__device__ __forceinline__ float4 ldcg4(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }
__device__ __forceinline__ void cons_sync() { named_sync(kConsBar, kPConsThreads); }
// barrier of the consumer warps that also ANDs a predicate over them
__device__ __forceinline__ bool cons_sync_and(bool p) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred pi, po;\n setp.ne.u32 pi, %1, 0;\n bar.red.and.pred po, %2, %3, pi;\n selp.u32 %0, 1, 0, po;\n}"
        : "=r"(r)
        : "r"((uint32_t)p), "r"(kConsBar), "r"(kPConsThreads)
        : "memory");
    return r != 0;
}

// Grid barrier of the persistent kernel, run by the consumer warps of every CTA: bar[0] counts the
// arrivals of this launch (the k-th barrier of a launch completes at (k + 1) x grid arrivals; the
// count is reset when the last CTA exits), bar[2] is the abort word: once a wait has run out every
// later barrier of the launch returns at once and the CTAs wind down. Arrival is a release
// reduction (no round trip); the wait polls the count. Returns false when the launch is aborted.
__device__ __forceinline__ bool grid_sync(unsigned* bar, unsigned target, int* err, int* s_flag) {
    cons_sync();
    if (threadIdx.x == 0) {
        int ok = *(volatile unsigned*)(bar + 2) == 0u;
        if (ok) {
            __threadfence();  // this CTA's writes (ordered before by the consumer barrier) before the arrival
            asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(bar) : "memory");
            const long long t0 = clock64();
            for (;;) {
                unsigned n;
                asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(n) : "l"(bar) : "memory");
                if ((int)(n - target) >= 0) break;
                if (*(volatile unsigned*)(bar + 2) != 0u) {
                    ok = 0;
                    break;
                }
                if (clock64() - t0 > kWaitCycles) {
                    atomicOr(err, kErrPersist);
                    atomicExch(bar + 2, 1u);
                    ok = 0;
                    break;
                }
            }
            __threadfence();  // acquire: the other CTAs' writes before this CTA's reads
        }
        *s_flag = ok;
    }
    cons_sync();
    return *(volatile int*)s_flag != 0;
}

// Input of one projection, prepared in shared memory by the consumer warps: per batch row b and
// 128-k block, X = rint(v * 16383 / max|v|) as two exact int8 limbs (column 2b: hi, 2b + 1: lo; cs
// bytes per column) and meta[b][blk] = (max|v| / 16383, sum v), the arithmetic of xprep_int_kernel.
// Warp w takes blocks w, w + 8, ... a few at a time: every load of a round is issued before the
// first use, and the blocks' reductions are interleaved step by step so the warp overlaps their
// latencies (eight warps per SM are too few to hide them otherwise). Sums are reduced in a fixed
// order (deterministic).
constexpr int kPrepBatch = 4;

template <int N>
__device__ __forceinline__ void prep_quant_n(const float4 (&x)[N], int w0, int nw, int nxb, int lane,
                                             unsigned char* xs, int cs, float2* xm, int nxbs) {
    float m[N], s[N];
#pragma unroll
    for (int j = 0; j < N; j++) {
        m[j] = fmaxf(fmaxf(fabsf(x[j].x), fabsf(x[j].y)), fmaxf(fabsf(x[j].z), fabsf(x[j].w)));
        s[j] = (x[j].x + x[j].y) + (x[j].z + x[j].w);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int j = 0; j < N; j++) {
            m[j] = fmaxf(m[j], __shfl_xor_sync(0xffffffffu, m[j], o));
            s[j] += __shfl_xor_sync(0xffffffffu, s[j], o);
        }
#pragma unroll
    for (int j = 0; j < N; j++) {
        const int wi = w0 + j * kPCons;
        if (wi >= nw) continue;
        const int b = wi / nxb, blk = wi % nxb, k = blk * kXBlock + 4 * lane;
        const float qi = m[j] > 0.f ? (float)kXLimbMax / m[j] : 0.f;
        const int X[4] = {__float2int_rn(x[j].x * qi), __float2int_rn(x[j].y * qi), __float2int_rn(x[j].z * qi),
                          __float2int_rn(x[j].w * qi)};
        uint32_t hi = 0, lo = 0;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int q = max(-kXLimbMax, min(kXLimbMax, X[i]));
            hi |= ((uint32_t)(q >> 7) & 0xFFu) << (8 * i);
            lo |= ((uint32_t)q & 0x7Fu) << (8 * i);
        }
        *reinterpret_cast<uint32_t*>(xs + (size_t)(2 * b) * cs + k) = hi;
        *reinterpret_cast<uint32_t*>(xs + (size_t)(2 * b + 1) * cs + k) = lo;
        if (lane == 0) xm[b * nxbs + blk] = make_float2(m[j] > 0.f ? m[j] / (float)kXLimbMax : 0.f, s[j]);
    }
}

// RMSNorm: x * inv_rms, times the f16 weight when there is one (engine.rs:294-350)
__device__ __forceinline__ float4 rms_scale(float4 x, float inv, uint2 w, bool has_w) {
    x.x *= inv, x.y *= inv, x.z *= inv, x.w *= inv;
    if (has_w) {
        x.x *= half_bits_to_float(w.x), x.y *= half_bits_to_float(w.x >> 16);
        x.z *= half_bits_to_float(w.y), x.w *= half_bits_to_float(w.y >> 16);
    }
    return x;
}

// mode kPrepNone: v = src[b][k]; kPrepNorm: v = rmsnorm(src[b])[k], the sums of squares from a first
// pass (the embedding's rows: nothing left them). src rows ld floats apart, K % 128 == 0.
__device__ __noinline__ void prep_stage(int mode, const float* src, int ld, const uint16_t* nw_, float eps, int K,
                                        int B, unsigned char* xs, int cs, float2* xm, int nxbs, float* s_red,
                                        float* s_inv) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nxb = K / kXBlock, nw = B * nxb;
    float4 v[kPrepBatch];
    if (mode == kPrepNorm) {
        // sums of squares of every row, per thread in block order, then warps, then the warps in order
        float ss[kPMaxB] = {0.f, 0.f, 0.f, 0.f};
        for (int w0 = warp; w0 < nw; w0 += kPrepBatch * kPCons) {
#pragma unroll
            for (int j = 0; j < kPrepBatch; j++) {
                const int wi = min(w0 + j * kPCons, nw - 1);
                v[j] = ldcg4(src + (size_t)(wi / nxb) * ld + (wi % nxb) * kXBlock + 4 * lane);
            }
#pragma unroll
            for (int j = 0; j < kPrepBatch; j++) {
                const int wi = w0 + j * kPCons;
                if (wi < nw) {
                    const float q = fmaf(v[j].w, v[j].w, fmaf(v[j].z, v[j].z, fmaf(v[j].y, v[j].y, v[j].x * v[j].x)));
                    const int b = wi / nxb;
#pragma unroll
                    for (int bb = 0; bb < kPMaxB; bb++) ss[bb] += b == bb ? q : 0.f;
                }
            }
        }
#pragma unroll
        for (int bb = 0; bb < kPMaxB; bb++) {
            const float t = warp_sum(ss[bb]);
            if (lane == 0) s_red[warp * kPMaxB + bb] = t;
        }
        cons_sync();
        if (tid < B) {
            float t = 0.f;
            for (int w = 0; w < kPCons; w++) t += s_red[w * kPMaxB + tid];
            s_inv[tid] = 1.0f / sqrtf(t / (float)K + eps);
        }
        cons_sync();
    }
    for (int w0 = warp; w0 < nw; w0 += kPrepBatch * kPCons) {
        uint2 wv[kPrepBatch];
#pragma unroll
        for (int j = 0; j < kPrepBatch; j++) {
            const int wi = min(w0 + j * kPCons, nw - 1);
            const int k = (wi % nxb) * kXBlock + 4 * lane;
            v[j] = ldcg4(src + (size_t)(wi / nxb) * ld + k);
            wv[j] = nw_ ? *reinterpret_cast<const uint2*>(nw_ + k) : make_uint2(0u, 0u);
        }
        if (mode == kPrepNorm)
#pragma unroll
            for (int j = 0; j < kPrepBatch; j++)
                v[j] = rms_scale(v[j], s_inv[min(w0 + j * kPCons, nw - 1) / nxb], wv[j], nw_ != nullptr);
        prep_quant_n<kPrepBatch>(v, w0, nw, nxb, lane, xs, cs, xm, nxbs);
    }
    cons_sync();
}

// RMSNorm input from the residual rows and the sums of squares their producers left (ssq: nparts
// partial sums per x row, summed here in index order), prepared like prep_stage. The x, weight and
// partial loads of the first round are issued together (one round trip).
__device__ __noinline__ void prep_norm_ssq(const float* src, const float* ssq, int nparts, const uint16_t* nw_,
                                           float eps, int K, int B, unsigned char* xs, int cs, float2* xm, int nxbs,
                                           float* s_red, float* s_inv) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nxb = K / kXBlock, nw = B * nxb;
    float4 v[kPrepBatch];
    uint2 wv[kPrepBatch];
#pragma unroll
    for (int j = 0; j < kPrepBatch; j++) {
        const int wi = min(warp + j * kPCons, nw - 1);
        const int k = (wi % nxb) * kXBlock + 4 * lane;
        v[j] = ldcg4(src + (size_t)(wi / nxb) * K + k);
        wv[j] = nw_ ? *reinterpret_cast<const uint2*>(nw_ + k) : make_uint2(0u, 0u);
    }
    float ss[kPMaxB] = {0.f, 0.f, 0.f, 0.f};
    for (int p = tid; p < nparts; p += kPConsThreads) {
        const float4 q = ldcg4(ssq + (size_t)p * kPMaxB);
        ss[0] += q.x, ss[1] += q.y, ss[2] += q.z, ss[3] += q.w;
    }
#pragma unroll
    for (int bb = 0; bb < kPMaxB; bb++) {
        const float t = warp_sum(ss[bb]);
        if (lane == 0) s_red[warp * kPMaxB + bb] = t;
    }
    cons_sync();
    if (tid < B) {
        float t = 0.f;
        for (int w = 0; w < kPCons; w++) t += s_red[w * kPMaxB + tid];
        s_inv[tid] = 1.0f / sqrtf(t / (float)K + eps);
    }
    cons_sync();
    for (int w0 = warp; w0 < nw; w0 += kPrepBatch * kPCons) {
        if (w0 != warp) {
#pragma unroll
            for (int j = 0; j < kPrepBatch; j++) {
                const int wi = min(w0 + j * kPCons, nw - 1);
                const int k = (wi % nxb) * kXBlock + 4 * lane;
                v[j] = ldcg4(src + (size_t)(wi / nxb) * K + k);
                wv[j] = nw_ ? *reinterpret_cast<const uint2*>(nw_ + k) : make_uint2(0u, 0u);
            }
        }
#pragma unroll
        for (int j = 0; j < kPrepBatch; j++)
            v[j] = rms_scale(v[j], s_inv[min(w0 + j * kPCons, nw - 1) / nxb], wv[j], nw_ != nullptr);
        prep_quant_n<kPrepBatch>(v, w0, nw, nxb, lane, xs, cs, xm, nxbs);
    }
    cons_sync();
}

// down's input v = g / (1 + exp(-g)) * u (engine.rs:671-677) prepared like prep_stage: a warp's
// blocks 7 at a time (the 112 blocks of the 8B model's FFN at one row of x in two rounds), every
// load of a round issued before the first use and the blocks' arithmetic interleaved.
constexpr int kSwiBatch = 7;
__device__ __noinline__ void prep_swiglu(const float* gu, int I, int B, unsigned char* xs, int cs, float2* xm,
                                         int nxbs) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nxb = I / kXBlock, nw = B * nxb;
    for (int w0 = warp; w0 < nw; w0 += kSwiBatch * kPCons) {
        float4 g[kSwiBatch], u[kSwiBatch];
#pragma unroll
        for (int j = 0; j < kSwiBatch; j++) {
            const int wi = min(w0 + j * kPCons, nw - 1);
            const float* r = gu + (size_t)(wi / nxb) * 2 * I + (wi % nxb) * kXBlock + 4 * lane;
            g[j] = ldcg4(r);
            u[j] = ldcg4(r + I);
        }
#pragma unroll
        for (int j = 0; j < kSwiBatch; j++) {  // fast exp and divide: far below the 15-bit limbs' rounding
            g[j].x = __fdividef(g[j].x, 1.0f + __expf(-g[j].x)) * u[j].x;
            g[j].y = __fdividef(g[j].y, 1.0f + __expf(-g[j].y)) * u[j].y;
            g[j].z = __fdividef(g[j].z, 1.0f + __expf(-g[j].z)) * u[j].z;
            g[j].w = __fdividef(g[j].w, 1.0f + __expf(-g[j].w)) * u[j].w;
        }
        prep_quant_n<kSwiBatch>(g, w0, nw, nxb, lane, xs, cs, xm, nxbs);
    }
    cons_sync();
}

// Combines the splits of (sequence b, kv head h): att = sum_s e^(m_s - M) acc_s / sum_s e^(m_s - M) l_s
// for each of its G query heads (1 / sum_exp, 0 when the sum is <= 1e-9), the arithmetic of
// attn_combine_kernel. 128 threads: warp w takes heads w and w + 4, lane l dims 4 l .. 4 l + 3; the
// (max, sum) pairs and the accumulators of up to 16 splits are loaded in one round (partials are
// read from L2: other CTAs wrote them), the weights e^(m_s - M) shared through shuffles.
__device__ __noinline__ void combine_head(const PArgs& a, int b, int h, int ns, int gt, int K_att) {
    const int w = gt >> 5, lane = gt & 31;
    const size_t sstride = (size_t)a.G * 130;
    for (int gq = w; gq < a.G; gq += 4) {
        const float* base = a.apart + (((size_t)b * a.nkv + h) * a.max_splits * a.G + gq) * 130;
        float4 num = make_float4(0.f, 0.f, 0.f, 0.f);
        float M = -INFINITY, den = 0.f;
        // splits in chunks of 16; M and den are exact running values (rescaled per chunk)
        for (int s0 = 0; s0 < ns; s0 += 16) {
            const int n = min(16, ns - s0);
            const float2 ml = lane < n ? __ldcg(reinterpret_cast<const float2*>(base + (s0 + lane) * sstride))
                                       : make_float2(-INFINITY, 0.f);
            float2 v[16][2];
#pragma unroll
            for (int j = 0; j < 16; j++) {
                const float* pp = base + (s0 + min(j, n - 1)) * sstride;
                v[j][0] = __ldcg(reinterpret_cast<const float2*>(pp + 2 + 4 * lane));
                v[j][1] = __ldcg(reinterpret_cast<const float2*>(pp + 4 + 4 * lane));
            }
            const float Mc = fmaxf(M, warp_max(ml.x));
            const float sc = expf(M - Mc);  // rescale what earlier chunks summed (M = -inf: 0)
            const float wl = lane < n ? expf(ml.x - Mc) : 0.f;
            den = fmaf(den, sc, warp_sum(wl * ml.y));
            num.x *= sc, num.y *= sc, num.z *= sc, num.w *= sc;
#pragma unroll
            for (int j = 0; j < 16; j++) {
                const float wt = __shfl_sync(0xffffffffu, wl, j);  // 0 past the chunk
                num.x = fmaf(wt, v[j][0].x, num.x);
                num.y = fmaf(wt, v[j][0].y, num.y);
                num.z = fmaf(wt, v[j][1].x, num.z);
                num.w = fmaf(wt, v[j][1].y, num.w);
            }
            M = Mc;
        }
        const float inv = den > 1e-9f ? 1.0f / den : 0.f;
        float* o = a.att + (size_t)b * K_att + (size_t)(h * a.G + gq) * 128 + 4 * lane;
        o[0] = num.x * inv;
        o[1] = num.y * inv;
        o[2] = num.z * inv;
        o[3] = num.w * inv;
    }
}

// One attention item, compiled as a separate function: its registers do not add to the pressure of
// the weight loops around it.
__device__ __noinline__ void persist_attn_item(const PArgs& a, int b, int h, int split, int l, AttnTcSmem& sm, int gt,
                                               int bar) {
    float* out = a.apart + ((((size_t)b * a.nkv + h) * a.max_splits + split) * a.G) * 130;
    attn_tc_item<kAttnDecode>(a.qkv + (size_t)b * a.qkv_rows, a.pos[b], a.btab + (size_t)b * a.mbps, a.kv_blocks,
                              a.kc, a.vc, l, a.L, a.nq, a.nkv, h, a.G, a.rope, split, out, a.err, sm, gt, bar);
}

// The weight stream. Each projection's row tiles u = cta, cta + grid, ... are cut into chunks of up
// to 32 consecutive k-blocks (consecutive 1088-byte tiles in memory); the producer warp copies one
// chunk per bulk copy into a ring of S chunk slots, running ahead across projections, stages and
// layers (weights are immutable). Slot s has a full barrier (the copy's bytes) and an empty barrier
// (one arrival per consumer warp).
struct ChunkRing {
    uint32_t base, full, empty;  // shared addresses: slots, full barriers [S], empty barriers [S]
    int S, slot;
    uint32_t phase;
};

struct GemvSmem {
    unsigned char* xs;
    float2* xm;
    float* red;
    int cs, nxbs;
    uint32_t zero;
};

// One projection on the consumer warps: y[b][row] (+ y when add_resid) = sum_k W[row][k] x[b][k]
// over this CTA's row tiles, x prepared in shared memory. In a chunk of n tiles, warp w takes tiles
// w, w + 8, ...; the eight warps' partial sums of a row tile are reduced in warp order. ok turns
// false (consumer-uniform) when a wait ran out; rs alternates the two partial slots.
__device__ __forceinline__ void gemv_stage(const PArgs& a, ChunkRing& r, const GemvSmem& gs, int st, float* y, int N,
                                           bool add_resid, bool& ok, int& rs) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
    const int cta = blockIdx.x, ncta = gridDim.x, B = a.B;
    const int nT = a.nT[st], nkb = a.nkb[st];
    for (int u = cta; u < nT && ok; u += ncta) {
        float acc0 = 0.f, acc1 = 0.f;  // rows g and g + 8 of the tile, x row t
        for (int c0 = 0; c0 < nkb; c0 += kChunkTiles) {
            const int n = min(kChunkTiles, nkb - c0);
            const bool f_ok = __all_sync(0xffffffffu, mbar_wait(r.full + 8 * r.slot, r.phase));
            if (!f_ok) {
                if (lane == 0) {
                    atomicOr(a.err, kErrPersist);
                    atomicExch(a.bar + 2, 1u);
                }
                ok = false;
                break;
            }
            const uint32_t cb = r.base + (uint32_t)r.slot * kChunkBytes;
            for (int j = warp; j < n; j += kPCons) {
                const uint32_t sa = cb + (uint32_t)j * kPTile;
                const uint4 wa = lds128(sa + lane * 16), wb = lds128(sa + 512 + lane * 16);
                const uint2 scw = lds64(sa + kTileBytes + 8 * g);
                const int kb = c0 + j;
                // x fragments: column g = 2 b + limb (b < B), k = 128 kb + 32 t .. + 31
                const bool xv = g < 2 * B;
                const uint32_t xa = xv ? smem_u32(gs.xs) + (uint32_t)(g * gs.cs + kb * 128 + 32 * t) : gs.zero;
                const uint4 v0 = lds128(xa), v1 = lds128(xv ? xa + 16 : gs.zero);
                int dl[4] = {0, 0, 0, 0}, dh[4] = {0, 0, 0, 0};
                imma_16832_u8s8(dl, wa.x & 0x0F0F0F0Fu, wb.x & 0x0F0F0F0Fu, wa.y & 0x0F0F0F0Fu, wb.y & 0x0F0F0F0Fu,
                                v0.x, v0.z);
                imma_16832_u8s8(dh, wa.x & 0xF0F0F0F0u, wb.x & 0xF0F0F0F0u, wa.y & 0xF0F0F0F0u, wb.y & 0xF0F0F0F0u,
                                v0.y, v0.w);
                imma_16832_u8s8(dl, wa.z & 0x0F0F0F0Fu, wb.z & 0x0F0F0F0Fu, wa.w & 0x0F0F0F0Fu, wb.w & 0x0F0F0F0Fu,
                                v1.x, v1.z);
                imma_16832_u8s8(dh, wa.z & 0xF0F0F0F0u, wb.z & 0xF0F0F0F0u, wa.w & 0xF0F0F0F0u, wb.w & 0xF0F0F0F0u,
                                v1.y, v1.w);
                if (t < B) {
                    const float2 mt = gs.xm[t * gs.nxbs + kb];
                    const float sx = mt.x * 0.0625f;  // S below is 16 * sum q X
                    const float2 s0 = __half22float2(*reinterpret_cast<const __half2*>(&scw.x));
                    const float2 s1 = __half22float2(*reinterpret_cast<const __half2*>(&scw.y));
                    const int S0 = (dl[0] * 16 + dh[0]) * 128 + (dl[1] * 16 + dh[1]);
                    const int S1 = (dl[2] * 16 + dh[2]) * 128 + (dl[3] * 16 + dh[3]);
                    acc0 = fmaf(s0.x, (float)S0 * sx, fmaf(s0.y, mt.y, acc0));
                    acc1 = fmaf(s1.x, (float)S1 * sx, fmaf(s1.y, mt.y, acc1));
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(r.empty + 8 * r.slot);  // this warp is done with the slot
            if (++r.slot == r.S) r.slot = 0, r.phase ^= 1u;
        }
        float* rw = gs.red + (rs * kPCons + warp) * 64;
        if (t < B) {
            rw[g * 4 + t] = acc0;
            rw[(g + 8) * 4 + t] = acc1;
        }
        // one barrier per tile suffices: slot rs is written again two tiles later, after the next
        // barrier, which the threads reducing this tile reach only when they are done
        ok = cons_sync_and(ok);
        if (ok && warp < 2) {  // warps 0 and 1: rows 0-7 and 8-15 of the tile (lane = 4 row + x row)
            float v = 0.f;
            const int row = u * 16 + (tid >> 2);
            if ((tid & 3) < B) {
                float p = 0.f;
#pragma unroll
                for (int w = 0; w < kPCons; w++) p += gs.red[(rs * kPCons + w) * 64 + tid];
                if (row < N) {
                    const size_t o = (size_t)(tid & 3) * N + row;
                    v = add_resid ? __ldcg(y + o) + p : p;
                    y[o] = v;
                }
            }
            if (st == 1 || st == 3) {
                // the new residual rows' sums of squares (per x row, this warp's 8 rows) for the next RMSNorm
                float q = v * v;
                q += __shfl_xor_sync(0xffffffffu, q, 4);
                q += __shfl_xor_sync(0xffffffffu, q, 8);
                q += __shfl_xor_sync(0xffffffffu, q, 16);
                if (lane < kPMaxB) a.ssq[((size_t)u * 2 + warp) * kPMaxB + lane] = q;
            }
        }
        rs ^= 1;
    }
}

// The producer warp (lane 0): every chunk of this CTA's sequence -- layers, then qkv, o, gate_up,
// down, then row tiles u = cta, cta + grid, ..., then chunks of 32 k-blocks -- into the ring, each
// after the consumers released its slot. Stops when the launch is aborted or a wait runs out, and
// returns only when none of its copies is still in flight.
__device__ __forceinline__ void producer(const PArgs& a, ChunkRing r, const PLayer* lys) {
    const int cta = blockIdx.x, ncta = gridDim.x;
    long long issued = 0;
    bool ok = true;
    for (int l = 0; l < a.L && ok; l++)
        for (int st = 0; st < 4 && ok; st++) {
            const int nT = a.nT[st], nkb = a.nkb[st];
            const uint8_t* w = lys[l].w[st];
            for (int u = cta; u < nT && ok; u += ncta)
                for (int c0 = 0; c0 < nkb; c0 += kChunkTiles) {
                    const int n = min(kChunkTiles, nkb - c0);
                    if (issued >= r.S) {  // the slot's previous chunk must have been released
                        if (!mbar_wait(r.empty + 8 * r.slot, r.phase ^ 1u) ||
                            *(volatile unsigned*)(a.bar + 2) != 0u) {
                            if (*(volatile unsigned*)(a.bar + 2) == 0u) {
                                atomicOr(a.err, kErrPersist);
                                atomicExch(a.bar + 2, 1u);
                            }
                            ok = false;
                            break;
                        }
                    }
                    const uint32_t bar = r.full + 8 * r.slot;
                    mbar_expect_tx(bar, (uint32_t)(n * kPTile));
                    bulk_g2s(r.base + (uint32_t)r.slot * kChunkBytes, w + ((size_t)u * nkb + c0) * kPTile,
                             (uint32_t)(n * kPTile), bar);
                    issued++;
                    if (++r.slot == r.S) r.slot = 0, r.phase ^= 1u;
                }
        }
    // the last min(S, issued) copies may still be in flight (consumers that stopped early): wait
    const int left = (int)min((long long)r.S, issued);
    for (int j = 0; j < left; j++) {
        if (r.slot == 0) r.slot = r.S, r.phase ^= 1u;
        r.slot--;
        mbar_wait(r.full + 8 * r.slot, r.phase);
    }
}

__global__ void __launch_bounds__(kPThreads, 1) decode_persist_kernel(const __grid_constant__ PArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int cta = blockIdx.x, ncta = gridDim.x, S = a.S, B = a.B;
    // shared memory: chunk slots [S] | full barriers [S] | empty barriers [S] | x region (prepared x,
    // or the attention items) | warp partials [2][8][64] | scalars | layer table
    const uint32_t sbase = smem_u32(smem);
    ChunkRing ring;
    ring.base = sbase;
    ring.full = sbase + (uint32_t)(S * kChunkBytes);
    ring.empty = ring.full + 8u * S;
    ring.S = S;
    ring.slot = 0;
    ring.phase = 0;
    unsigned char* xreg = smem + a.off_x;
    float* red = reinterpret_cast<float*>(smem + a.off_red);
    float* s_red = red + 2 * kPCons * 64;        // [8 warps][4 rows]
    float* s_inv = s_red + kPCons * kPMaxB;      // [4]
    int* s_flag = reinterpret_cast<int*>(s_inv + kPMaxB);  // [1 + kPGroups] flags, then 16 zero bytes
    int* s_ns = s_flag + 8;                      // [4] attention splits per sequence
    // the layer table (tile pointers, norm weights) in shared memory
    PLayer* lys = reinterpret_cast<PLayer*>(smem + a.off_lys);
    for (int i = tid; i < a.L * (int)(sizeof(PLayer) / 8); i += kPThreads)
        reinterpret_cast<unsigned long long*>(lys)[i] = reinterpret_cast<const unsigned long long*>(a.layers)[i];
    if (tid < B) {
        const uint32_t p = a.pos[tid];
        s_ns[tid] = p < (uint32_t)a.mbps * kPage ? min(a.max_splits, (int)((p + kSplitTok) / kSplitTok)) : 0;
    }
    if (tid < 4) s_flag[4 + tid] = 0;
    if (tid == 0)
        for (int i = 0; i < S; i++) {
            mbar_init(ring.full + 8 * i, 1);
            mbar_init(ring.empty + 8 * i, kPCons);
        }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    __syncthreads();

    if (warp == kPCons) {
        if (lane == 0) producer(a, ring, lys);
    } else {
        unsigned char* xs = xreg;
        float2* xm = reinterpret_cast<float2*>(xreg + a.off_xm);
        const int cs = a.cs, nxbs = a.nxbs;
        GemvSmem gs{xs, xm, red, cs, nxbs, smem_u32(s_flag + 4)};
        bool ok = true;
        int rs = 0;  // partial slot of the next row tile
        const int K_att = a.nq * 128;
        unsigned bar_k = 0;  // arrivals that complete the next grid barrier
        for (int l = 0; l < a.L && ok; l++) {
            const PLayer& ly = lys[l];
            // ---- A: qkv = W_qkv rmsnorm(x) ----
            if (l == 0)  // the embedding has no sums of squares
                prep_stage(kPrepNorm, a.x, a.H, ly.attn_norm, a.eps, a.H, B, xs, cs, xm, nxbs, s_red, s_inv);
            else
                prep_norm_ssq(a.x, a.ssq, 2 * a.nT[3], ly.attn_norm, a.eps, a.H, B, xs, cs, xm, nxbs, s_red, s_inv);
            gemv_stage(a, ring, gs, 0, a.qkv, a.qkv_rows, false, ok, rs);
            if (!(ok = ok && grid_sync(a.bar, (bar_k += ncta), a.err, s_flag))) break;

            // ---- B: attention items and the combine of each (sequence, kv head) ----
            {
                const int* ns = s_ns;  // positions are fixed during a launch
                int total = 0;
                for (int b = 0; b < B; b++) {
                    total += a.nkv * ns[b];
                    if (!ns[b] && cta == 0) {  // beyond the block table: reported, output 0
                        if (tid == 0) atomicOr(a.err, kErrAttnPos);
                        for (int i = tid; i < K_att; i += kPConsThreads) a.att[(size_t)b * K_att + i] = 0.f;
                    }
                }
                const int grp = warp >> 2, gt = tid & 127;
                AttnTcSmem& sm = reinterpret_cast<AttnTcSmem*>(xreg)[grp];
                for (int it = cta * kPGroups + grp; it < total; it += ncta * kPGroups) {
                    int b = 0, r = it;
                    while (r >= a.nkv * ns[b]) r -= a.nkv * ns[b++];
                    const int h = r / ns[b], split = r % ns[b];
                    persist_attn_item(a, b, h, split, l, sm, gt, 1 + grp);
                    named_sync(1 + grp, 128);
                    if (gt == 0) {
                        __threadfence();
                        const unsigned prev = atomicAdd(a.tickets + b * a.nkv + h, 1u);
                        const int last = prev == (unsigned)(ns[b] - 1);
                        if (last) {
                            atomicExch(a.tickets + b * a.nkv + h, 0u);
                            __threadfence();
                        }
                        s_flag[1 + grp] = last;
                    }
                    named_sync(1 + grp, 128);
                    if (s_flag[1 + grp]) combine_head(a, b, h, ns[b], gt, K_att);
                }
            }
            if (!(ok = ok && grid_sync(a.bar, (bar_k += ncta), a.err, s_flag))) break;

            // ---- D: x += W_o att ----
            prep_stage(kPrepNone, a.att, K_att, nullptr, 0.f, K_att, B, xs, cs, xm, nxbs, s_red, s_inv);
            gemv_stage(a, ring, gs, 1, a.x, a.H, true, ok, rs);
            if (!(ok = ok && grid_sync(a.bar, (bar_k += ncta), a.err, s_flag))) break;

            // ---- E: gu = W_gu rmsnorm(x) ----
            prep_norm_ssq(a.x, a.ssq, 2 * a.nT[1], ly.mlp_norm, a.eps, a.H, B, xs, cs, xm, nxbs, s_red, s_inv);
            gemv_stage(a, ring, gs, 2, a.gu, 2 * a.I, false, ok, rs);
            if (!(ok = ok && grid_sync(a.bar, (bar_k += ncta), a.err, s_flag))) break;

            // ---- F: x += W_down silu(g) * u ----
            prep_swiglu(a.gu, a.I, B, xs, cs, xm, nxbs);
            gemv_stage(a, ring, gs, 3, a.x, a.H, true, ok, rs);
            if (l + 1 < a.L && !(ok = ok && grid_sync(a.bar, (bar_k += ncta), a.err, s_flag))) break;
        }
        if (!ok && tid == 0) atomicExch(a.bar + 2, 1u);  // the producer stops at its next wait
    }
    // the last CTA out resets the arrival count and the abort word for the next launch
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        if (atomicAdd(a.bar + 3, 1u) == (unsigned)ncta - 1) {
            atomicExch(a.bar, 0u);
            atomicExch(a.bar + 2, 0u);
            atomicExch(a.bar + 3, 0u);
        }
    }
}

// ---- host side ----
struct PPlan {
    int S = 0, off_x = 0, off_xm = 0, off_red = 0, off_lys = 0, cs = 0, nxbs = 0, total = 0;
};

static PPlan persist_plan(const pox_model* m, int B) {
    PPlan p;
    const int Kp = std::max(std::max(m->H, m->nq * 128), m->I);  // multiples of 128
    p.cs = Kp + 16;  // neighbouring columns in different banks
    p.nxbs = (Kp / kXBlock + 1) & ~1;
    const int xbytes = 2 * B * p.cs;
    p.off_xm = (xbytes + 15) & ~15;
    const int xreg = std::max(p.off_xm + B * p.nxbs * 8, kPGroups * (int)sizeof(AttnTcSmem));
    const int xreg_a = (xreg + 127) & ~127;
    const int scal = 256;  // sums of squares [8][4], RMSNorm scales [4], flags, zero bytes, split counts
    const int tail = 2 * kPCons * 64 * 4 + scal + (int)sizeof(PLayer) * m->L;  // partials, scalars, layer table
    const int budget = 227 * 1024 - xreg_a - tail;
    p.S = std::min(8, budget / (kChunkBytes + 16));
    if (p.S < 2) {
        p.S = 0;
        return p;
    }
    p.off_x = (p.S * (kChunkBytes + 16) + 127) & ~127;
    p.off_red = p.off_x + xreg_a;
    p.off_lys = p.off_red + 2 * kPCons * 64 * 4 + scal;
    p.total = p.off_red + tail;
    return p;
}

static bool tile_i4(const pox_tensor* t, size_t rows, size_t cols) {
    return t && t->dtype == POX_I4 && t->tiled && t->gs == 128 && !t->row_ptr && t->rows == rows && t->cols == cols;
}

bool persist_supported(const pox_model* m, int B) {
    if (!m->persist || !m->players || m->comm.tp != 1 || B < 1 || B > kPMaxB) return false;
    if (m->hd != 128 || m->G < 4 || m->G > 8) return false;
    for (int l = 0; l < m->L; l++) {
        const LayerW& w = m->layers[l];
        if (!m->pready[l] || !tile_i4(w.qkv, m->qkv_rows, m->H) || !tile_i4(w.o, m->H, (size_t)m->nq * 128) ||
            !tile_i4(w.gu, 2 * (size_t)m->I, m->H) || !tile_i4(w.down, m->H, m->I))
            return false;
    }
    return persist_plan(m, B).S > 0;
}

int persist_set_layer(pox_model* m, int l) {
    if (!m->players) return POX_OK;
    const LayerW& w = m->layers[l];
    PLayer h{};
    const pox_tensor* ts[4] = {w.qkv, w.o, w.gu, w.down};
    for (int i = 0; i < 4; i++) h.w[i] = ts[i] ? static_cast<const uint8_t*>(ts[i]->w) : nullptr;
    h.attn_norm = w.attn_norm;
    h.mlp_norm = w.mlp_norm;
    const cudaError_t e = cudaMemcpy(m->players + l, &h, sizeof(h), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_error(e, "cudaMemcpy(persistent layer table)");
    m->pready[l] = h.w[0] && h.w[1] && h.w[2] && h.w[3] && h.attn_norm && h.mlp_norm;
    return POX_OK;
}

int persist_launch(pox_model* m, int B, cudaStream_t st) {
    const PPlan pl = persist_plan(m, B);
    {
        static std::mutex mu;
        static unsigned done = 0;  // devices (ids < 32) whose attribute is set to the largest plan
        std::lock_guard<std::mutex> lk(mu);
        const int dev = m->ctx->device;
        if (dev >= 32 || !(done & (1u << dev))) {
            const cudaError_t e =
                cudaFuncSetAttribute(decode_persist_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
            if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(decode_persist_kernel)");
            if (dev < 32) done |= 1u << dev;
        }
    }
    PArgs a{};
    a.layers = m->players;
    a.L = m->L;
    const int rows[4] = {m->qkv_rows, m->H, 2 * m->I, m->H};
    const int cols[4] = {m->H, m->nq * 128, m->H, m->I};
    for (int i = 0; i < 4; i++) {
        a.nT[i] = (rows[i] + 15) / 16;
        a.nkb[i] = cols[i] / 128;
    }
    a.x = m->x;
    a.qkv = m->qkv;
    a.att = m->att;
    a.gu = m->gu;
    a.apart = m->apart;
    a.pos = m->pos;
    a.btab = m->btab;
    a.kc = m->kc;
    a.vc = m->vc;
    a.rope = m->rope;
    a.tickets = m->ptickets;
    a.ssq = m->pssq;
    a.bar = m->pbar;
    a.err = m->ctx->err_dev;
    a.B = B;
    a.H = m->H;
    a.I = m->I;
    a.nq = m->nq;
    a.nkv = m->nkv;
    a.G = m->G;
    a.qkv_rows = m->qkv_rows;
    a.mbps = (int)m->max_blocks_per_seq;
    a.kv_blocks = (int)m->kv_blocks;
    a.max_splits = m->max_splits;
    a.eps = m->cfg.rms_eps;
    a.S = pl.S;
    a.off_x = pl.off_x;
    a.off_xm = pl.off_xm;
    a.off_red = pl.off_red;
    a.off_lys = pl.off_lys;
    a.cs = pl.cs;
    a.nxbs = pl.nxbs;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)m->ctx->num_sms, 1, 1);
    cfg.blockDim = dim3(kPThreads, 1, 1);
    cfg.dynamicSmemBytes = (size_t)pl.total;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident at once: the grid barriers wait on each other
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, decode_persist_kernel, a);
    return e == cudaSuccess ? POX_OK : cuda_error(e, "persistent decode launch");
}

}  // namespace pox
