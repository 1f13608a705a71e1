// attn.cuh -- device code of the paged GQA decode attention shared by the per-layer kernels of
// engine.cu and the persistent decode kernel of persist.cu: RoPE from the model's (cos, sin)
// table, the KV append, and the tensor-core attention of one (sequence, kv head, 64-token split)
// item, run by 128 threads that synchronise on one named barrier.
//
// Reference: the attention of PoxEngine::forward_token (crates/paraoxidizer-runtime/src/engine.rs:
// 580-641) over fp16 pages of 16 tokens addressed through a block table
// (crates/paraoxidizer-runtime/src/paged_cache.rs:149-162).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "gemv.cuh"
#include "model.h"
#include "tc05.cuh"

namespace pox {

__device__ __forceinline__ float2 rope_pair(float a0, float a1, float c, float s) {
    return make_float2(__fsub_rn(__fmul_rn(a0, c), __fmul_rn(a1, s)), __fadd_rn(__fmul_rn(a0, s), __fmul_rn(a1, c)));
}

// What the attention kernels do besides attending: the decode step ropes q and appends the row's own
// k and v; prefill ropes q over pages a separate kernel already filled for every row of the pass;
// the kernel-level entry point takes q as given over filled pages.
enum { kAttnDecode = 0, kAttnPrefill = 1, kAttnPlain = 2 };

// bar.sync on named barrier `id` for `n` threads (n = the whole block for id 0 in a block of n).
__device__ __forceinline__ void named_sync(int id, int n) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// q of the item's G query heads into shared memory (qs [8][HD]), rotated by RoPE (engine.rs:353-408)
// from the model's (cos, sin) table unless MODE is kAttnPlain; in kAttnDecode the item whose split
// holds position p also rotates k and appends k and v to the page btab_row[p / 16], slot p % 16 (an
// entry outside [0, kv_blocks) is reported and nothing is written). Threads tid = 0 .. nthr - 1.
// q, k and v are read from L2 (ld.global.cg): in the persistent kernel another CTA wrote them.
template <int HD, int MODE>
__device__ __forceinline__ void load_q_append_kv(const float* row, uint32_t p, const int32_t* btab_row, int kv_blocks,
                                                 __half* kc, __half* vc, int layer, int L, int nq, int nkv, int h,
                                                 int G, const float2* rope, int t0, float* qs, int* err, int tid,
                                                 int nthr) {
    constexpr int DH = HD / 2;
    const float2* rp = MODE != kAttnPlain ? rope + (size_t)p * DH : nullptr;  // (cos, sin) at position p
    for (int j = tid; j < G * DH; j += nthr) {
        const int g = j / DH, i = j % DH;
        const float* q = row + (size_t)(h * G + g) * HD;
        float2 r = make_float2(__ldcg(q + 2 * i), __ldcg(q + 2 * i + 1));
        if (MODE != kAttnPlain) {
            const float2 cs = rp[i];
            r = rope_pair(r.x, r.y, cs.x, cs.y);
        }
        qs[g * HD + 2 * i] = r.x;
        qs[g * HD + 2 * i + 1] = r.y;
    }
    if (MODE == kAttnDecode && (int)p < t0 + kSplitTok) {  // this split holds the new position: append k, v
        const int blk = btab_row[p / kPage];
        if (blk < 0 || blk >= kv_blocks) {
            if (h == 0 && tid == 0) atomicOr(err, kErrAttnPage);
            return;
        }
        const size_t off = ((((size_t)blk * L + layer) * nkv + h) * kPage + p % kPage) * HD;
        const float* k = row + (size_t)(nq + h) * HD;
        const float* v = row + (size_t)(nq + nkv + h) * HD;
        for (int i = tid; i < DH; i += nthr) {
            const float2 cs = rp[i];
            const float2 r = rope_pair(__ldcg(k + 2 * i), __ldcg(k + 2 * i + 1), cs.x, cs.y);
            *reinterpret_cast<__half2*>(kc + off + 2 * i) = __floats2half2_rn(r.x, r.y);
            *reinterpret_cast<__half2*>(vc + off + 2 * i) = __floats2half2_rn(__ldcg(v + 2 * i), __ldcg(v + 2 * i + 1));
        }
    }
}

__device__ __forceinline__ void ldsm_x4(uint32_t a, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(a));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t a, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(a));
}
// (hi, lo) f16 pairs of (x0, x1): hi = f16(x), lo = f16(x - hi)
__device__ __forceinline__ void split_f16x2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(x0, x1);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(x0 - hf.x, x1 - hf.y);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
}

// Where the attention's combined output also goes as the o projection's prepared input (one 128-k
// block per query head of 128): the GEMV path's limbs and meta (cols / meta, strides Kp / nxbs), the
// integer small-M path's swizzled limbs and meta (xl / xm, padded batch Bp), or the f16 small-M
// path's swizzled halves (xs, row scale 1 in xscale). All NULL: att only.
struct OPrep {
    uint8_t* cols = nullptr;
    float2* meta = nullptr;
    int Kp = 0, nxbs = 0;
    uint8_t* xs = nullptr;
    float* xscale = nullptr;
    uint8_t* xl = nullptr;
    float2* xm = nullptr;
    int Bp = 0;
};

// The split combine fused into the attention kernel: the item that finishes a (sequence, kv head)
// last (a ticket per pair, zero between launches) combines its splits.
struct AttnFuse {
    uint32_t* tickets = nullptr;  // [B][nkv]; NULL: the combine is a kernel of its own
    float* att = nullptr;         // [B][nq * 128]
    OPrep op;
};

// att of the G query heads of kv head h, sequence b, from its ns split partials (base: [splits][G][130]
// floats of (max, sum, acc[128])): att = sum_s e^(m_s - M) acc_s / sum_s e^(m_s - M) l_s, 0 when the
// sum is <= 1e-9 (engine.rs:620-641). 128 threads: warp w takes heads w and w + 4, lane l dims
// 4 l .. 4 l + 3; the (max, sum) pairs and accumulators of 16 splits are loaded in one round (read
// from L2: other CTAs wrote them) with M and the sum carried exactly across rounds. Also writes the
// o projection's prepared input of those heads (op), xprep_int_kernel's arithmetic per 128-block.
__device__ __forceinline__ void attn_combine_heads(const float* base, int ns, int G, int b, int h, float* att_b,
                                                   const OPrep& op, int tid) {
    const int w = tid >> 5, lane = tid & 31;
    const size_t sstride = (size_t)G * 130;
    for (int gq = w; gq < G; gq += 4) {
        const float* hb = base + (size_t)gq * 130;
        float4 num = make_float4(0.f, 0.f, 0.f, 0.f);
        float M = -INFINITY, den = 0.f;
        for (int s0 = 0; s0 < ns; s0 += 16) {
            const int n = min(16, ns - s0);
            const float2 ml = lane < n ? __ldcg(reinterpret_cast<const float2*>(hb + (s0 + lane) * sstride))
                                       : make_float2(-INFINITY, 0.f);
            float2 v[16][2];
#pragma unroll
            for (int j = 0; j < 16; j++) {
                const float* pp = hb + (s0 + min(j, n - 1)) * sstride;
                v[j][0] = __ldcg(reinterpret_cast<const float2*>(pp + 2 + 4 * lane));
                v[j][1] = __ldcg(reinterpret_cast<const float2*>(pp + 4 + 4 * lane));
            }
            const float Mc = fmaxf(M, warp_max(ml.x));
            const float sc = M == -INFINITY ? 0.f : expf(M - Mc);
            const float wl = lane < n ? expf(ml.x - Mc) : 0.f;
            den = fmaf(den, sc, warp_sum(wl * ml.y));
            num.x *= sc, num.y *= sc, num.z *= sc, num.w *= sc;
#pragma unroll
            for (int j = 0; j < 16; j++) {
                const float wt = __shfl_sync(0xffffffffu, wl, j);  // 0 past the round's splits
                num.x = fmaf(wt, v[j][0].x, num.x);
                num.y = fmaf(wt, v[j][0].y, num.y);
                num.z = fmaf(wt, v[j][1].x, num.z);
                num.w = fmaf(wt, v[j][1].y, num.w);
            }
            M = Mc;
        }
        const float inv = den > 1e-9f ? 1.0f / den : 0.f;
        const float4 o = make_float4(num.x * inv, num.y * inv, num.z * inv, num.w * inv);
        const int blk = h * G + gq, e = blk * 128 + 4 * lane;
        *reinterpret_cast<float4*>(att_b + e) = o;
        if (op.cols || op.xl) {
            const float m = warp_max(fmaxf(fmaxf(fabsf(o.x), fabsf(o.y)), fmaxf(fabsf(o.z), fabsf(o.w))));
            const float sm = warp_sum((o.x + o.y) + (o.z + o.w));
            const float qi = m > 0.f ? (float)kXLimbMax / m : 0.f;
            const int X[4] = {__float2int_rn(o.x * qi), __float2int_rn(o.y * qi), __float2int_rn(o.z * qi),
                              __float2int_rn(o.w * qi)};
            uint32_t hi = 0, lo = 0;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int q = max(-kXLimbMax, min(kXLimbMax, X[i]));
                hi |= ((uint32_t)(q >> 7) & 0xFFu) << (8 * i);
                lo |= ((uint32_t)q & 0x7Fu) << (8 * i);
            }
            const float2 mt = make_float2(m > 0.f ? m / (float)kXLimbMax : 0.f, sm);
            if (op.cols) {
                *reinterpret_cast<uint32_t*>(op.cols + (size_t)(2 * b) * op.Kp + e) = hi;
                *reinterpret_cast<uint32_t*>(op.cols + (size_t)(2 * b + 1) * op.Kp + e) = lo;
                if (lane == 0) op.meta[(size_t)b * op.nxbs + blk] = mt;
            } else {
                uint8_t* tile = op.xl + (size_t)blk * (2 * op.Bp) * 128;
                *reinterpret_cast<uint32_t*>(tile + sw128_off(2 * b, lane >> 2) + ((4 * lane) & 15)) = hi;
                *reinterpret_cast<uint32_t*>(tile + sw128_off(2 * b + 1, lane >> 2) + ((4 * lane) & 15)) = lo;
                if (lane == 0) op.xm[(size_t)blk * op.Bp + b] = mt;
            }
        } else if (op.xs) {
            const int kk = 4 * lane;
            const size_t off = ((size_t)blk * 2 + (kk >> 6)) * (size_t)op.Bp * 128 + sw128_off(b, (kk & 63) >> 3) +
                               2 * (kk & 7);
            const __half2 h01 = __floats2half2_rn(o.x, o.y), h23 = __floats2half2_rn(o.z, o.w);
            uint2 hv;
            hv.x = *reinterpret_cast<const uint32_t*>(&h01);
            hv.y = *reinterpret_cast<const uint32_t*>(&h23);
            *reinterpret_cast<uint2*>(op.xs + off) = hv;
            if (blk == 0 && lane == 0) op.xscale[b] = 1.0f;
        }
    }
}

// Shared memory of one tensor-core attention item (head_dim 128, 128 threads).
constexpr int kAttnRS = 128 + 8;  // staged row stride in halves (272 B: ldmatrix rows in distinct banks)
struct __align__(16) AttnTcSmem {
    float qs[8][128];
    float red_m[4][8], red_l[4][8];
    __half kv_s[2][4][16][kAttnRS];  // [K, V][warp][token][dim]; then the warps' outputs (f32 [4][8][128])
};

// One attention item on the tensor cores: tokens [64 split, min(p + 1, 64 split + 64)) of one
// sequence (row = its qkv row, p its position, btab_row its block table) for the G (4..8) query
// heads of kv head h, head_dim 128. The caller has checked p against the block table and that the
// split holds at least one token. Each of the 4 warps stages its 16-token page of K and V in shared
// memory and runs S = Q K^T and O = P V on mma.sync m16n8k16 with f32 accumulation, the G query
// heads being the rows of A (padded to 16) and q and p split into f16 hi + lo terms (about 22
// significant bits for values >= 2^-4, an absolute error under 2^-24 below); K fragments come from
// ldmatrix, V fragments from ldmatrix.trans; rows of a page past the context are zero. Writes
// (max, sum, acc[128]) per query head to out[G][130] for the combine. Threads tid = 0..127 of the
// item synchronise on named barrier `bar` (0 when the item is the whole block).
template <int MODE>
__device__ __forceinline__ void attn_tc_item(const float* row, uint32_t p, const int32_t* btab_row, int kv_blocks,
                                             __half* kc, __half* vc, int layer, int L, int nq, int nkv, int h, int G,
                                             const float2* rope, int split, float* out, int* err, AttnTcSmem& sm,
                                             int tid, int bar) {
    constexpr int HD = 128, RS = kAttnRS;
    const int ctx = (int)p + 1;
    const int t0 = split * kSplitTok;
    const int nt = min(ctx - t0, kSplitTok);
    const int warp = tid >> 5, lane = tid & 31;
    float (*acc_s)[8][HD] = reinterpret_cast<float (*)[8][HD]>(&sm.kv_s[0][0][0][0]);
    // this warp's page (tokens t0 + 16 warp ..): unless the page takes this step's append, its K and V
    // rows are copied before q is loaded, so the two round trips overlap
    int nw = max(0, min(16, nt - 16 * warp));
    size_t page = 0;
    if (nw > 0) {
        const int blk = btab_row[(t0 + 16 * warp) / kPage];
        if (blk < 0 || blk >= kv_blocks) {  // invalid page: reported, its tokens left out (rows zero)
            if (lane == 0) atomicOr(err, kErrAttnPage);
            nw = 0;
        } else {
            page = (((size_t)blk * L + layer) * nkv + h) * kPage * HD;
        }
    }
    const bool appends = MODE == kAttnDecode && nw > 0 && (int)p / kPage == (t0 + 16 * warp) / kPage;
    // staged by asynchronous copies (no registers held), rows past the context zero
    auto stage_page = [&]() {
#pragma unroll
        for (int u = 0; u < 16 * (HD / 8) / 32; u++) {
            const int idx = lane + 32 * u, r = idx / (HD / 8), c = idx % (HD / 8);
            const uint32_t dk = smem_u32(&sm.kv_s[0][warp][r][8 * c]), dv = smem_u32(&sm.kv_s[1][warp][r][8 * c]);
            if (r < nw) {
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dk),
                             "l"(reinterpret_cast<const uint4*>(kc + page + (size_t)r * HD) + c) : "memory");
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dv),
                             "l"(reinterpret_cast<const uint4*>(vc + page + (size_t)r * HD) + c) : "memory");
            } else {
                *reinterpret_cast<uint4*>(&sm.kv_s[0][warp][r][8 * c]) = make_uint4(0u, 0u, 0u, 0u);
                *reinterpret_cast<uint4*>(&sm.kv_s[1][warp][r][8 * c]) = make_uint4(0u, 0u, 0u, 0u);
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    if (!appends) stage_page();
    load_q_append_kv<HD, MODE>(row, p, btab_row, kv_blocks, kc, vc, layer, L, nq, nkv, h, G, rope, t0,
                                &sm.qs[0][0], err, tid, 128);
    named_sync(bar, 128);
    if (appends) stage_page();  // after the append into this page
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncwarp();

    const int g = lane >> 2, t = lane & 3, mi = lane >> 3, mr = lane & 7;
    // S = Q K^T: A rows = query heads (g < G; rows g + 8 are padding), B = the staged K rows
    float sacc[2][4];
#pragma unroll
    for (int nb = 0; nb < 2; nb++) sacc[nb][0] = sacc[nb][1] = sacc[nb][2] = sacc[nb][3] = 0.f;
    const uint32_t kbase = smem_u32(&sm.kv_s[0][warp][0][0]), vbase = smem_u32(&sm.kv_s[1][warp][0][0]);
#pragma unroll
    for (int ks = 0; ks < HD / 16; ks++) {
        uint32_t qh0, ql0, qh1, ql1;
        const int c0 = 16 * ks + 2 * t;
        split_f16x2(g < G ? sm.qs[g][c0] : 0.f, g < G ? sm.qs[g][c0 + 1] : 0.f, qh0, ql0);
        split_f16x2(g < G ? sm.qs[g][c0 + 8] : 0.f, g < G ? sm.qs[g][c0 + 9] : 0.f, qh1, ql1);
        uint32_t b00, b01, b10, b11;  // tokens 0-7: (b00, b01), tokens 8-15: (b10, b11)
        ldsm_x4(kbase + (uint32_t)(((8 * (mi >> 1) + mr) * RS + 16 * ks + 8 * (mi & 1)) * 2), b00, b01, b10, b11);
        mma_16816(sacc[0], qh0, 0u, qh1, 0u, b00, b01);
        mma_16816(sacc[0], ql0, 0u, ql1, 0u, b00, b01);
        mma_16816(sacc[1], qh0, 0u, qh1, 0u, b10, b11);
        mma_16816(sacc[1], ql0, 0u, ql1, 0u, b10, b11);
    }
    // scores of head g: tokens 8 nb + 2 t + e of this page
    const float scale = 1.0f / sqrtf(fmaxf((float)HD, 1.0f));
    float sc[2][2];
    float m = -INFINITY;
#pragma unroll
    for (int nb = 0; nb < 2; nb++)
#pragma unroll
        for (int e = 0; e < 2; e++) {
            const int jj = 8 * nb + 2 * t + e;
            sc[nb][e] = (g < G && jj < nw) ? sacc[nb][e] * scale : -INFINITY;
            m = fmaxf(m, sc[nb][e]);
        }
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
    if (t == 0 && g < G) sm.red_m[warp][g] = m;
    named_sync(bar, 128);
    float mx = g < G ? fmaxf(fmaxf(sm.red_m[0][g], sm.red_m[1][g]), fmaxf(sm.red_m[2][g], sm.red_m[3][g])) : 0.f;
    if (!isfinite(mx)) mx = 0.f;
    float pv[2][2], l = 0.f;
#pragma unroll
    for (int nb = 0; nb < 2; nb++)
#pragma unroll
        for (int e = 0; e < 2; e++) {
            float v = 0.f;
            if (g < G && 8 * nb + 2 * t + e < nw) {
                v = expf(sc[nb][e] - mx);
                if (!isfinite(v)) v = 0.f;
            }
            pv[nb][e] = v;
            l += v;
        }
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    if (t == 0 && g < G) sm.red_l[warp][g] = l;
    // O = P V: A = P (tokens 2t, 2t+1 | 2t+8, 2t+9 of head g), B = V rows through ldmatrix.trans
    uint32_t ph0, pl0, ph1, pl1;
    split_f16x2(pv[0][0], pv[0][1], ph0, pl0);
    split_f16x2(pv[1][0], pv[1][1], ph1, pl1);
    float oacc[HD / 8][4];
#pragma unroll
    for (int nd = 0; nd < HD / 8; nd++) oacc[nd][0] = oacc[nd][1] = oacc[nd][2] = oacc[nd][3] = 0.f;
#pragma unroll
    for (int j = 0; j < HD / 16; j++) {
        uint32_t v00, v01, v10, v11;  // dims 16 j ..: (v00, v01), dims 16 j + 8 ..: (v10, v11)
        ldsm_x4_t(vbase + (uint32_t)(((8 * (mi & 1) + mr) * RS + 16 * j + 8 * (mi >> 1)) * 2), v00, v01, v10, v11);
        mma_16816(oacc[2 * j], ph0, 0u, ph1, 0u, v00, v01);
        mma_16816(oacc[2 * j], pl0, 0u, pl1, 0u, v00, v01);
        mma_16816(oacc[2 * j + 1], ph0, 0u, ph1, 0u, v10, v11);
        mma_16816(oacc[2 * j + 1], pl0, 0u, pl1, 0u, v10, v11);
    }
    named_sync(bar, 128);  // every warp is done with the staged pages (acc_s reuses them); red_l complete
    if (g < G)
#pragma unroll
        for (int nd = 0; nd < HD / 8; nd++) {
            acc_s[warp][g][8 * nd + 2 * t] = oacc[nd][0];
            acc_s[warp][g][8 * nd + 2 * t + 1] = oacc[nd][1];
        }
    named_sync(bar, 128);
    for (int i = tid; i < G * HD; i += 128) {
        const int gg = i / HD, d = i % HD;
        out[(size_t)gg * (HD + 2) + 2 + d] = (acc_s[0][gg][d] + acc_s[1][gg][d]) + (acc_s[2][gg][d] + acc_s[3][gg][d]);
    }
    if (tid < G) {
        float mt = fmaxf(fmaxf(sm.red_m[0][tid], sm.red_m[1][tid]), fmaxf(sm.red_m[2][tid], sm.red_m[3][tid]));
        if (!isfinite(mt)) mt = 0.f;
        out[(size_t)tid * (HD + 2)] = mt;
        out[(size_t)tid * (HD + 2) + 1] = (sm.red_l[0][tid] + sm.red_l[1][tid]) + (sm.red_l[2][tid] + sm.red_l[3][tid]);
    }
}

}  // namespace pox
