// engine.cu -- one decode step of a Llama-architecture model on B200 (sm_100a): the CUDA
// counterpart of PoxEngine::forward_token (crates/paraoxidizer-runtime/src/engine.rs:411-716) for a
// batch of sequences, with the KV cache in fp16 pages of 16 tokens addressed through per-sequence
// block tables (the block-table semantics of crates/paraoxidizer-runtime/src/paged_cache.rs:149-162).
//
// Per layer: 4 GEMV launches on resident re-tiled weights (QKV and gate/up are concatenated at
// load, so every projection row is computed exactly as in the separate tensors):
//   qkv  = W_qkv  rmsnorm(x, attn_norm)            (norm fused into the GEMV's x preparation)
//   att  = paged GQA attention over 0..=pos          (attn_decode_tc_kernel on the tensor cores for
//          head_dim 128 with 4-8 query heads per kv head, attn_decode_kernel otherwise: RoPE on q
//          and k from the model's (cos, sin) table, k and v appended to the KV pages,
//          split-context partials; attn_combine_kernel: the splits combined and written as the o
//          projection's prepared input)
//   x   += W_o att                                   (residual fused into the GEMV epilogue)
//   gu   = W_gu   rmsnorm(x, mlp_norm)
//   x   += W_down silu(g) * u                        (SwiGLU fused into the x preparation)
// then logits = W_head rmsnorm(x, final_norm) (F16 GEMV), non-finite logits -> 0, greedy argmax.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <vector>

#include "../../include/pox_cuda.h"
#include "api_internal.h"
#include "common.cuh"
#include "gemv.cuh"
#include "attn.cuh"
#include "model.h"
#include "persist.h"
#include "tc05.cuh"

#ifdef POX_HAVE_NCCL
#include <nccl.h>
#endif

namespace pox {

// ---- embedding (engine.rs:420-524): f16 row of token % vocab; a row with no |x| > 1e-6 becomes
// sin(tok * 0.17) * 0.1 everywhere ----
__global__ void embed_kernel(const uint32_t* __restrict__ tokens, const uint16_t* __restrict__ embed, int V, int H,
                             float* __restrict__ x) {
    pdl_launch_dependents();
    pdl_wait();
    const int b = blockIdx.x;
    const uint32_t tok = tokens[b] % (uint32_t)V;
    const uint16_t* row = embed + (size_t)tok * H;
    float* xr = x + (size_t)b * H;
    int sig = 0;
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
        const float v = half_bits_to_float(row[i]);
        xr[i] = v;
        sig |= fabsf(v) > 1e-6f;
    }
    if (!__syncthreads_or(sig)) {
        const float val = __fmul_rn(sinf(__fmul_rn((float)tok, 0.17f)), 0.1f);
        for (int i = threadIdx.x; i < H; i += blockDim.x) xr[i] = val;
    }
}

// ---- RoPE (engine.rs:353-408, interleaved pairs): cos / sin of pair i at position p ----
__device__ __forceinline__ void rope_cs(uint32_t p, int i, int hd, float theta, float& c, float& s) {
    const float th = fmaxf(theta, 1.0f);
    const float exponent = __fdiv_rn((float)(2 * i), (float)hd);
    const float freq = __fdiv_rn(1.0f, powf(th, exponent));
    const float angle = __fmul_rn((float)p, freq);
    c = 1.0f;
    s = 0.0f;
    if (isfinite(angle)) {
        c = cosf(angle);
        s = sinf(angle);
    }
}
// The (cos, sin) table of every position a sequence of the model can reach, computed once with
// rope_cs, so attention looks the values up instead of evaluating powf / cosf / sinf in each of
// its context splits (identical bits either way).
__global__ void rope_table_kernel(float2* __restrict__ t, int npos, int hd, float theta) {
    const int half = hd / 2;
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (long long)npos * half) return;
    float c, s;
    rope_cs((uint32_t)(idx / half), (int)(idx % half), hd, theta, c, s);
    t[idx] = make_float2(c, s);
}
// ---- paged GQA decode attention (engine.rs:580-641), split over the context, RoPE and the KV
// append fused in ----
// CTA (split, kv head, batch row) takes tokens [64 split, min(ctx, 64 split + 64)) for the G query
// heads of its kv head. q is roped into shared memory; the CTA whose split holds the new position
// ropes k and writes k and v into the page (block_table[pos / 16], slot pos % 16) first. Warp w
// takes the 16 tokens of one page: two lanes per token read its K row (one half each) and the
// warp reads the 16 V rows, all issued before any use; scores, the split's softmax partial and
// sum_t p_t v_t follow. Writes (max, sum, acc[hd]) per query head for the combine kernel.
template <int HD, int MODE>
__global__ void __launch_bounds__(128) attn_decode_kernel(const float* __restrict__ qkv, int qkv_rows,
                                                          const uint32_t* __restrict__ pos,
                                                          const int32_t* __restrict__ btab, int mbps, int kv_blocks,
                                                          __half* __restrict__ kc, __half* __restrict__ vc, int layer,
                                                          int L, int nq, int nkv, int G, int max_splits,
                                                          const float2* __restrict__ rope, float* __restrict__ apart,
                                                          int* __restrict__ err) {
    constexpr int DH = HD / 2;   // K dims per lane (two lanes per token)
    constexpr int DPL = HD / 32; // V dims per lane
    pdl_launch_dependents();
    pdl_wait();
    const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const uint32_t p = pos[b];
    if (p >= (uint32_t)mbps * kPage) {  // beyond the block table (invalid input): reported, nothing read
        if (split == 0 && h == 0 && threadIdx.x == 0) atomicOr(err, kErrAttnPos);
        return;
    }
    const int ctx = (int)p + 1;
    const int t0 = split * kSplitTok;
    if (t0 >= ctx) return;  // the combine kernel reads only ceil(ctx / 64) splits
    const int nt = min(ctx - t0, kSplitTok);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    __shared__ float qs[8][HD];
    __shared__ float ps[8][kSplitTok];
    __shared__ float red_m[4][8], red_l[4][8];
    __shared__ float acc_s[4][8][HD];
    const float* row = qkv + (size_t)b * qkv_rows;
    load_q_append_kv<HD, MODE>(row, p, btab + (size_t)b * mbps, kv_blocks, kc, vc, layer, L, nq, nkv, h, G,
                                rope, t0, &qs[0][0], err, (int)threadIdx.x, (int)blockDim.x);
    __syncthreads();

    // this warp's page: tokens t0 + 16 warp .. + 15 (t0 is a multiple of 64, pages hold 16)
    const int jt = 16 * warp + (lane & 15), hh = lane >> 4;
    int nw = max(0, min(16, nt - 16 * warp));  // valid tokens of this warp
    uint4 kr[DH / 8];
    uint2 vr[16];
    const int blk = nw > 0 ? btab[(size_t)b * mbps + (t0 + 16 * warp) / kPage] : 0;
    if (nw > 0 && (blk < 0 || blk >= kv_blocks)) {  // invalid page: reported, its tokens left out
        if (lane == 0) atomicOr(err, kErrAttnPage);
        nw = 0;
    }
    if (nw > 0) {
        const size_t page = (((size_t)blk * L + layer) * nkv + h) * kPage * HD;
        if ((lane & 15) < nw) {
            const __half* kp = kc + page + (size_t)(lane & 15) * HD + hh * DH;
#pragma unroll
            for (int i = 0; i < DH / 8; i++) kr[i] = __ldcg(reinterpret_cast<const uint4*>(kp) + i);
        }
#pragma unroll
        for (int u = 0; u < 16; u++) {
            vr[u] = make_uint2(0u, 0u);
            if (u < nw) {
                const __half* vp = vc + page + (size_t)u * HD + DPL * lane;
                if constexpr (DPL == 4) vr[u] = __ldcg(reinterpret_cast<const uint2*>(vp));
                else if constexpr (DPL == 2) vr[u].x = __ldcg(reinterpret_cast<const unsigned int*>(vp));
                else vr[u].x = __ldcg(reinterpret_cast<const unsigned short*>(vp));
            }
        }
    }
    const float scale = 1.0f / sqrtf(fmaxf((float)HD, 1.0f));
    float sc[8];
#pragma unroll
    for (int g = 0; g < 8; g++) {
        float dot = 0.f;
        if (g < G && (lane & 15) < nw) {
#pragma unroll
            for (int i = 0; i < DH / 8; i++) {
                const __half2* hp = reinterpret_cast<const __half2*>(&kr[i]);
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const float2 f = __half22float2(hp[j]);
                    dot = fmaf(qs[g][hh * DH + 8 * i + 2 * j], f.x, dot);
                    dot = fmaf(qs[g][hh * DH + 8 * i + 2 * j + 1], f.y, dot);
                }
            }
        }
        dot += __shfl_xor_sync(0xffffffffu, dot, 16);
        sc[g] = (g < G && (lane & 15) < nw) ? dot * scale : -INFINITY;
        float m = sc[g];
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) red_m[warp][g] = m;
    }
    __syncthreads();
    float mx[8];
#pragma unroll
    for (int g = 0; g < 8; g++) {
        mx[g] = fmaxf(fmaxf(red_m[0][g], red_m[1][g]), fmaxf(red_m[2][g], red_m[3][g]));
        if (!isfinite(mx[g])) mx[g] = 0.f;
        float pv = 0.f;
        if (g < G && (lane & 15) < nw) {
            pv = expf(sc[g] - mx[g]);
            if (!isfinite(pv)) pv = 0.f;
            if (hh == 0) ps[g][jt] = pv;
        }
        float l = hh == 0 ? pv : 0.f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
        if (lane == 0) red_l[warp][g] = l;
    }
    __syncthreads();
    // sum_t p_t v_t over this warp's tokens; lane holds dims DPL lane .. + DPL
    float acc[8][DPL];
#pragma unroll
    for (int g = 0; g < 8; g++)
#pragma unroll
        for (int q = 0; q < DPL; q++) acc[g][q] = 0.f;
#pragma unroll
    for (int u = 0; u < 16; u++) {
        if (u < nw) {
            float vf[DPL];
            if constexpr (DPL == 4) {
                const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&vr[u].x));
                const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&vr[u].y));
                vf[0] = f0.x;
                vf[1] = f0.y;
                vf[2] = f1.x;
                vf[3] = f1.y;
            } else if constexpr (DPL == 2) {
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&vr[u].x));
                vf[0] = f.x;
                vf[1] = f.y;
            } else {
                vf[0] = __half2float(__ushort_as_half((unsigned short)vr[u].x));
            }
#pragma unroll
            for (int g = 0; g < 8; g++) {
                if (g < G) {
                    const float pw = ps[g][16 * warp + u];
#pragma unroll
                    for (int q = 0; q < DPL; q++) acc[g][q] = fmaf(pw, vf[q], acc[g][q]);
                }
            }
        }
    }
#pragma unroll
    for (int g = 0; g < 8; g++)
        if (g < G)
#pragma unroll
            for (int q = 0; q < DPL; q++) acc_s[warp][g][DPL * lane + q] = acc[g][q];
    __syncthreads();
    float* out = apart + ((((size_t)b * nkv + h) * max_splits + split) * G) * (HD + 2);
    for (int i = tid; i < G * HD; i += 128) {
        const int g = i / HD, d = i % HD;
        out[(size_t)g * (HD + 2) + 2 + d] = (acc_s[0][g][d] + acc_s[1][g][d]) + (acc_s[2][g][d] + acc_s[3][g][d]);
    }
    if (tid < G) {
        out[(size_t)tid * (HD + 2)] = mx[tid];
        out[(size_t)tid * (HD + 2) + 1] = (red_l[0][tid] + red_l[1][tid]) + (red_l[2][tid] + red_l[3][tid]);
    }
}

// Tensor-core variant of attn_decode_kernel for head_dim 128 and 4..8 query heads per kv head
// (the Llama-3 8B / 70B layouts); same grid, splits, RoPE, KV append and partial output. Each warp
// stages its page of K and V (16 tokens) in shared memory and runs both products on mma.sync
// m16n8k16 with f32 accumulation: S = Q K^T with the G query heads as the rows of A (padded to
// 16) and q split into two f16 terms (hi = f16(q), lo = f16(q - hi): about 22 significant bits for
// |q| >= 2^-4, an absolute error under 2^-24 below), then
// O = P V with P likewise split. Fragments come from ldmatrix (V transposed); rows of a page past
// the context are zero.
// With fz.tickets the split combine runs here: the CTA that finishes a (sequence, kv head) last
// combines its splits into att and o_proj's prepared input (attn_combine_heads), so the combine
// needs no launch of its own.
template <int HD, int MODE>
__global__ void __launch_bounds__(128) attn_decode_tc_kernel(const float* __restrict__ qkv, int qkv_rows,
                                                             const uint32_t* __restrict__ pos,
                                                             const int32_t* __restrict__ btab, int mbps,
                                                             int kv_blocks, __half* __restrict__ kc,
                                                             __half* __restrict__ vc, int layer, int L, int nq,
                                                             int nkv, int G, int max_splits,
                                                             const float2* __restrict__ rope,
                                                             float* __restrict__ apart, int* __restrict__ err,
                                                             AttnFuse fz) {
    static_assert(HD == 128, "head_dim 128");
    pdl_launch_dependents();
    pdl_wait();
    const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const uint32_t p = pos[b];
    const float* base = apart + (((size_t)b * nkv + h) * max_splits) * G * (HD + 2);
    if (p >= (uint32_t)mbps * kPage) {  // beyond the block table (invalid input): reported, nothing read
        if (split == 0 && h == 0 && threadIdx.x == 0) atomicOr(err, kErrAttnPos);
        if (fz.tickets && split == 0)  // output 0, as the combine kernel writes for no splits
            attn_combine_heads(base, 0, G, b, h, fz.att + (size_t)b * nq * HD, fz.op, (int)threadIdx.x);
        return;
    }
    const int ns = min(max_splits, (int)((p + kSplitTok) / kSplitTok));
    if (split >= ns) return;  // the combine reads only ceil(ctx / 64) splits
    __shared__ AttnTcSmem sm;
    __shared__ int s_last;
    float* out = apart + ((((size_t)b * nkv + h) * max_splits + split) * G) * (HD + 2);
    attn_tc_item<MODE>(qkv + (size_t)b * qkv_rows, p, btab + (size_t)b * mbps, kv_blocks, kc, vc, layer, L, nq, nkv,
                       h, G, rope, split, out, err, sm, (int)threadIdx.x, 0);
    if (!fz.tickets) return;
    __syncthreads();  // this split's partial is written
    if (threadIdx.x == 0) {
        __threadfence();
        uint32_t* tk = fz.tickets + (size_t)b * nkv + h;
        const int last = atomicAdd(tk, 1u) == (uint32_t)(ns - 1);
        if (last) {
            atomicExch(tk, 0u);
            __threadfence();
        }
        s_last = last;
    }
    __syncthreads();
    if (s_last) attn_combine_heads(base, ns, G, b, h, fz.att + (size_t)b * nq * HD, fz.op, (int)threadIdx.x);
}

// Combines the splits of the attention output and prepares it as the o projection's input:
// att = sum_s e^(m_s - M) acc_s / sum_s e^(m_s - M) l_s (the reference's 1 / sum_exp, 0 when the
// sum is <= 1e-9). CTA (128-element block blk of the row, batch row b); thread d = element
// 128 blk + d. Writes att (f32) and, for the GEMV that follows:
//  * cols / meta (batch <= 8): the 15-bit two-limb fixed point of the block and (max/16383, sum),
//    as xprep_int_kernel computes them;
//  * xl / xm (integer small-M path): the same limbs as rows 2b / 2b + 1 of each block's
//    128-byte-swizzled [2 Bp][128 B] tile, and the block's (max/16383, sum) at [block][b];
//  * xs (f16 small-M path): f16(att) in the 128-byte-swizzled k-block-major layout, row scale 1
//    (|att| <= max|v| <= 65504, the f16 range, so no scaling is needed).
__global__ void __launch_bounds__(128) attn_combine_kernel(const uint32_t* __restrict__ pos, uint32_t max_pos, int nq,
                                                           int nkv, int G, int hd, int max_splits,
                                                           const float* __restrict__ apart, float* __restrict__ att,
                                                           OPrep op) {
    pdl_launch_dependents();
    pdl_wait();
    const int blk = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
    const int e = blk * 128 + d, hq = e / hd, dd = e % hd;
    if (e >= nq * hd) return;  // only when nq hd % 128 != 0, where nothing is prepared (no barrier below)
    // ceil((pos + 1) / 64) splits; none (output 0) for a position beyond the block table, which the
    // attention kernel reported and skipped
    const int ns = pos[b] >= max_pos ? 0 : min(max_splits, (int)((pos[b] + (uint32_t)kSplitTok) / kSplitTok));
    const int h = hq / G, g = hq % G;
    const float* base = apart + (((size_t)b * nkv + h) * max_splits * G + g) * (hd + 2);
    const size_t sstride = (size_t)G * (hd + 2);
    float M = -INFINITY;
    for (int s = 0; s < ns; s++) M = fmaxf(M, base[s * sstride]);
    float num = 0.f, den = 0.f;
    for (int s = 0; s < ns; s++) {
        const float* pp = base + s * sstride;
        const float w = expf(pp[0] - M);
        den = fmaf(w, pp[1], den);
        num = fmaf(w, pp[2 + dd], num);
    }
    const float inv = den > 1e-9f ? 1.0f / den : 0.f;
    const float v = num * inv;
    const int K = nq * hd;
    att[(size_t)b * K + e] = v;
    if (op.cols || op.xl) {
        __shared__ float red[4];
        const int warp = d >> 5, lane = d & 31;
        float m = warp_max(fabsf(v));
        if (lane == 0) red[warp] = m;
        __syncthreads();
        m = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
        __syncthreads();
        const float qi = m > 0.f ? (float)kXLimbMax / m : 0.f;
        const int X = max(-kXLimbMax, min(kXLimbMax, __float2int_rn(v * qi)));
        const uint8_t hi = (uint8_t)((uint32_t)(X >> 7) & 0xFFu), lo = (uint8_t)((uint32_t)X & 0x7Fu);
        if (op.cols) {
            op.cols[(size_t)(2 * b) * op.Kp + e] = hi;
            op.cols[(size_t)(2 * b + 1) * op.Kp + e] = lo;
        } else {
            uint8_t* tile = op.xl + (size_t)blk * (2 * op.Bp) * 128;  // blk = e / 128
            tile[sw128_off(2 * b, d >> 4) + (d & 15)] = hi;
            tile[sw128_off(2 * b + 1, d >> 4) + (d & 15)] = lo;
        }
        const float sw = warp_sum(v);
        if (lane == 0) red[warp] = sw;
        __syncthreads();
        const float2 mt = make_float2(m > 0.f ? m / (float)kXLimbMax : 0.f, (red[0] + red[1]) + (red[2] + red[3]));
        if (d == 0) {
            if (op.cols) op.meta[(size_t)b * op.nxbs + blk] = mt;
            else op.xm[(size_t)blk * op.Bp + b] = mt;
        }
    } else if (op.xs) {
        const int kb = e >> 7, kk = e & 127;
        const size_t off = ((size_t)kb * 2 + (kk >> 6)) * (size_t)op.Bp * 128 + sw128_off(b, (kk & 63) >> 3) + 2 * (kk & 7);
        *reinterpret_cast<__half*>(op.xs + off) = __float2half_rn(v);
        if (blk == 0 && d == 0) op.xscale[b] = 1.0f;
    }
}

// Non-finite logits -> 0 (engine.rs:709-713), then greedy argmax: the first index of the maximum
// (sampler.rs:55-65, strict >), in two passes. Pass 1: block (p, b) takes vocab entries
// [p chunk, (p + 1) chunk) of row b and writes its first maximum as (logit, index bits).
__device__ __forceinline__ void first_max(float& v, int& i, float ov, int oi) {
    if (ov > v || (ov == v && oi < i)) {
        v = ov;
        i = oi;
    }
}

__global__ void __launch_bounds__(256) argmax_part_kernel(float* __restrict__ logits, int V, int chunk,
                                                          float2* __restrict__ part) {
    pdl_launch_dependents();
    pdl_wait();
    const int p = blockIdx.x, b = blockIdx.y;
    float* lr = logits + (size_t)b * V;
    const int i1 = min(V, (p + 1) * chunk);
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = p * chunk + threadIdx.x; i < i1; i += blockDim.x) {
        float v = lr[i];
        if (!isfinite(v)) {
            v = 0.f;
            lr[i] = 0.f;
        }
        if (v > bv) {
            bv = v;
            bi = i;
        }
    }
    __shared__ float sv[8];
    __shared__ int si[8];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        first_max(bv, bi, __shfl_xor_sync(0xffffffffu, bv, o), __shfl_xor_sync(0xffffffffu, bi, o));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        sv[warp] = bv;
        si[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); w++) first_max(bv, bi, sv[w], si[w]);
        part[(size_t)b * kArgmaxParts + p] = make_float2(bv, __int_as_float(bi));
    }
}

// Pass 2: one warp per row over its parts. One rank: next[b]. Tensor parallel: the rank's pair
// (logit, token index in the whole vocabulary) for the pick across ranks.
__global__ void argmax_final_kernel(const float2* __restrict__ part, int parts, int B, int vocab_off,
                                    uint32_t* __restrict__ next, float2* __restrict__ pairs) {
    pdl_launch_dependents();
    pdl_wait();
    const int b = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (b >= B) return;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int p = lane; p < parts; p += 32) {
        const float2 q = part[(size_t)b * kArgmaxParts + p];
        first_max(bv, bi, q.x, __float_as_int(q.y));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        first_max(bv, bi, __shfl_xor_sync(0xffffffffu, bv, o), __shfl_xor_sync(0xffffffffu, bi, o));
    if (lane == 0) {
        if (pairs)
            pairs[b] = make_float2(bv, __int_as_float(bi == 0x7fffffff ? bi : bi + vocab_off));
        else
            next[b] = bi == 0x7fffffff ? 0u : (uint32_t)bi;
    }
}

// Feeds the greedy tokens back and advances the positions (a self-contained multi-step loop).
__global__ void advance_kernel(uint32_t* tok, uint32_t* pos, const uint32_t* next, int B) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b < B) {
        tok[b] = next[b];
        pos[b] += 1;
    }
}

// Launch of the split-context attention kernels (MODE: kAttnDecode, kAttnPrefill or kAttnPlain).
// Tensor cores for head_dim 128 with 4..8 query heads per kv head, the FMA kernel otherwise.
struct AttnLaunch {
    const float* qkv = nullptr;
    int qkv_rows = 0;
    const uint32_t* pos = nullptr;
    const int32_t* btab = nullptr;
    int mbps = 0, kv_blocks = 0;
    __half* kc = nullptr;
    __half* vc = nullptr;
    int layer = 0, L = 1, nq = 0, nkv = 0, hd = 0, G = 0, max_splits = 0;
    const float2* rope = nullptr;
    float* apart = nullptr;
    int* err = nullptr;
    AttnFuse fuse;  // tickets set: the tensor-core kernel combines the splits itself
};
// Whether the split combine runs inside the attention kernel: the tensor-core layout, and at most
// 16 splits (contexts up to 1024), which the last CTA of a (sequence, kv head) loads in one round.
// Longer contexts measured faster with the combine kernel's parallel merge (70B at context 4096,
// two GPUs, batch 16: 616 against 682 tok/s).
static bool attention_combines(const AttnLaunch& a) { return a.hd == 128 && a.G >= 4 && a.max_splits <= 16; }
template <int MODE>
static cudaError_t launch_attention_t(const AttnLaunch& a, int B, cudaStream_t st) {
    const dim3 grid(a.max_splits, a.nkv, B), block(128);
    if (a.hd == 128 && a.G >= 4)
        return launch_pdl(attn_decode_tc_kernel<128, MODE>, grid, block, 0, st, a.qkv, a.qkv_rows, a.pos, a.btab,
                          a.mbps, a.kv_blocks, a.kc, a.vc, a.layer, a.L, a.nq, a.nkv, a.G, a.max_splits, a.rope,
                          a.apart, a.err, a.fuse);
    if (a.hd == 128)
        return launch_pdl(attn_decode_kernel<128, MODE>, grid, block, 0, st, a.qkv, a.qkv_rows, a.pos, a.btab, a.mbps,
                          a.kv_blocks, a.kc, a.vc, a.layer, a.L, a.nq, a.nkv, a.G, a.max_splits, a.rope, a.apart,
                          a.err);
    if (a.hd == 64)
        return launch_pdl(attn_decode_kernel<64, MODE>, grid, block, 0, st, a.qkv, a.qkv_rows, a.pos, a.btab, a.mbps,
                          a.kv_blocks, a.kc, a.vc, a.layer, a.L, a.nq, a.nkv, a.G, a.max_splits, a.rope, a.apart,
                          a.err);
    return launch_pdl(attn_decode_kernel<32, MODE>, grid, block, 0, st, a.qkv, a.qkv_rows, a.pos, a.btab, a.mbps,
                      a.kv_blocks, a.kc, a.vc, a.layer, a.L, a.nq, a.nkv, a.G, a.max_splits, a.rope, a.apart, a.err);
}
static cudaError_t launch_attention(const AttnLaunch& a, int B, int mode, cudaStream_t st) {
    if (mode == kAttnDecode) return launch_attention_t<kAttnDecode>(a, B, st);
    if (mode == kAttnPrefill) return launch_attention_t<kAttnPrefill>(a, B, st);
    return launch_attention_t<kAttnPlain>(a, B, st);
}

// Prefill: every row's k (rotated at its position) and v appended to its page before any row attends,
// so rows of one sequence in the same pass see each other causally. Block (kv head, row); thread i =
// RoPE pair i (engine.rs:383-390 order), the arithmetic of load_q_append_kv's append.
__global__ void kv_append_kernel(const float* __restrict__ qkv, int qkv_rows, const uint32_t* __restrict__ pos,
                                 const int32_t* __restrict__ btab, int mbps, int kv_blocks, __half* __restrict__ kc,
                                 __half* __restrict__ vc, int layer, int L, int nq, int nkv, int hd,
                                 const float2* __restrict__ rope, int* __restrict__ err) {
    pdl_launch_dependents();
    pdl_wait();
    const int h = blockIdx.x, b = blockIdx.y, half = hd / 2;
    const uint32_t p = pos[b];
    if (p >= (uint32_t)mbps * kPage) {
        if (h == 0 && threadIdx.x == 0) atomicOr(err, kErrAttnPos);
        return;
    }
    const int blk = btab[(size_t)b * mbps + p / kPage];
    if (blk < 0 || blk >= kv_blocks) {
        if (h == 0 && threadIdx.x == 0) atomicOr(err, kErrAttnPage);
        return;
    }
    const float* row = qkv + (size_t)b * qkv_rows;
    const float* k = row + (size_t)(nq + h) * hd;
    const float* v = row + (size_t)(nq + nkv + h) * hd;
    const float2* rp = rope + (size_t)p * half;
    const size_t off = ((((size_t)blk * L + layer) * nkv + h) * kPage + p % kPage) * hd;
    for (int i = threadIdx.x; i < half; i += blockDim.x) {
        const float2 cs = rp[i];
        const float2 r = rope_pair(k[2 * i], k[2 * i + 1], cs.x, cs.y);
        *reinterpret_cast<__half2*>(kc + off + 2 * i) = __floats2half2_rn(r.x, r.y);
        *reinterpret_cast<__half2*>(vc + off + 2 * i) = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
    }
}

// Rows sel[j] of x gathered into out [n][H] (the rows prefill returns logits for).
__global__ void gather_rows_kernel(const float* __restrict__ x, const uint32_t* __restrict__ sel, int H,
                                   float* __restrict__ out) {
    pdl_launch_dependents();
    pdl_wait();
    const float* src = x + (size_t)sel[blockIdx.x] * H;
    float* dst = out + (size_t)blockIdx.x * H;
    for (int i = threadIdx.x; i < H; i += blockDim.x) dst[i] = src[i];
}

static void destroy_model(pox_model* m);

// Destroys the models still registered on a context that is being destroyed.
void destroy_ctx_extras(pox_cuda_ctx* ctx) {
    std::vector<pox_model*> ms;
    {
        std::lock_guard<std::mutex> lk(ctx->mu);
        ms.swap(ctx->models);
    }
    for (pox_model* m : ms) destroy_model(m);
}

static int check_launch(const char* what) {
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? POX_OK : cuda_error(e, what);
}

// Concatenates INT4 projections with equal cols / group size row-wise (.pox payloads are row
// major, so the bytes concatenate; outlier flat indices shift by the rows before them).
static int concat_i4(const pox_tensor_desc* parts, int n, std::vector<uint8_t>& data, std::vector<uint8_t>& scales,
                     std::vector<uint8_t>& outl, pox_tensor_desc* out) {
    size_t rows = 0;
    std::vector<uint32_t> idx;
    std::vector<uint16_t> val;
    data.clear();
    scales.clear();
    for (int i = 0; i < n; i++) {
        const pox_tensor_desc& d = parts[i];
        if (d.dtype != POX_I4 || d.cols != parts[0].cols || d.group_size != parts[0].group_size)
            return set_error(POX_ERR_UNSUPPORTED, "model projections must be INT4 with one cols / group size");
        const size_t rb = (d.cols + 1) / 2, sb = (d.cols + d.group_size - 1) / d.group_size * 4;
        if (!d.data || d.data_len < d.rows * rb || !d.scales || d.scale_len < d.rows * sb)
            return set_error(POX_ERR_LAYOUT, "projection %d: buffer layout incompatible with 2D GEMV", i);
        data.insert(data.end(), d.data, d.data + d.rows * rb);
        scales.insert(scales.end(), d.scales, d.scales + d.rows * sb);
        if (d.outliers && d.outlier_len >= 4) {
            uint32_t cnt;
            std::memcpy(&cnt, d.outliers, 4);
            if (4 + 6 * (size_t)cnt > d.outlier_len) return set_error(POX_ERR_LAYOUT, "outlier table truncated");
            for (uint32_t e = 0; e < cnt; e++) {
                uint32_t fi;
                uint16_t fv;
                std::memcpy(&fi, d.outliers + 4 + 4 * (size_t)e, 4);
                std::memcpy(&fv, d.outliers + 4 + 4 * (size_t)cnt + 2 * (size_t)e, 2);
                if ((uint64_t)fi >= (uint64_t)d.rows * d.cols) continue;  // never matches a row
                idx.push_back((uint32_t)(fi + rows * d.cols));
                val.push_back(fv);
            }
        }
        rows += d.rows;
    }
    outl.clear();
    if (!idx.empty()) {
        const uint32_t cnt = (uint32_t)idx.size();
        outl.resize(4 + 6 * (size_t)cnt);
        std::memcpy(outl.data(), &cnt, 4);
        std::memcpy(outl.data() + 4, idx.data(), 4 * (size_t)cnt);
        std::memcpy(outl.data() + 4 + 4 * (size_t)cnt, val.data(), 2 * (size_t)cnt);
    }
    *out = pox_tensor_desc{};
    out->dtype = POX_I4;
    out->rows = rows;
    out->cols = parts[0].cols;
    out->group_size = parts[0].group_size;
    out->data = data.data();
    out->data_len = data.size();
    out->scales = scales.data();
    out->scale_len = scales.size();
    out->outliers = outl.empty() ? nullptr : outl.data();
    out->outlier_len = outl.size();
    return POX_OK;
}

static int upload_f16(const uint16_t* h, size_t n, uint16_t** d, cudaStream_t st) {
    if (!h) return set_error(POX_ERR_INVALID, "f16 buffer is NULL");
    cudaError_t e = cudaMalloc(d, n * 2);
    if (e == cudaSuccess) e = cudaMemcpyAsync(*d, h, n * 2, cudaMemcpyDefault, st);  // host or device source
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    return e == cudaSuccess ? POX_OK : cuda_error(e, "f16 upload");
}

static void free_tensor(pox_cuda_ctx* ctx, pox_tensor*& t) {
    if (t) pox_cuda_tensor_free(ctx, t);
    t = nullptr;
}

// x += W x_in for a row-split projection (o_proj, down_proj). One rank: the residual is added in
// the GEMV epilogue. Tensor parallel: each rank's GEMV writes its partial (rank 0's carrying the
// residual) where exchange `call` expects it, and the exchange leaves the sum over ranks in x.
static int row_split_gemv(pox_model* m, const pox_tensor* t, const float* xin, int B, int call, const PrepOp* op,
                          cudaStream_t st, bool prepared = false) {
    if (m->comm.tp == 1) return gemv_launch(m->ctx, t, xin, B, m->x, st, op, m->x, prepared);
    float* y = comm_partial(m->comm, call, m->x);
    int rc = gemv_launch(m->ctx, t, xin, B, y, st, op, m->comm.rank == 0 ? m->x : nullptr, prepared);
    if (rc) return rc;
    return comm_allreduce(m->comm, call, 2 * m->L + 1, m->x, (size_t)B * m->H, st);
}

// One pass of B rows through the model on device buffers already filled (m->tok, m->pos, m->btab).
// Decode: each row appends its own k / v inside the attention kernel; logits of every row.
// Prefill (n_out > 0): every row's k / v is appended before the attention of the layer, so rows of
// one sequence see each other causally; logits only of the n_out rows listed in m->sel.
static int forward_step(pox_model* m, int B, cudaStream_t st, bool prefill, int n_out) {
    pox_cuda_ctx* ctx = m->ctx;
    int rc;
    if (m->comm.tp > 1 && !m->comm.mode) return set_error(POX_ERR_INVALID, "tensor-parallel exchange not set up");
    cudaError_t le = launch_pdl(embed_kernel, dim3(B), dim3(256), 0, st, (const uint32_t*)m->tok,
                                (const uint16_t*)m->embed, m->V_full, m->H, m->x);
    if (le != cudaSuccess) return cuda_error(le, "embed launch");
    PrepOp norm;
    norm.mode = kPrepNorm;
    norm.eps = m->cfg.rms_eps;
    const bool persistent = !prefill && persist_supported(m, B);
    if (persistent && (rc = persist_launch(m, B, st))) return rc;
    for (int l = 0; l < m->L && !persistent; l++) {
        const LayerW& w = m->layers[l];
        if (!w.qkv) return set_error(POX_ERR_INVALID, "layer %d has no weights", l);
        norm.norm_w = w.attn_norm;
        if ((rc = gemv_launch(ctx, w.qkv, m->x, B, m->qkv, st, &norm))) return rc;
        AttnLaunch al;
        al.qkv = m->qkv;
        al.qkv_rows = m->qkv_rows;
        al.pos = m->pos;
        al.btab = m->btab;
        al.mbps = (int)m->max_blocks_per_seq;
        al.kv_blocks = (int)m->kv_blocks;
        al.kc = m->kc;
        al.vc = m->vc;
        al.layer = l;
        al.L = m->L;
        al.nq = m->nq;
        al.nkv = m->nkv;
        al.hd = m->hd;
        al.G = m->G;
        al.max_splits = m->max_splits;
        al.rope = m->rope;
        al.apart = m->apart;
        al.err = ctx->err_dev;
        cudaError_t e = cudaSuccess;
        if (prefill)
            e = launch_pdl(kv_append_kernel, dim3(m->nkv, B), dim3(64), 0, st, (const float*)m->qkv, m->qkv_rows,
                           (const uint32_t*)m->pos, (const int32_t*)m->btab, (int)m->max_blocks_per_seq,
                           (int)m->kv_blocks, m->kc, m->vc, l, m->L, m->nq, m->nkv, m->hd, (const float2*)m->rope,
                           ctx->err_dev);
        // the combine writes the o projection's prepared input when that tensor takes one
        OPrep op;
        XTarget xt;
        const bool fuse = (m->nq * m->hd) % 128 == 0 && w.o->tiled && w.o->dtype == POX_I4 &&
                          (size_t)B <= (gemv_uses_small_m(w.o, B) ? 128u : 8u) &&
                          gemv_x_target(ctx, w.o, B, st, &xt) == POX_OK;
        if (fuse) {
            op.cols = xt.cols;
            op.meta = xt.meta;
            op.Kp = xt.Kp;
            op.nxbs = xt.nxbs;
            op.xs = xt.xs;
            op.xscale = xt.xscale;
            op.xl = xt.xl;
            op.xm = xt.xm;
            op.Bp = xt.Bp;
        }
        // the tensor-core attention combines its splits itself (tickets shared with the persistent
        // kernel: the two never run at once); other layouts launch the combine kernel
        if (attention_combines(al)) {
            al.fuse.tickets = m->ptickets;
            al.fuse.att = m->att;
            al.fuse.op = op;
        }
        if (e == cudaSuccess) e = launch_attention(al, B, prefill ? kAttnPrefill : kAttnDecode, st);
        if (e != cudaSuccess) return cuda_error(e, "attention launch");
        if (!attention_combines(al)) {
            e = launch_pdl(attn_combine_kernel, dim3((m->nq * m->hd + 127) / 128, B), dim3(128), 0, st,
                           (const uint32_t*)m->pos, (uint32_t)(m->max_blocks_per_seq * kPage), m->nq, m->nkv, m->G,
                           m->hd, m->max_splits, (const float*)m->apart, m->att, op);
            if (e != cudaSuccess) return cuda_error(e, "attention combine launch");
        }
        if ((rc = row_split_gemv(m, w.o, m->att, B, 2 * l, nullptr, st, fuse))) return rc;
        norm.norm_w = w.mlp_norm;
        if ((rc = gemv_launch(ctx, w.gu, m->x, B, m->gu, st, &norm))) return rc;
        PrepOp sw;
        sw.mode = kPrepSwiGLU;
        sw.up = m->gu + m->I;
        sw.ld_x = 2 * m->I;
        sw.ld_up = 2 * m->I;
        if ((rc = row_split_gemv(m, w.down, m->gu, B, 2 * l + 1, &sw, st))) return rc;
    }
    norm.norm_w = m->final_norm;
    const float* xh = m->x;
    if (prefill) {
        le = launch_pdl(gather_rows_kernel, dim3(n_out), dim3(256), 0, st, (const float*)m->x, (const uint32_t*)m->sel,
                        m->H, m->xsel);
        if (le != cudaSuccess) return cuda_error(le, "gather launch");
        xh = m->xsel;
        B = n_out;
    }
    if ((rc = gemv_launch(ctx, m->lm_head, xh, B, m->logits, st, &norm))) return rc;
    const int parts = std::min(kArgmaxParts, (m->V + 2047) / 2048);
    const int chunk = (m->V + parts - 1) / parts;
    le = launch_pdl(argmax_part_kernel, dim3(parts, B), dim3(256), 0, st, m->logits, m->V, chunk, m->amax);
    if (le != cudaSuccess) return cuda_error(le, "argmax launch");
    const bool tp = m->comm.tp > 1;
    le = launch_pdl(argmax_final_kernel, dim3((B + 7) / 8), dim3(256), 0, st, (const float2*)m->amax, parts, B,
                    m->vocab_off, m->next, tp ? m->comm.pairs : (float2*)nullptr);
    if (le != cudaSuccess) return cuda_error(le, "argmax launch");
    if (tp) return comm_pick(m->comm, 2 * m->L, 2 * m->L + 1, B, m->next, st);
    return POX_OK;
}

}  // namespace pox

using namespace pox;

extern "C" int pox_cuda_model_create(pox_cuda_ctx* ctx, const pox_llama_config* cfg, uint32_t max_batch,
                                     uint32_t kv_blocks, uint32_t max_blocks_per_seq, pox_model** out) {
    return pox_cuda_model_create_tp(ctx, cfg, max_batch, kv_blocks, max_blocks_per_seq, 0, 1, out);
}

extern "C" int pox_cuda_model_create_tp(pox_cuda_ctx* ctx, const pox_llama_config* cfg, uint32_t max_batch,
                                        uint32_t kv_blocks, uint32_t max_blocks_per_seq, uint32_t tp_rank,
                                        uint32_t tp_size, pox_model** out) {
    if (!ctx || !cfg || !out) return set_error(POX_ERR_INVALID, "NULL argument");
    *out = nullptr;
    if (tp_size == 0 || tp_size > (uint32_t)kMaxTP || tp_rank >= tp_size)
        return set_error(POX_ERR_INVALID, "tensor-parallel rank %u of %u (at most %d ranks)", tp_rank, tp_size, kMaxTP);
    if (!cfg->hidden || !cfg->heads || !cfg->kv_heads || !cfg->layers || !cfg->vocab || !cfg->intermediate ||
        !max_batch || !kv_blocks || !max_blocks_per_seq)
        return set_error(POX_ERR_INVALID, "zero dimension in the model configuration");
    if (cfg->hidden % cfg->heads || cfg->heads % cfg->kv_heads)
        return set_error(POX_ERR_UNSUPPORTED, "hidden %% heads or heads %% kv_heads is not 0");
    const uint32_t hd = cfg->hidden / cfg->heads, G = cfg->heads / cfg->kv_heads;
    if ((hd != 32 && hd != 64 && hd != 128) || G > 8)
        return set_error(POX_ERR_UNSUPPORTED, "head_dim %u / %u query heads per kv head not supported", hd, G);
    if (cfg->hidden % 128 || cfg->intermediate % 128)
        return set_error(POX_ERR_UNSUPPORTED, "hidden and intermediate must be multiples of 128");
    if (cfg->heads % tp_size || cfg->kv_heads % tp_size || cfg->vocab % tp_size ||
        cfg->intermediate % (128 * tp_size))
        return set_error(POX_ERR_UNSUPPORTED,
                         "tensor parallel %u needs heads, kv_heads, vocab divisible by it and intermediate by 128x it",
                         tp_size);
    std::lock_guard<std::mutex> lk(ctx->mu);
    cudaError_t e = cudaSetDevice(ctx->device);
    if (e != cudaSuccess) return cuda_error(e, "cudaSetDevice");
    auto* m = new pox_model();
    m->ctx = ctx;
    m->cfg = *cfg;
    m->H = (int)cfg->hidden;
    m->I = (int)(cfg->intermediate / tp_size);
    m->V_full = (int)cfg->vocab;
    m->V = (int)(cfg->vocab / tp_size);
    m->vocab_off = (int)tp_rank * m->V;
    m->L = (int)cfg->layers;
    m->nq = (int)(cfg->heads / tp_size);
    m->nkv = (int)(cfg->kv_heads / tp_size);
    m->hd = (int)hd;
    m->G = (int)G;
    m->qkv_rows = (m->nq + 2 * m->nkv) * m->hd;
    m->max_batch = max_batch;
    m->kv_blocks = kv_blocks;
    m->max_blocks_per_seq = max_blocks_per_seq;
    m->max_splits = (int)((max_blocks_per_seq * kPage + kSplitTok - 1) / kSplitTok);
    m->layers.resize(m->L);
    m->pready.assign(m->L, 0);
    const size_t B = max_batch;
    const size_t kv_elems = (size_t)kv_blocks * m->L * m->nkv * kPage * m->hd;
    struct A { void** p; size_t bytes; } allocs[] = {
        {(void**)&m->kc, kv_elems * 2},
        {(void**)&m->vc, kv_elems * 2},
        {(void**)&m->x, B * m->H * 4},
        {(void**)&m->qkv, B * m->qkv_rows * 4},
        {(void**)&m->att, B * m->nq * m->hd * 4},
        {(void**)&m->gu, B * 2 * m->I * 4},
        {(void**)&m->logits, B * m->V * 4},
        {(void**)&m->apart, B * m->nkv * m->max_splits * m->G * (m->hd + 2) * 4},
        {(void**)&m->amax, B * kArgmaxParts * sizeof(float2)},
        {(void**)&m->tok, B * 4},
        {(void**)&m->pos, B * 4},
        {(void**)&m->next, B * 4},
        {(void**)&m->btab, B * max_blocks_per_seq * 4},
        {(void**)&m->rope, (size_t)max_blocks_per_seq * kPage * (m->hd / 2) * sizeof(float2)},
        {(void**)&m->sel, B * 4},
        {(void**)&m->xsel, B * m->H * 4},
        {(void**)&m->players, (size_t)m->L * sizeof(PLayer)},
        {(void**)&m->ptickets, B * m->nkv * 4},
        {(void**)&m->pbar, 4 * sizeof(unsigned)},
        {(void**)&m->pssq, (size_t)(m->H / 16) * 2 * kPMaxB * 4},
    };
    for (auto& a : allocs) {
        e = cudaMalloc(a.p, a.bytes);
        if (e != cudaSuccess) {
            for (auto& f : allocs) cudaFree(*f.p);
            delete m;
            return cuda_error(e, "cudaMalloc(model buffers)");
        }
    }
    if (tp_size > 1) {
        const int rc = comm_alloc(m->comm, (int)tp_rank, (int)tp_size, B, (size_t)m->H, ctx->err_dev);
        if (rc) {
            comm_free(m->comm);
            for (auto& f : allocs) cudaFree(*f.p);
            delete m;
            return rc;
        }
    }
    cudaMemsetAsync(m->players, 0, (size_t)m->L * sizeof(PLayer), ctx->stream);
    cudaMemsetAsync(m->ptickets, 0, B * m->nkv * 4, ctx->stream);
    cudaMemsetAsync(m->pbar, 0, 4 * sizeof(unsigned), ctx->stream);
    cudaMemsetAsync(m->kc, 0, kv_elems * 2, ctx->stream);
    cudaMemsetAsync(m->vc, 0, kv_elems * 2, ctx->stream);
    {
        const long long n = (long long)max_blocks_per_seq * kPage * (m->hd / 2);
        rope_table_kernel<<<(unsigned)((n + 255) / 256), 256, 0, ctx->stream>>>(
            m->rope, (int)(max_blocks_per_seq * kPage), m->hd, m->cfg.rope_theta);
    }
    e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) return cuda_error(e, "cudaMemset(KV pages)");
    ctx->models.push_back(m);
    *out = m;
    return POX_OK;
}

extern "C" void pox_cuda_model_destroy(pox_model* m) {
    if (!m) return;
    pox_cuda_ctx* ctx = m->ctx;
    {
        std::lock_guard<std::mutex> lk(ctx->mu);
        auto it = std::find(ctx->models.begin(), ctx->models.end(), m);
        if (it == ctx->models.end()) return;  // already destroyed with its context
        ctx->models.erase(it);
    }
    pox::destroy_model(m);
}

namespace pox {
static void destroy_model(pox_model* m) {
    pox_cuda_ctx* ctx = m->ctx;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    for (auto& w : m->layers) {
        free_tensor(ctx, w.qkv);
        free_tensor(ctx, w.o);
        free_tensor(ctx, w.gu);
        free_tensor(ctx, w.down);
        cudaFree(w.attn_norm);
        cudaFree(w.mlp_norm);
    }
    free_tensor(ctx, m->lm_head);
    void* bufs[] = {m->embed, m->final_norm, m->kc, m->vc, m->x, m->qkv, m->att, m->gu, m->logits, m->apart,
                    m->amax, m->tok, m->pos, m->next, m->btab, m->rope, m->sel, m->xsel,
                    m->players, m->ptickets, m->pbar, m->pssq};
    for (void* p : bufs) cudaFree(p);
    comm_free(m->comm);
    delete m;
}
}  // namespace pox

extern "C" int pox_cuda_model_set_embeddings(pox_model* m, const uint16_t* embed, const uint16_t* final_norm,
                                             const uint16_t* lm_head) {
    if (!m) return set_error(POX_ERR_INVALID, "model is NULL");
    pox_cuda_ctx* ctx = m->ctx;
    cudaStream_t st = ctx->stream;
    {
        std::lock_guard<std::mutex> lk(ctx->mu);
        cudaSetDevice(ctx->device);
        cudaFree(m->embed);
        cudaFree(m->final_norm);
        m->embed = m->final_norm = nullptr;
        int rc = upload_f16(embed, (size_t)m->V_full * m->H, &m->embed, st);
        if (!rc) rc = upload_f16(final_norm, (size_t)m->H, &m->final_norm, st);
        if (rc) return rc;
    }
    free_tensor(ctx, m->lm_head);
    pox_tensor_desc d = {};
    d.dtype = POX_F16;
    d.rows = (size_t)m->V;
    d.cols = (size_t)m->H;
    d.data = reinterpret_cast<const uint8_t*>(lm_head);
    d.data_len = (size_t)m->V * m->H * 2;
    return pox_cuda_tensor_upload(ctx, &d, &m->lm_head);
}

extern "C" int pox_cuda_model_set_layer(pox_model* m, uint32_t layer, const pox_tensor_desc* proj,
                                        const uint16_t* attn_norm, const uint16_t* mlp_norm) {
    if (!m || !proj) return set_error(POX_ERR_INVALID, "NULL argument");
    if (layer >= (uint32_t)m->L) return set_error(POX_ERR_INVALID, "layer %u out of range", layer);
    const size_t H = m->H, I = m->I, qd = (size_t)m->nq * m->hd, kvd = (size_t)m->nkv * m->hd;
    const size_t want[7][2] = {{qd, H}, {kvd, H}, {kvd, H}, {H, qd}, {I, H}, {I, H}, {H, I}};
    for (int i = 0; i < 7; i++)
        if (proj[i].rows != want[i][0] || proj[i].cols != want[i][1])
            return set_error(POX_ERR_LAYOUT, "projection %d is %zux%zu, expected %zux%zu", i, proj[i].rows,
                             proj[i].cols, want[i][0], want[i][1]);
    pox_cuda_ctx* ctx = m->ctx;
    LayerW& w = m->layers[layer];
    m->pready[layer] = 0;
    free_tensor(ctx, w.qkv);
    free_tensor(ctx, w.o);
    free_tensor(ctx, w.gu);
    free_tensor(ctx, w.down);
    std::vector<uint8_t> d0, s0, o0;
    pox_tensor_desc cat;
    int rc = concat_i4(proj, 3, d0, s0, o0, &cat);
    if (!rc) rc = pox_cuda_tensor_upload(ctx, &cat, &w.qkv);
    if (!rc) rc = concat_i4(proj + 3, 1, d0, s0, o0, &cat);
    if (!rc) rc = pox_cuda_tensor_upload(ctx, &cat, &w.o);
    if (!rc) rc = concat_i4(proj + 4, 2, d0, s0, o0, &cat);
    if (!rc) rc = pox_cuda_tensor_upload(ctx, &cat, &w.gu);
    if (!rc) rc = concat_i4(proj + 6, 1, d0, s0, o0, &cat);
    if (!rc) rc = pox_cuda_tensor_upload(ctx, &cat, &w.down);
    if (rc) return rc;
    for (pox_tensor* t : {w.qkv, w.o, w.gu, w.down})
        if (!t->tiled) return set_error(POX_ERR_UNSUPPORTED, "projections need cols %% 128 == 0 and group size %% 128 == 0");
    std::lock_guard<std::mutex> lk(ctx->mu);
    cudaSetDevice(ctx->device);
    cudaFree(w.attn_norm);
    cudaFree(w.mlp_norm);
    w.attn_norm = w.mlp_norm = nullptr;
    rc = upload_f16(attn_norm, H, &w.attn_norm, ctx->stream);
    if (!rc) rc = upload_f16(mlp_norm, H, &w.mlp_norm, ctx->stream);
    if (!rc) rc = persist_set_layer(m, (int)layer);
    return rc;
}

extern "C" int pox_cuda_model_set_layer_tensors(pox_model* m, uint32_t layer, pox_tensor* qkv, pox_tensor* o,
                                                pox_tensor* gate_up, pox_tensor* down, const uint16_t* attn_norm,
                                                const uint16_t* mlp_norm) {
    if (!m || !qkv || !o || !gate_up || !down) return set_error(POX_ERR_INVALID, "NULL argument");
    if (layer >= (uint32_t)m->L) return set_error(POX_ERR_INVALID, "layer %u out of range", layer);
    const size_t H = m->H, I = m->I, qd = (size_t)m->nq * m->hd;
    struct Want { pox_tensor* t; size_t rows, cols; } want[4] = {
        {qkv, (size_t)m->qkv_rows, H}, {o, H, qd}, {gate_up, 2 * I, H}, {down, H, I}};
    for (const Want& w : want) {
        if (w.t->rows != w.rows || w.t->cols != w.cols)
            return set_error(POX_ERR_LAYOUT, "tensor is %zux%zu, expected %zux%zu", w.t->rows, w.t->cols, w.rows,
                             w.cols);
        if (w.t->dtype != POX_I4 || !w.t->tiled)
            return set_error(POX_ERR_UNSUPPORTED, "layer tensors must be INT4 in the tiled layout");
    }
    pox_cuda_ctx* ctx = m->ctx;
    LayerW& lw = m->layers[layer];
    m->pready[layer] = 0;
    free_tensor(ctx, lw.qkv);
    free_tensor(ctx, lw.o);
    free_tensor(ctx, lw.gu);
    free_tensor(ctx, lw.down);
    lw.qkv = qkv;
    lw.o = o;
    lw.gu = gate_up;
    lw.down = down;
    std::lock_guard<std::mutex> lk(ctx->mu);
    cudaSetDevice(ctx->device);
    cudaFree(lw.attn_norm);
    cudaFree(lw.mlp_norm);
    lw.attn_norm = lw.mlp_norm = nullptr;
    int rc = upload_f16(attn_norm, H, &lw.attn_norm, ctx->stream);
    if (!rc) rc = upload_f16(mlp_norm, H, &lw.mlp_norm, ctx->stream);
    if (!rc) rc = persist_set_layer(m, (int)layer);
    return rc;
}

extern "C" int pox_cuda_model_set_persistent(pox_model* m, int enable) {
    if (!m) return set_error(POX_ERR_INVALID, "model is NULL");
    m->persist = enable ? 1 : 0;
    return POX_OK;
}

extern "C" int pox_cuda_model_step_persistent(const pox_model* m, uint32_t batch) {
    return m && persist_supported(m, (int)batch) ? 1 : 0;
}

extern "C" int pox_cuda_model_decode_device(pox_model* m, uint32_t batch, const uint32_t* tokens_dev,
                                            const uint32_t* positions_dev, const int32_t* block_tables_dev,
                                            float* logits_dev, uint32_t* next_dev, int advance, void* stream) {
    if (!m) return set_error(POX_ERR_INVALID, "model is NULL");
    if (batch == 0) return POX_OK;
    if (batch > m->max_batch) return set_error(POX_ERR_INVALID, "batch %u > max_batch %u", batch, m->max_batch);
    if (!m->embed || !m->lm_head) return set_error(POX_ERR_INVALID, "embeddings not set");
    pox_cuda_ctx* ctx = m->ctx;
    cudaError_t e = cudaSetDevice(ctx->device);
    if (e != cudaSuccess) return cuda_error(e, "cudaSetDevice");
    cudaStream_t st = stream ? (cudaStream_t)stream : ctx->stream;
    const size_t B = batch;
    if (tokens_dev && tokens_dev != m->tok)
        cudaMemcpyAsync(m->tok, tokens_dev, B * 4, cudaMemcpyDeviceToDevice, st);
    if (positions_dev && positions_dev != m->pos)
        cudaMemcpyAsync(m->pos, positions_dev, B * 4, cudaMemcpyDeviceToDevice, st);
    if (block_tables_dev && block_tables_dev != m->btab)
        cudaMemcpyAsync(m->btab, block_tables_dev, B * m->max_blocks_per_seq * 4, cudaMemcpyDeviceToDevice, st);
    int rc = forward_step(m, (int)batch, st, false, 0);
    if (rc) return rc;
    if (logits_dev) cudaMemcpyAsync(logits_dev, m->logits, B * m->V * 4, cudaMemcpyDeviceToDevice, st);
    if (next_dev) cudaMemcpyAsync(next_dev, m->next, B * 4, cudaMemcpyDeviceToDevice, st);
    if (advance) {
        advance_kernel<<<(batch + 127) / 128, 128, 0, st>>>(m->tok, m->pos, m->next, (int)batch);
        if ((rc = check_launch("advance"))) return rc;
    }
    e = cudaGetLastError();
    return e == cudaSuccess ? POX_OK : cuda_error(e, "decode step");
}

extern "C" int pox_cuda_model_decode(pox_model* m, uint32_t batch, const uint32_t* tokens, const uint32_t* positions,
                                     const int32_t* block_tables, float* logits, uint32_t* next_tokens) {
    if (!m) return set_error(POX_ERR_INVALID, "model is NULL");
    if (batch == 0) return POX_OK;
    if (!tokens || !positions || !block_tables) return set_error(POX_ERR_INVALID, "NULL input");
    if (batch > m->max_batch) return set_error(POX_ERR_INVALID, "batch %u > max_batch %u", batch, m->max_batch);
    for (uint32_t b = 0; b < batch; b++) {
        const uint32_t nb = positions[b] / kPage + 1;
        if (nb > m->max_blocks_per_seq)
            return set_error(POX_ERR_OOM, "position %u needs %u KV blocks, max_blocks_per_seq is %u", positions[b], nb,
                             m->max_blocks_per_seq);
        for (uint32_t j = 0; j < nb; j++) {
            const int32_t blk = block_tables[(size_t)b * m->max_blocks_per_seq + j];
            if (blk < 0 || (uint32_t)blk >= m->kv_blocks)
                return set_error(POX_ERR_INVALID, "block table entry %d of row %u out of range", blk, b);
        }
    }
    pox_cuda_ctx* ctx = m->ctx;
    std::lock_guard<std::mutex> lk(ctx->mu);
    cudaError_t e = cudaSetDevice(ctx->device);
    if (e != cudaSuccess) return cuda_error(e, "cudaSetDevice");
    cudaStream_t st = ctx->stream;
    const size_t B = batch;
    e = cudaMemcpyAsync(m->tok, tokens, B * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(m->pos, positions, B * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(m->btab, block_tables, B * m->max_blocks_per_seq * 4, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return cuda_error(e, "cudaMemcpy(decode inputs)");
    int rc = comm_reset(m->comm, st);
    if (!rc) rc = forward_step(m, (int)batch, st, false, 0);
    if (rc) return rc;
    if (logits) e = cudaMemcpyAsync(logits, m->logits, B * m->V * 4, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess && next_tokens) e = cudaMemcpyAsync(next_tokens, m->next, B * 4, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_error(e, "decode step");
    return take_kernel_error(ctx);
}

extern "C" int pox_cuda_model_prefill(pox_model* m, uint32_t rows, const uint32_t* tokens, const uint32_t* positions,
                                      const int32_t* block_tables, uint32_t n_out, const uint32_t* out_rows,
                                      float* logits, uint32_t* next_tokens) {
    if (!m) return set_error(POX_ERR_INVALID, "model is NULL");
    if (rows == 0) return POX_OK;
    if (!tokens || !positions || !block_tables || (n_out && !out_rows)) return set_error(POX_ERR_INVALID, "NULL input");
    if (rows > m->max_batch) return set_error(POX_ERR_INVALID, "%u rows > max_batch %u (split the pass)", rows, m->max_batch);
    if (n_out == 0 || n_out > rows) return set_error(POX_ERR_INVALID, "n_out %u must be in 1..rows", n_out);
    if (!m->embed || !m->lm_head) return set_error(POX_ERR_INVALID, "embeddings not set");
    for (uint32_t j = 0; j < n_out; j++)
        if (out_rows[j] >= rows) return set_error(POX_ERR_INVALID, "out_rows[%u] = %u >= rows", j, out_rows[j]);
    for (uint32_t b = 0; b < rows; b++) {
        const uint32_t nb = positions[b] / kPage + 1;
        if (nb > m->max_blocks_per_seq)
            return set_error(POX_ERR_OOM, "position %u needs %u KV blocks, max_blocks_per_seq is %u", positions[b], nb,
                             m->max_blocks_per_seq);
        for (uint32_t j = 0; j < nb; j++) {
            const int32_t blk = block_tables[(size_t)b * m->max_blocks_per_seq + j];
            if (blk < 0 || (uint32_t)blk >= m->kv_blocks)
                return set_error(POX_ERR_INVALID, "block table entry %d of row %u out of range", blk, b);
        }
    }
    pox_cuda_ctx* ctx = m->ctx;
    std::lock_guard<std::mutex> lk(ctx->mu);
    cudaError_t e = cudaSetDevice(ctx->device);
    if (e != cudaSuccess) return cuda_error(e, "cudaSetDevice");
    cudaStream_t st = ctx->stream;
    const size_t B = rows;
    e = cudaMemcpyAsync(m->tok, tokens, B * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(m->pos, positions, B * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(m->btab, block_tables, B * m->max_blocks_per_seq * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(m->sel, out_rows, (size_t)n_out * 4, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return cuda_error(e, "cudaMemcpy(prefill inputs)");
    int rc = comm_reset(m->comm, st);
    if (!rc) rc = forward_step(m, (int)rows, st, true, (int)n_out);
    if (rc) return rc;
    if (logits) e = cudaMemcpyAsync(logits, m->logits, (size_t)n_out * m->V * 4, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess && next_tokens)
        e = cudaMemcpyAsync(next_tokens, m->next, (size_t)n_out * 4, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_error(e, "prefill");
    return take_kernel_error(ctx);
}

extern "C" int pox_cuda_model_set_state(pox_model* m, uint32_t batch, const uint32_t* tokens, const uint32_t* positions,
                                        const int32_t* block_tables) {
    if (!m || !tokens || !positions || !block_tables) return set_error(POX_ERR_INVALID, "NULL argument");
    if (batch == 0 || batch > m->max_batch) return set_error(POX_ERR_INVALID, "batch %u out of range", batch);
    for (uint32_t b = 0; b < batch * m->max_blocks_per_seq; b++)
        if (block_tables[b] >= (int32_t)m->kv_blocks)
            return set_error(POX_ERR_INVALID, "block table entry %d out of range", block_tables[b]);
    for (uint32_t b = 0; b < batch; b++) {  // the pages up to each row's next position must exist
        const uint32_t nb = positions[b] / kPage + 1;
        if (nb > m->max_blocks_per_seq)
            return set_error(POX_ERR_OOM, "position %u needs %u KV blocks, max_blocks_per_seq is %u", positions[b], nb,
                             m->max_blocks_per_seq);
        for (uint32_t j = 0; j < nb; j++)
            if (block_tables[(size_t)b * m->max_blocks_per_seq + j] < 0)
                return set_error(POX_ERR_INVALID, "row %u: page %u (position %u) has no block", b, j, positions[b]);
    }
    pox_cuda_ctx* ctx = m->ctx;
    std::lock_guard<std::mutex> lk(ctx->mu);
    cudaError_t e = cudaSetDevice(ctx->device);
    const size_t B = batch;
    if (e == cudaSuccess) e = cudaMemcpyAsync(m->tok, tokens, B * 4, cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(m->pos, positions, B * 4, cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(m->btab, block_tables, B * m->max_blocks_per_seq * 4, cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess && comm_reset(m->comm, ctx->stream)) return POX_ERR_CUDA;
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    return e == cudaSuccess ? POX_OK : cuda_error(e, "set_state");
}

extern "C" int pox_cuda_model_buffers(pox_model* m, uint32_t** tokens_dev, uint32_t** positions_dev,
                                      int32_t** block_tables_dev, float** logits_dev, uint32_t** next_dev) {
    if (!m) return set_error(POX_ERR_INVALID, "model is NULL");
    if (tokens_dev) *tokens_dev = m->tok;
    if (positions_dev) *positions_dev = m->pos;
    if (block_tables_dev) *block_tables_dev = m->btab;
    if (logits_dev) *logits_dev = m->logits;
    if (next_dev) *next_dev = m->next;
    return POX_OK;
}

extern "C" int pox_cuda_comm_unique_id(uint8_t id[128]) {
    if (!id) return set_error(POX_ERR_INVALID, "NULL argument");
#ifdef POX_HAVE_NCCL
    ncclUniqueId uid;
    const ncclResult_t r = ncclGetUniqueId(&uid);
    if (r != ncclSuccess) return set_error(POX_ERR_NCCL, "ncclGetUniqueId: %s", ncclGetErrorString(r));
    std::memcpy(id, &uid, 128);
    return POX_OK;
#else
    return set_error(POX_ERR_UNSUPPORTED, "built without NCCL");
#endif
}

static int tp_model(pox_model* m) {
    if (!m) return set_error(POX_ERR_INVALID, "model is NULL");
    if (m->comm.tp < 2) return set_error(POX_ERR_INVALID, "model is not tensor parallel");
    const cudaError_t e = cudaSetDevice(m->ctx->device);
    return e == cudaSuccess ? POX_OK : cuda_error(e, "cudaSetDevice");
}

extern "C" int pox_cuda_model_comm_nccl(pox_model* m, const uint8_t id[128]) {
    int rc = tp_model(m);
    if (rc) return rc;
    if (!id) return set_error(POX_ERR_INVALID, "NULL id");
    return comm_init_nccl(m->comm, id);
}

extern "C" int pox_cuda_model_comm_ipc_handle(pox_model* m, uint8_t handle[64]) {
    int rc = tp_model(m);
    if (rc) return rc;
    if (!handle) return set_error(POX_ERR_INVALID, "NULL handle");
    return comm_ipc_handle(m->comm, handle);
}

extern "C" int pox_cuda_model_comm_peer(pox_model* m, const uint8_t* handles) {
    int rc = tp_model(m);
    if (rc) return rc;
    if (!handles) return set_error(POX_ERR_INVALID, "NULL handles");
    return comm_open_peers(m->comm, handles);
}

extern "C" int pox_cuda_model_comm_mode(pox_model* m, int mode) {
    int rc = tp_model(m);
    if (rc) return rc;
    if (mode == POX_COMM_NCCL && !m->comm.nccl) return set_error(POX_ERR_INVALID, "NCCL communicator not set up");
    if (mode == POX_COMM_PEER && !m->comm.peer_ready) return set_error(POX_ERR_INVALID, "peer buffers not opened");
    if (mode != POX_COMM_NCCL && mode != POX_COMM_PEER) return set_error(POX_ERR_INVALID, "unknown mode %d", mode);
    m->comm.mode = mode;
    return POX_OK;
}

extern "C" int pox_cuda_paged_attention(pox_cuda_ctx* ctx, const float* q_dev, const uint16_t* k_pages_dev,
                                        const uint16_t* v_pages_dev, const int32_t* block_tables_dev,
                                        const uint32_t* positions_dev, uint32_t batch, uint32_t heads,
                                        uint32_t kv_heads, uint32_t head_dim, uint32_t num_blocks,
                                        uint32_t max_blocks_per_seq, float* out_dev, void* stream) {
    if (!ctx) return set_error(POX_ERR_INVALID, "ctx is NULL");
    if (batch == 0) return POX_OK;
    if (!q_dev || !k_pages_dev || !v_pages_dev || !block_tables_dev || !positions_dev || !out_dev)
        return set_error(POX_ERR_INVALID, "NULL device pointer");
    if (!heads || !kv_heads || !num_blocks || !max_blocks_per_seq)
        return set_error(POX_ERR_INVALID, "zero heads, kv_heads, num_blocks or max_blocks_per_seq");
    if (heads % kv_heads || heads / kv_heads > 8 || (head_dim != 32 && head_dim != 64 && head_dim != 128))
        return set_error(POX_ERR_UNSUPPORTED, "%u heads over %u kv heads of dim %u (supported: head_dim 32/64/128, "
                         "at most 8 query heads per kv head)", heads, kv_heads, head_dim);
    if ((((uintptr_t)k_pages_dev | (uintptr_t)v_pages_dev) & 15) || ((uintptr_t)q_dev & 7) || ((uintptr_t)out_dev & 3))
        return set_error(POX_ERR_INVALID, "K/V pages must be 16-byte aligned, q 8-byte aligned");
    if (batch > 65535 || max_blocks_per_seq > (1u << 20))
        return set_error(POX_ERR_UNSUPPORTED, "batch %u / max_blocks_per_seq %u too large", batch, max_blocks_per_seq);
    const int G = (int)(heads / kv_heads);
    const int max_splits = (int)((max_blocks_per_seq * kPage + kSplitTok - 1) / kSplitTok);
    const size_t need = (size_t)batch * kv_heads * max_splits * G * (head_dim + 2) * sizeof(float);
    cudaError_t e = cudaSetDevice(ctx->device);
    if (e != cudaSuccess) return cuda_error(e, "cudaSetDevice");
    cudaStream_t st = stream ? (cudaStream_t)stream : ctx->stream;
    float* apart = nullptr;
    {
        std::lock_guard<std::mutex> lk(ctx->mu);
        if (need > ctx->attn_scratch_bytes) {
            cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
            if (cudaStreamIsCapturing(st, &cs) == cudaSuccess && cs != cudaStreamCaptureStatusNone)
                return set_error(POX_ERR_INVALID, "attention scratch must be sized by a call before stream capture");
            e = cudaDeviceSynchronize();  // the old scratch may still be in use by earlier calls
            if (e == cudaSuccess) {
                cudaFree(ctx->attn_scratch);
                ctx->attn_scratch = nullptr;
                ctx->attn_scratch_bytes = 0;
                e = cudaMalloc(&ctx->attn_scratch, need);
            }
            if (e != cudaSuccess) return cuda_error(e, "cudaMalloc(attention partials)");
            ctx->attn_scratch_bytes = need;
        }
        apart = static_cast<float*>(ctx->attn_scratch);
    }
    AttnLaunch al;
    al.qkv = q_dev;
    al.qkv_rows = (int)(heads * head_dim);
    al.pos = positions_dev;
    al.btab = block_tables_dev;
    al.mbps = (int)max_blocks_per_seq;
    al.kv_blocks = (int)num_blocks;
    al.kc = reinterpret_cast<__half*>(const_cast<uint16_t*>(k_pages_dev));  // read only in kAttnPlain
    al.vc = reinterpret_cast<__half*>(const_cast<uint16_t*>(v_pages_dev));
    al.layer = 0;
    al.L = 1;
    al.nq = (int)heads;
    al.nkv = (int)kv_heads;
    al.hd = (int)head_dim;
    al.G = G;
    al.max_splits = max_splits;
    al.apart = apart;
    al.err = ctx->err_dev;
    e = launch_attention(al, (int)batch, kAttnPlain, st);
    if (e != cudaSuccess) return cuda_error(e, "attention launch");
    e = launch_pdl(attn_combine_kernel, dim3((heads * head_dim + 127) / 128, batch), dim3(128), 0, st, positions_dev,
                   (uint32_t)(max_blocks_per_seq * kPage), (int)heads, (int)kv_heads, G, (int)head_dim, max_splits,
                   (const float*)apart, out_dev, OPrep());
    if (e != cudaSuccess) return cuda_error(e, "attention combine launch");
    return POX_OK;
}
