// gemv_stream.cu -- the batch <= 8 quantized GEMV as one persistent stream per SM, with the x
// preparation (and the decode step's RMSNorm / SwiGLU) fused in.
//
// Same contract as quant::gemv_int4 / gemv_int8 and the F16 projection (crates/paraoxidizer-quant/
// src/kernels.rs:177-255, crates/paraoxidizer-runtime/src/engine.rs:235-250) and the same arithmetic
// as gemv_tc_kernel (gemv.cu): INT4 / INT8 tiles enter mma.sync m16n8k32 as exact integers against x
// as the 15-bit two-limb fixed point of each 128-k block, the group's affine map applied once per
// tile; F16 tiles take x as f16 hi / lo pairs; outliers add (v - dequant(q)) x[c] per row.
//
// What differs is how the work reaches the SMs:
//  * One CTA per SM (at most one per row tile of 16 rows). The tiles are one row-tile-major stream of
//    nT * nkb tiles; CTA c takes the contiguous slice [c L / C, (c + 1) L / C), i.e. one contiguous
//    byte range of the weights, so every CTA streams the same number of bytes.
//  * One producer thread copies that range into a ring of shared-memory stages with bulk copies
//    (one stage = up to 8 consecutive tiles of one row tile), starting before the kernel waits on
//    its predecessor: weights are immutable.
//  * Eight consumer warps take one tile each per stage. Before that they build the prepared x of the
//    whole K range in shared memory from the raw f32 rows (with the fused pre-op), after the
//    programmatic-dependent-launch wait.
//  * The ring takes the shared memory the x staging leaves: under load the memory system needs about
//    100 KB in flight per SM to reach the copy bandwidth.
//  * A row tile split between two CTAs (only the first and the last row tile of a slice can be) is
//    finished by whichever of the two arrives second (a per-row-tile ticket): it adds the two partial
//    sums in CTA order, so results do not depend on timing. Tickets reset themselves.
//  * Every wait is bounded; a timeout raises the context error flag and stops the CTA's stream after
//    the copies in flight have landed.
#include <algorithm>
#include <cstdlib>
#include <map>
#include <mutex>
#include <tuple>

#include "common.cuh"
#include "gemv.cuh"
#include "tc05.cuh"

namespace pox {

constexpr int kSW = 8;                  // consumer warps (one tile each per stage)
constexpr int kSThreads = (kSW + 1) * 32;
constexpr int kSEntCap = 1024;          // outlier entries of a row tile staged in shared memory
constexpr int kErrWaitStream = 256;     // bit of the kernel error flag
constexpr int kStreamSmemMax = 227 * 1024;
// Shared memory a CTA may use (ring stages fill what the x staging leaves). POX_STREAM_SMEM_KB in the
// environment overrides it (110 keeps a CTA within half an SM, so the next launch's CTA fits beside).
static int stream_smem_budget() {
    static const int v = [] {
        const char* e = getenv("POX_STREAM_SMEM_KB");
        const int kb = e ? atoi(e) : 220;
        return std::max(48, std::min(kb, 226)) * 1024;
    }();
    return v;
}
constexpr int kStreamMaxStages = 32;
constexpr int kPrepBatch = 8;           // x items whose loads one warp issues together

struct StreamPlan {
    int nst, cstride, nxr;
    int ring, bars, xs, xm, red, ocorr, ent, zero, misc, total;
};

__host__ __device__ inline StreamPlan stream_plan(int kind, int B, int K, bool outl, int nst) {
    StreamPlan p;
    const int XB = kind == kKindF16 ? 2 : 1;
    const int tb = kind_tile_bytes(kind);
    const int Kp = ((K + kXBlock - 1) / kXBlock) * kXBlock;
    p.nst = nst;
    p.cstride = ((Kp * XB + 127) & ~127) + (kind == kKindI4 ? 16 : 64);
    p.nxr = ((Kp / kXBlock) + 1) & ~1;
    int o = 0;
    p.ring = o; o += nst * kSW * tb;
    p.bars = o; o += (2 * nst + 4) * 8;
    o = (o + 15) & ~15;
    p.xs = o;   o += (2 * B * p.cstride + 15) & ~15;
    p.xm = o;   o += kind == kKindF16 ? 0 : B * p.nxr * 8;
    p.red = o;  o += 2 * kSW * 128 * 4;
    p.ocorr = o; o += 2 * 128 * 4;
    p.ent = o;  o += outl ? 2 * kSEntCap * 8 : 0;
    p.zero = o; o += 32;
    p.misc = o; o += 64;  // RMSNorm scales [8], flags
    p.total = o;
    return p;
}

// Bounded mbarrier wait that gives up at once when the CTA has already aborted.
__device__ __forceinline__ bool stream_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* err) {
    if (*abort_flag) return false;
    if (mbar_wait(bar, parity)) return true;
    *abort_flag = 1;
    atomicOr(err, kErrWaitStream);
    return false;
}

__device__ __forceinline__ void consumer_sync() {
    asm volatile("bar.sync 1, %0;" ::"r"(kSW * 32) : "memory");
}

template <int KIND, int BT>
__global__ void __launch_bounds__(kSThreads, 1) gemv_stream_kernel(const StreamArgs a, const int nst) {
    constexpr int KB = KIND == kKindI4 ? 128 : (KIND == kKindI8 ? 64 : 32);
    constexpr int NB = BT > 4 ? 2 : 1;
    constexpr int TB = kTileBytes + (KIND == kKindI4 ? 64 : 0);
    constexpr int SB = kSW * TB;  // stage bytes
    extern __shared__ __align__(128) unsigned char smem[];

    const int B = BT > 4 ? a.B : BT;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
    const int nkb = a.nkb, K = a.K;
    const bool has_out = KIND == kKindI4 && a.row_ptr != nullptr;
    const StreamPlan P = stream_plan(KIND, B, K, has_out, nst);
    const uint32_t sbase = smem_u32(smem);
    const uint32_t ring = sbase + P.ring;
    auto full = [&](int s) { return sbase + P.bars + 8 * s; };
    auto empty = [&](int s) { return sbase + P.bars + 8 * (nst + s); };
    auto ebar = [&](int p) { return sbase + P.bars + 8 * (2 * nst + p); };
    auto efree = [&](int p) { return sbase + P.bars + 8 * (2 * nst + 2 + p); };
    const uint32_t xs = sbase + P.xs, zero = sbase + P.zero;
    const int cs = P.cstride;
    float2* xms = reinterpret_cast<float2*>(smem + P.xm);
    float* red = reinterpret_cast<float*>(smem + P.red);
    float* ocorr = reinterpret_cast<float*>(smem + P.ocorr);
    const uint2* ent_s = reinterpret_cast<const uint2*>(smem + P.ent);
    float* s_inv = reinterpret_cast<float*>(smem + P.misc);
    volatile int* s_abort = reinterpret_cast<volatile int*>(smem + P.misc + 32);
    volatile int* s_last = reinterpret_cast<volatile int*>(smem + P.misc + 36);

    // this CTA's slice of the row-tile-major tile stream
    const long long L = (long long)a.nT * nkb;
    const int c = blockIdx.x;
    const long long j0 = L * c / a.C, j1 = L * (c + 1) / a.C;
    const int T0 = (int)(j0 / nkb), T1 = (int)((j1 - 1) / nkb);

    if (tid == 0) {
        for (int s = 0; s < nst; s++) {
            mbar_init(full(s), 1);
            mbar_init(empty(s), kSW);
        }
        for (int p = 0; p < 2; p++) {
            mbar_init(ebar(p), 1);
            mbar_init(efree(p), 1);
        }
        *s_abort = 0;
    }
    if (tid < 8) reinterpret_cast<uint32_t*>(smem + P.zero)[tid] = 0u;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    __syncthreads();
    pdl_launch_dependents();

    if (warp == kSW) {
        // ---------------- producer: the slice's tiles, stage by stage, and each row tile's entries ----------------
        if (lane == 0) {
            int gi = 0, ni = 0;  // stages and entry copies issued
            for (int T = T0; T <= T1 && !*s_abort; T++, ni++) {
                const int ka = T == T0 ? (int)(j0 - (long long)T * nkb) : 0;
                const int kz = T == T1 ? (int)(j1 - (long long)T * nkb) : nkb;
                if (has_out) {
                    const int p = ni & 1;
                    if (ni >= 2 && !stream_wait(efree(p), ((ni - 2) >> 1) & 1, s_abort, a.err)) break;
                    const uint32_t lo = __ldg(a.row_ptr + T * 16) & ~1u;
                    const uint32_t hi = __ldg(a.row_ptr + min(T * 16 + 16, a.N));
                    const uint32_t n = min((hi - lo + 1) & ~1u, (uint32_t)kSEntCap);  // entries carry 2 pad slots
                    mbar_expect_tx(ebar(p), n * 8);
                    if (n) bulk_g2s(sbase + P.ent + p * kSEntCap * 8, a.ent + lo, n * 8, ebar(p));
                }
                for (int k = ka; k < kz; k += kSW) {
                    const int nt = min(kSW, kz - k), s = gi % nst;
                    if (gi >= nst && !stream_wait(empty(s), ((gi / nst) - 1) & 1, s_abort, a.err)) break;
                    mbar_expect_tx(full(s), nt * TB);
                    bulk_g2s(ring + s * SB, a.w + ((size_t)T * nkb + k) * TB, nt * TB, full(s));
                    gi++;
                }
            }
            if (*s_abort) {
                // never leave with copies in flight into this CTA's shared memory: the last stages and
                // entry buffers issued are waited for (bounded) before the warp exits
                for (int q = max(0, gi - nst); q < gi; q++) mbar_wait(full(q % nst), (q / nst) & 1);
                for (int q = max(0, ni - 2); q < ni && has_out; q++) mbar_wait(ebar(q & 1), (q >> 1) & 1);
            }
        }
        return;
    }

    // ---------------- consumers: prepared x of the whole K range into shared memory ----------------
    // Loads are issued in batches of kPrepBatch independent items per warp (one L2 round trip per
    // batch instead of one per item).
    pdl_wait();
    const PrepOp& op = a.op;
    const int ldx = op.ld_x ? op.ld_x : K;
    if (op.mode == kPrepNorm) {
        // RMSNorm scale of each row: thread sums of squares in k order, warps in a butterfly, then
        // the warps' sums in warp order
        for (int b = 0; b < B; b++) {
            const float* xr = a.x + (size_t)b * ldx;
            float s = 0.f;
            for (int k0 = 4 * tid; k0 < K; k0 += 4 * kSW * 32 * kPrepBatch) {
                float4 v[kPrepBatch];
#pragma unroll
                for (int q = 0; q < kPrepBatch; q++) {
                    const int k = k0 + q * 4 * kSW * 32;
                    v[q] = k < K ? *reinterpret_cast<const float4*>(xr + k) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int q = 0; q < kPrepBatch; q++) {
                    s = fmaf(v[q].x, v[q].x, s);
                    s = fmaf(v[q].y, v[q].y, s);
                    s = fmaf(v[q].z, v[q].z, s);
                    s = fmaf(v[q].w, v[q].w, s);
                }
            }
            s = warp_sum(s);
            if (lane == 0) red[b * kSW + warp] = s;
        }
        consumer_sync();
        if (tid < B) {
            float s = 0.f;
            for (int w = 0; w < kSW; w++) s += red[tid * kSW + w];
            s_inv[tid] = 1.0f / sqrtf(s / (float)K + op.eps);
        }
        consumer_sync();
    }
    const bool swiglu = op.mode == kPrepSwiGLU, norm = op.mode == kPrepNorm;
    if (KIND == kKindF16) {
        // f16 hi / lo pairs, two elements per lane, 64 elements per warp item
        const int per = (K + 63) / 64, nit = B * per;
        for (int base = warp; base < nit; base += kSW * kPrepBatch) {
            float2 v[kPrepBatch], u[kPrepBatch];
            uint32_t w2[kPrepBatch];
#pragma unroll
            for (int q = 0; q < kPrepBatch; q++) {
                const int it = base + q * kSW, b = it / per, k = (it % per) * 64 + 2 * lane;
                v[q] = u[q] = make_float2(0.f, 0.f);
                w2[q] = 0x3C003C00u;  // f16 (1, 1)
                if (it < nit && k < K) {
                    v[q] = *reinterpret_cast<const float2*>(a.x + (size_t)b * ldx + k);
                    if (swiglu) u[q] = *reinterpret_cast<const float2*>(op.up + (size_t)b * op.ld_up + k);
                    if (norm && op.norm_w) w2[q] = *reinterpret_cast<const uint32_t*>(op.norm_w + k);
                }
            }
#pragma unroll
            for (int q = 0; q < kPrepBatch; q++) {
                const int it = base + q * kSW, b = it / per, k = (it % per) * 64 + 2 * lane;
                if (it >= nit) continue;
                float2 e = v[q];
                if (k < K) {
                    if (norm) {
                        e.x *= s_inv[b];
                        e.y *= s_inv[b];
                        if (op.norm_w) {
                            e.x *= half_bits_to_float(w2[q]);
                            e.y *= half_bits_to_float(w2[q] >> 16);
                        }
                    } else if (swiglu) {
                        e.x = e.x / (1.0f + expf(-e.x)) * u[q].x;
                        e.y = e.y / (1.0f + expf(-e.y)) * u[q].y;
                    }
                }
                const __half h0 = __float2half_rn(e.x), h1 = __float2half_rn(e.y);
                const __half l0 = __float2half_rn(e.x - __half2float(h0)), l1 = __float2half_rn(e.y - __half2float(h1));
                *reinterpret_cast<__half2*>(smem + P.xs + (2 * b) * cs + 2 * k) = __halves2half2(h0, h1);
                *reinterpret_cast<__half2*>(smem + P.xs + (2 * b + 1) * cs + 2 * k) = __halves2half2(l0, l1);
            }
        }
    } else {
        // per 128-k block: X = rint(x * 16383 / max|x|) as exact int8 limbs X = 128 hi + lo, and
        // (max|x| / 16383, sum x) -- the arithmetic of xprep_int_kernel. The kPrepBatch items of a
        // batch go through each step together, so their shuffle reductions overlap instead of
        // forming one long dependent chain per item.
        const int nxb = (K + kXBlock - 1) / kXBlock, nit = B * nxb;
        for (int base = warp; base < nit; base += kSW * kPrepBatch) {
            float4 v[kPrepBatch];
#pragma unroll
            for (int q = 0; q < kPrepBatch; q++) {
                const int it = base + q * kSW, b = it / nxb, k = (it % nxb) * kXBlock + lane * 4;
                v[q] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (it < nit && k < K) v[q] = *reinterpret_cast<const float4*>(a.x + (size_t)b * ldx + k);
            }
            if (norm || swiglu) {
#pragma unroll
                for (int q = 0; q < kPrepBatch; q++) {
                    const int it = base + q * kSW, b = it / nxb, k = (it % nxb) * kXBlock + lane * 4;
                    if (it < nit && k < K) {
                        if (norm) {
                            const float si = s_inv[b];
                            v[q].x *= si;
                            v[q].y *= si;
                            v[q].z *= si;
                            v[q].w *= si;
                            if (op.norm_w) {
                                const uint2 w4 = *reinterpret_cast<const uint2*>(op.norm_w + k);
                                v[q].x *= half_bits_to_float(w4.x);
                                v[q].y *= half_bits_to_float(w4.x >> 16);
                                v[q].z *= half_bits_to_float(w4.y);
                                v[q].w *= half_bits_to_float(w4.y >> 16);
                            }
                        } else {
                            const float4 u = *reinterpret_cast<const float4*>(op.up + (size_t)b * op.ld_up + k);
                            v[q].x = v[q].x / (1.0f + expf(-v[q].x)) * u.x;
                            v[q].y = v[q].y / (1.0f + expf(-v[q].y)) * u.y;
                            v[q].z = v[q].z / (1.0f + expf(-v[q].z)) * u.z;
                            v[q].w = v[q].w / (1.0f + expf(-v[q].w)) * u.w;
                        }
                    }
                }
            }
            float m[kPrepBatch], sm[kPrepBatch];
#pragma unroll
            for (int q = 0; q < kPrepBatch; q++) {
                m[q] = fmaxf(fmaxf(fabsf(v[q].x), fabsf(v[q].y)), fmaxf(fabsf(v[q].z), fabsf(v[q].w)));
                sm[q] = (v[q].x + v[q].y) + (v[q].z + v[q].w);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1)
#pragma unroll
                for (int q = 0; q < kPrepBatch; q++) {
                    m[q] = fmaxf(m[q], __shfl_xor_sync(0xffffffffu, m[q], o));
                    sm[q] += __shfl_xor_sync(0xffffffffu, sm[q], o);
                }
#pragma unroll
            for (int q = 0; q < kPrepBatch; q++) {
                const int it = base + q * kSW, b = it / nxb, blk = it % nxb, k = blk * kXBlock + lane * 4;
                if (it >= nit) continue;  // warp-uniform
                const float inv = m[q] > 0.f ? (float)kXLimbMax / m[q] : 0.f;
                const int X[4] = {__float2int_rn(v[q].x * inv), __float2int_rn(v[q].y * inv),
                                  __float2int_rn(v[q].z * inv), __float2int_rn(v[q].w * inv)};
                uint32_t hi = 0, lo = 0;
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const int qv = max(-kXLimbMax, min(kXLimbMax, X[i]));
                    hi |= ((uint32_t)(qv >> 7) & 0xFFu) << (8 * i);
                    lo |= ((uint32_t)qv & 0x7Fu) << (8 * i);
                }
                *reinterpret_cast<uint32_t*>(smem + P.xs + (2 * b) * cs + k) = hi;
                *reinterpret_cast<uint32_t*>(smem + P.xs + (2 * b + 1) * cs + k) = lo;
                if (lane == 0) xms[b * P.nxr + blk] = make_float2(m[q] > 0.f ? m[q] / (float)kXLimbMax : 0.f, sm[q]);
            }
        }
    }
    consumer_sync();

    // ---------------- consumers: the slice's row tiles ----------------
    const float oscale = KIND == kKindI8 ? a.i8_scale : 1.f;
    int gi = 0, ni = 0;
    for (int T = T0; T <= T1; T++, ni++) {
        const int ka = T == T0 ? (int)(j0 - (long long)T * nkb) : 0;
        const int kz = T == T1 ? (int)(j1 - (long long)T * nkb) : nkb;
        const int p = ni & 1;
        // outlier CSR bounds of this warp's two rows (prefetched; used after the tiles)
        uint32_t rb0 = 0, rb1 = 0, rb2 = 0, elo = 0;
        if (has_out) {
            const int r0 = min(T * 16 + 2 * warp, a.N);
            rb0 = __ldg(a.row_ptr + r0);
            rb1 = __ldg(a.row_ptr + min(r0 + 1, a.N));
            rb2 = __ldg(a.row_ptr + min(r0 + 2, a.N));
            elo = __ldg(a.row_ptr + T * 16) & ~1u;
        }
        float acc[NB][2], fd[NB][4];
#pragma unroll
        for (int nb = 0; nb < NB; nb++) {
            acc[nb][0] = acc[nb][1] = 0.f;
            fd[nb][0] = fd[nb][1] = fd[nb][2] = fd[nb][3] = 0.f;
        }
        for (int k = ka; k < kz; k += kSW, gi++) {
            const int nt = min(kSW, kz - k), s = gi % nst;
            const bool ok = stream_wait(full(s), (gi / nst) & 1, s_abort, a.err);
            if (ok && warp < nt) {
                const int kb = k + warp;
                const uint32_t tile = ring + s * SB + warp * TB;
                const uint4 wa = lds128(tile + lane * 16), wb = lds128(tile + lane * 16 + 512);
                if (KIND == kKindI4) {
                    const uint2 scw = lds64(tile + kTileBytes + 8 * g);
                    int dl[NB][4], dh[NB][4];
                    uint32_t X[NB][8];
#pragma unroll
                    for (int nb = 0; nb < NB; nb++) {
                        const bool v = g + 8 * nb < 2 * B;
                        const uint32_t xa = v ? xs + (g + 8 * nb) * cs + (uint32_t)kb * 128u + 32u * t : zero;
                        const uint4 v0 = lds128(xa), v1 = lds128(v ? xa + 16 : zero + 16);
                        X[nb][0] = v0.x, X[nb][1] = v0.y, X[nb][2] = v0.z, X[nb][3] = v0.w;
                        X[nb][4] = v1.x, X[nb][5] = v1.y, X[nb][6] = v1.z, X[nb][7] = v1.w;
                        dl[nb][0] = dl[nb][1] = dl[nb][2] = dl[nb][3] = 0;
                        dh[nb][0] = dh[nb][1] = dh[nb][2] = dh[nb][3] = 0;
                    }
                    const uint32_t ra[4] = {wa.x, wa.y, wa.z, wa.w};
                    const uint32_t rbw[4] = {wb.x, wb.y, wb.z, wb.w};
#pragma unroll
                    for (int j = 0; j < 2; j++) {
                        const uint32_t a0 = ra[2 * j] & 0x0F0F0F0Fu, a1 = rbw[2 * j] & 0x0F0F0F0Fu;
                        const uint32_t a2 = ra[2 * j + 1] & 0x0F0F0F0Fu, a3 = rbw[2 * j + 1] & 0x0F0F0F0Fu;
                        const uint32_t h0 = ra[2 * j] & 0xF0F0F0F0u, h1 = rbw[2 * j] & 0xF0F0F0F0u;
                        const uint32_t h2 = ra[2 * j + 1] & 0xF0F0F0F0u, h3 = rbw[2 * j + 1] & 0xF0F0F0F0u;
#pragma unroll
                        for (int nb = 0; nb < NB; nb++) {
                            imma_16832_u8s8(dl[nb], a0, a1, a2, a3, X[nb][4 * j], X[nb][4 * j + 2]);
                            imma_16832_u8s8(dh[nb], h0, h1, h2, h3, X[nb][4 * j + 1], X[nb][4 * j + 3]);
                        }
                    }
                    const float2 s0 = __half22float2(*reinterpret_cast<const __half2*>(&scw.x));
                    const float2 s1 = __half22float2(*reinterpret_cast<const __half2*>(&scw.y));
#pragma unroll
                    for (int nb = 0; nb < NB; nb++) {
                        const int b = t + 4 * nb;
                        if (b < B) {
                            const float2 m = xms[b * P.nxr + kb];
                            const float sx = m.x * 0.0625f;  // S below is 16 * sum q X
                            const int S0 = (dl[nb][0] * 16 + dh[nb][0]) * 128 + (dl[nb][1] * 16 + dh[nb][1]);
                            const int S1 = (dl[nb][2] * 16 + dh[nb][2]) * 128 + (dl[nb][3] * 16 + dh[nb][3]);
                            acc[nb][0] = fmaf(s0.x, (float)S0 * sx, fmaf(s0.y, m.y, acc[nb][0]));
                            acc[nb][1] = fmaf(s1.x, (float)S1 * sx, fmaf(s1.y, m.y, acc[nb][1]));
                        }
                    }
                } else if (KIND == kKindI8) {
                    uint32_t X[NB][4];
                    int d[NB][4];
#pragma unroll
                    for (int nb = 0; nb < NB; nb++) {
                        const bool v = g + 8 * nb < 2 * B;
                        const uint4 v0 = lds128(v ? xs + (g + 8 * nb) * cs + (uint32_t)kb * 64u + 16u * t : zero);
                        X[nb][0] = v0.x, X[nb][1] = v0.y, X[nb][2] = v0.z, X[nb][3] = v0.w;
                        d[nb][0] = d[nb][1] = d[nb][2] = d[nb][3] = 0;
                    }
                    const uint32_t ra[4] = {wa.x, wa.y, wa.z, wa.w};
                    const uint32_t rbw[4] = {wb.x, wb.y, wb.z, wb.w};
#pragma unroll
                    for (int mm = 0; mm < 2; mm++)
#pragma unroll
                        for (int nb = 0; nb < NB; nb++)
                            imma_16832_s8s8(d[nb], ra[2 * mm], rbw[2 * mm], ra[2 * mm + 1], rbw[2 * mm + 1],
                                            X[nb][2 * mm], X[nb][2 * mm + 1]);
                    const int xbl = (kb * 64) / kXBlock;
#pragma unroll
                    for (int nb = 0; nb < NB; nb++) {
                        const int b = t + 4 * nb;
                        if (b < B) {
                            const float sx = xms[b * P.nxr + xbl].x;
                            acc[nb][0] = fmaf((float)(d[nb][0] * 128 + d[nb][1]), sx, acc[nb][0]);
                            acc[nb][1] = fmaf((float)(d[nb][2] * 128 + d[nb][3]), sx, acc[nb][1]);
                        }
                    }
                } else {
#pragma unroll
                    for (int nb = 0; nb < NB; nb++) {
                        const bool v = g + 8 * nb < 2 * B;
                        const uint4 v0 =
                            lds128(v ? xs + (g + 8 * nb) * cs + ((uint32_t)kb * 32u + 8u * t) * 2u : zero);
                        mma_16816(fd[nb], wa.x, wb.x, wa.y, wb.y, v0.x, v0.y);
                        mma_16816(fd[nb], wa.z, wb.z, wa.w, wb.w, v0.z, v0.w);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty(s));  // this warp is done with the stage
        }
        if (KIND == kKindF16) {
#pragma unroll
            for (int nb = 0; nb < NB; nb++) {
                acc[nb][0] = fd[nb][0] + fd[nb][1];  // hi + lo column of batch row t + 4 nb
                acc[nb][1] = fd[nb][2] + fd[nb][3];
            }
        }
        // this warp's partial of the row tile (lane t holds batch rows t, t + 4)
        float* rw = red + (p * kSW + warp) * 128;
#pragma unroll
        for (int nb = 0; nb < NB; nb++) {
            const int b = t + 4 * nb;
            if (b < B) {
                rw[g * 8 + b] = acc[nb][0];
                rw[(g + 8) * 8 + b] = acc[nb][1];
            }
        }
        // outlier correction of this warp's rows 2 warp, 2 warp + 1 (16 lanes each): the entries
        // whose column lies in the k range this CTA covered of the row tile
        if (has_out) {
            const bool eok = stream_wait(ebar(p), (ni >> 1) & 1, s_abort, a.err);
            const int half = lane >> 4, sub = lane & 15;
            const uint32_t eb = half ? rb1 : rb0, ee = half ? rb2 : rb1;
            const int c0 = ka * KB, c1 = kz * KB;
            const uint2* es = ent_s + p * kSEntCap;
            float o[8];
#pragma unroll
            for (int b = 0; b < 8; b++) o[b] = 0.f;
            if (eok) {
                for (uint32_t e = eb + sub; e < ee; e += 16) {
                    const uint32_t ei = e - elo;
                    const uint2 en = ei < (uint32_t)kSEntCap ? es[ei] : __ldg(a.ent + e);
                    const int col = (int)en.x;
                    if (col >= c0 && col < c1) {
                        const float corr = __uint_as_float(en.y);
#pragma unroll
                        for (int b = 0; b < 8; b++) {
                            if (b < B) {
                                const int X = (int)(int8_t)smem[P.xs + (2 * b) * cs + col] * 128 +
                                              (int)(int8_t)smem[P.xs + (2 * b + 1) * cs + col];
                                o[b] = fmaf(corr, (float)X * xms[b * P.nxr + col / kXBlock].x, o[b]);
                            }
                        }
                    }
                }
            }
#pragma unroll
            for (int b = 0; b < 8; b++) {
                if (b < B) {
#pragma unroll
                    for (int off = 8; off > 0; off >>= 1) o[b] += __shfl_xor_sync(0xffffffffu, o[b], off);
                    if (sub == 0) ocorr[p * 128 + (2 * warp + half) * 8 + b] = o[b];
                }
            }
        }
        consumer_sync();  // the row tile's partials (and corrections) are in shared memory
        if (has_out && tid == 0) mbar_arrive(efree(p));
        // sum over warps in warp order; a whole row tile is written, a split one goes through the ticket
        const int rr = tid >> 3, bb = tid & 7, row = T * 16 + rr;
        float val = 0.f;
        if (tid < 128 && bb < B) {
            for (int w = 0; w < kSW; w++) val += red[(p * kSW + w) * 128 + tid];
            if (has_out) val += ocorr[p * 128 + tid];
        }
        if (ka == 0 && kz == nkb) {
            if (tid < 128 && bb < B && row < a.N) {
                const size_t o = (size_t)bb * a.N + row;
                a.y[o] = a.resid ? a.resid[o] + val * oscale : val * oscale;
            }
        } else {
            // split row tile: this CTA's partial is piece 0 (T is its first row tile, the CTA before
            // holds the rest) or piece 1 (T is its last; the next CTA holds the rest)
            const int piece = (T == T0 && ka > 0) ? 0 : 1;
            if (tid < 128) a.ws[((size_t)c * 2 + piece) * 128 + tid] = val;
            consumer_sync();  // every partial written before thread 0 publishes them (release below)
            if (tid == 0) {
                __threadfence();
                const int prev = atomicAdd(a.tickets + T, 1);
                *s_last = prev == 1;
                if (prev == 1) {
                    a.tickets[T] = 0;  // ready for the next launch
                    __threadfence();   // acquire: the other CTA's partial is visible below
                }
            }
            consumer_sync();
            if (*s_last) {
                const int cA = piece == 0 ? c - 1 : c;  // the CTA holding the row tile's first k blocks
                if (tid < 128 && bb < B && row < a.N) {
                    const float vA = __ldcg(a.ws + ((size_t)cA * 2 + 1) * 128 + tid);
                    const float vB = __ldcg(a.ws + ((size_t)(cA + 1) * 2 + 0) * 128 + tid);
                    const float v = vA + vB;
                    const size_t o = (size_t)bb * a.N + row;
                    a.y[o] = a.resid ? a.resid[o] + v * oscale : v * oscale;
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
static int stream_stages(int kind, int B, int K, bool outl) {
    const StreamPlan p0 = stream_plan(kind, B, K, outl, 0);
    const int per = kSW * kind_tile_bytes(kind) + 16;
    const int n = (stream_smem_budget() - p0.total) / per;
    return std::min(n, kStreamMaxStages);
}

bool gemv_stream_fits(int kind, int B, int K, bool outl) {
    return B >= 1 && B <= kMaxBatch && stream_stages(kind, B, K, outl) >= 3;
}

size_t gemv_stream_ws_bytes(int num_sms, int nT) {
    return (size_t)num_sms * 2 * 128 * sizeof(float) + (size_t)nT * sizeof(int);
}

template <int KIND, int BT>
static cudaError_t prepare_stream(int dev) {
    static std::mutex mu;
    static unsigned done_mask = 0;
    std::lock_guard<std::mutex> lk(mu);
    if (dev < 32 && ((done_mask >> dev) & 1u)) return cudaSuccess;
    const cudaError_t e = cudaFuncSetAttribute(gemv_stream_kernel<KIND, BT>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, kStreamSmemMax);
    if (e == cudaSuccess && dev < 32) done_mask |= 1u << dev;
    return e;
}

template <int KIND, int BT>
static cudaError_t launch_stream_t(const StreamArgs& in, int num_sms, bool pdl, cudaStream_t st) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaError_t e = prepare_stream<KIND, BT>(dev);
    if (e != cudaSuccess) return e;
    const bool outl = KIND == kKindI4 && in.row_ptr != nullptr;
    const int nst = stream_stages(KIND, in.B, in.K, outl);
    if (nst < 3) return cudaErrorInvalidConfiguration;
    StreamArgs a = in;
    a.C = std::max(1, std::min(num_sms, a.nT));  // a slice holds at least one row tile's worth of tiles
    const StreamPlan P = stream_plan(KIND, in.B, in.K, outl, nst);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.C, 1, 1);
    cfg.blockDim = dim3(kSThreads, 1, 1);
    cfg.dynamicSmemBytes = P.total;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gemv_stream_kernel<KIND, BT>, a, nst);
}

template <int KIND>
static cudaError_t launch_stream_kind(const StreamArgs& a, int num_sms, bool pdl, cudaStream_t st) {
    switch (a.B) {
        case 1: return launch_stream_t<KIND, 1>(a, num_sms, pdl, st);
        case 2: return launch_stream_t<KIND, 2>(a, num_sms, pdl, st);
        case 3: return launch_stream_t<KIND, 3>(a, num_sms, pdl, st);
        case 4: return launch_stream_t<KIND, 4>(a, num_sms, pdl, st);
        default: return launch_stream_t<KIND, 8>(a, num_sms, pdl, st);
    }
}

cudaError_t launch_gemv_stream(int kind, const StreamArgs& a, int num_sms, bool pdl, cudaStream_t st) {
    if (a.B < 1 || a.B > kMaxBatch || a.nT < 1 || a.nkb < 1) return cudaErrorInvalidValue;
    if ((uintptr_t)a.x & 15) return cudaErrorInvalidValue;
    switch (kind) {
        case kKindI4: return launch_stream_kind<kKindI4>(a, num_sms, pdl, st);
        case kKindI8: return launch_stream_kind<kKindI8>(a, num_sms, pdl, st);
        default: return launch_stream_kind<kKindF16>(a, num_sms, pdl, st);
    }
}

}  // namespace pox
