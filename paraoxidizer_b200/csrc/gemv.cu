// gemv.cu -- weight-only quantized GEMV (INT4 affine groups, INT8 per-tensor, F16) for the decode
// hot path on B200 (sm_100a), with the sparse outlier correction fused into the epilogue.
//
// Replaces quant::gemv_int4 / gemv_int8 (crates/paraoxidizer-quant/src/kernels.rs:177-255), the
// Metal gemv_int4_kernel (crates/paraoxidizer-runtime/src/metal_backend.rs:11-54) and the F16
// projection of project_tensor (crates/paraoxidizer-runtime/src/engine.rs:235-250).
//
// Design (HBM-bound at batch <= 8):
//  * x preparation (xprep_kernel): per 128-k block, x becomes a 15-bit fixed-point value split
//    into two exact int8 limbs (hi, lo) plus (block scale, block sum); F16 weights take x as an
//    exact f16 hi/lo pair instead.
//  * One CTA = one row tile (16 rows) x one k-split; its W warps stride over the tile's k-blocks
//    (tile kb = k0 + warp, + W, ...), so a CTA streams a contiguous byte range. Each warp loads
//    four 1 KiB tiles at a time with 128-bit non-allocating loads straight into registers; the
//    lane's bytes are already MMA A fragments (see TileLayout).
//  * INT4: mma.sync m16n8k32 u8 x s8 -> s32. Low nibbles (w & 0x0F0F0F0F) and high nibbles
//    (w & 0xF0F0F0F0 = 16 q) go to two MMAs, so unpacking costs one LOP3 per 4 weights. The
//    s32 results are exact; the per-group affine map is applied once per tile:
//    sum_c (min + q*scale) x_c = scale * sum_c q x_c + min * sum_c x_c.
//    INT8: m16n8k32 s8 x s8. F16: m16n8k16 f16 x f16 -> f32.
//  * x of the CTA's k-range is staged in shared memory; the prepared meta likewise.
//  * Outliers (values that replace the dequantized weight, kernels.rs:211-219) are a per-row
//    CSR of (col, v - dequant(q)); each row's entries are loaded before the main loop and
//    applied with x from shared memory after it, reduced in a fixed order.
//  * Warps reduce through shared memory in warp order; k-splits of one row tile form a thread
//    block cluster and reduce through distributed shared memory in rank order. Results are
//    deterministic; there is no global scratch and no atomic.
//  * Programmatic dependent launch: the first weight loads are issued before
//    griddepcontrol.wait, overlapping the x preparation kernel.
#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>

#include "common.cuh"
#include "gemv.cuh"

namespace pox {

// ------------------------------------------------------------------------------------------
// x preparation
// ------------------------------------------------------------------------------------------
size_t xprep_bytes(int kind, int K) {
    const size_t Kp = (size_t)((K + kXBlock - 1) / kXBlock) * kXBlock;
    const size_t cols = 2 * (size_t)kMaxBatch * Kp * (kind == kKindF16 ? 2 : 1);
    const size_t meta = (size_t)kMaxBatch * (((Kp / kXBlock) + 1) & ~(size_t)1) * sizeof(float2);
    return ((cols + 255) & ~(size_t)255) + meta;
}

XPrep xprep_view(void* scratch, int kind, int K) {
    XPrep v;
    v.Kp = ((K + kXBlock - 1) / kXBlock) * kXBlock;
    v.nxb = v.Kp / kXBlock;
    v.nxbs = (v.nxb + 1) & ~1;
    const size_t cols = 2 * (size_t)kMaxBatch * v.Kp * (kind == kKindF16 ? 2 : 1);
    v.cols = scratch;
    v.meta = reinterpret_cast<float2*>((char*)scratch + ((cols + 255) & ~(size_t)255));
    return v;
}


// One warp per (batch row, 128-k block); lane l covers k = 4l .. 4l+3 of the block.
__global__ void __launch_bounds__(256) xprep_int_kernel(const float* __restrict__ x, int B, int K, uint8_t* cols,
                                                        float2* meta, int Kp, int nxb, int nxbs, PrepOp op) {
    pdl_launch_dependents();
    pdl_wait();
    const int nwb = blockDim.x >> 5, wid0 = blockIdx.x * nwb;
    const int wid = wid0 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    __shared__ float s_inv[8];  // RMSNorm scales of the rows this block's warps cover (at most 8)
    const int b0 = wid0 / nxb;
    if (op.mode == kPrepNorm && wid0 < B * nxb)
        block_rms_inv(x, op.ld_x, K, op.eps, b0, min(B * nxb - 1, wid0 + nwb - 1) / nxb, s_inv);
    if (wid >= B * nxb) return;
    const int b = wid / nxb, blk = wid % nxb;
    const int k = blk * kXBlock + lane * 4;
    PrepRow r;
    r.x = x + (size_t)b * op.ld_x;
    r.up = op.up ? op.up + (size_t)b * op.ld_up : nullptr;
    r.inv = op.mode == kPrepNorm ? s_inv[b - b0] : 1.f;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (k < K) {
        v = *reinterpret_cast<const float4*>(r.x + k);  // K % 4 == 0 on this path
        v.x = prep_elem(op, r, k, v.x);
        v.y = prep_elem(op, r, k + 1, v.y);
        v.z = prep_elem(op, r, k + 2, v.z);
        v.w = prep_elem(op, r, k + 3, v.w);
    }
    float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float inv = m > 0.f ? (float)kXLimbMax / m : 0.f;
    int X[4] = {__float2int_rn(v.x * inv), __float2int_rn(v.y * inv), __float2int_rn(v.z * inv),
                __float2int_rn(v.w * inv)};
    uint32_t hi = 0, lo = 0;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int q = max(-kXLimbMax, min(kXLimbMax, X[i]));
        hi |= ((uint32_t)(q >> 7) & 0xFFu) << (8 * i);
        lo |= ((uint32_t)q & 0x7Fu) << (8 * i);
    }
    *reinterpret_cast<uint32_t*>(cols + (size_t)(2 * b) * Kp + k) = hi;
    *reinterpret_cast<uint32_t*>(cols + (size_t)(2 * b + 1) * Kp + k) = lo;
    const float s = warp_sum((v.x + v.y) + (v.z + v.w));
    if (lane == 0) meta[(size_t)b * nxbs + blk] = make_float2(m > 0.f ? m / (float)kXLimbMax : 0.f, s);
}

// One warp per (batch row, 64 elements); lane l covers 2 elements: hi = f16(x), lo = f16(x - hi).
__global__ void __launch_bounds__(256) xprep_f16_kernel(const float* __restrict__ x, int B, int K, __half* cols,
                                                        int Kp, PrepOp op) {
    pdl_launch_dependents();
    pdl_wait();
    const int per = Kp / 64;  // warps per row
    const int nwb = blockDim.x >> 5, wid0 = blockIdx.x * nwb;
    const int wid = wid0 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    __shared__ float s_inv[8];
    const int b0 = wid0 / per;
    if (op.mode == kPrepNorm && wid0 < B * per)
        block_rms_inv(x, op.ld_x, K, op.eps, b0, min(B * per - 1, wid0 + nwb - 1) / per, s_inv);
    if (wid >= B * per) return;
    const int b = wid / per, k = (wid % per) * 64 + 2 * lane;
    PrepRow r;
    r.x = x + (size_t)b * op.ld_x;
    r.up = op.up ? op.up + (size_t)b * op.ld_up : nullptr;
    r.inv = op.mode == kPrepNorm ? s_inv[b - b0] : 1.f;
    float2 v = make_float2(0.f, 0.f);
    if (k < K) {
        v = *reinterpret_cast<const float2*>(r.x + k);  // K % 32 == 0 on this path
        v.x = prep_elem(op, r, k, v.x);
        v.y = prep_elem(op, r, k + 1, v.y);
    }
    const __half h0 = __float2half_rn(v.x), h1 = __float2half_rn(v.y);
    const __half l0 = __float2half_rn(v.x - __half2float(h0)), l1 = __float2half_rn(v.y - __half2float(h1));
    *reinterpret_cast<__half2*>(cols + (size_t)(2 * b) * Kp + k) = __halves2half2(h0, h1);
    *reinterpret_cast<__half2*>(cols + (size_t)(2 * b + 1) * Kp + k) = __halves2half2(l0, l1);
}

cudaError_t launch_xprep(int kind, const float* x, int B, int K, const XPrep& xp, const PrepOp& op_in, bool pdl,
                         cudaStream_t st) {
    PrepOp op = op_in;
    if (op.ld_x == 0) op.ld_x = K;
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(256, 1, 1);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    if (kind == kKindF16) {
        const int warps = B * (xp.Kp / 64);
        cfg.gridDim = dim3((warps + 7) / 8, 1, 1);
        return cudaLaunchKernelEx(&cfg, xprep_f16_kernel, x, B, K, (__half*)xp.cols, xp.Kp, op);
    }
    const int warps = B * xp.nxb;
    cfg.gridDim = dim3((warps + 7) / 8, 1, 1);
    return cudaLaunchKernelEx(&cfg, xprep_int_kernel, x, B, K, (uint8_t*)xp.cols, xp.meta, xp.Kp, xp.nxb, xp.nxbs,
                              op);
}

// ------------------------------------------------------------------------------------------
// Tensor-core GEMV
// ------------------------------------------------------------------------------------------
// Shared-memory plan of a CTA (bytes):
//   [weight rings: W warps x kStages x (tile + INT4 scale words)] [ring mbarriers, x / entry mbarriers]
//   [x columns] [x meta] [warp partials] [outlier sums] [cluster partials] [outlier entries + row bounds]
//   [32 zero bytes]
// Staged x columns are padded so that 128-bit reads of neighbouring columns fall in different banks.
constexpr int kStages = 3;     // weight tiles in flight per warp (one 1 KiB tile per stage)
constexpr int kEntCap = 1024;  // outlier entries of a row tile staged in shared memory

struct SmemPlan {
    int kbr;                   // max k-blocks per CTA
    int cstride;               // bytes per staged x column
    int nxr;                   // x meta blocks per batch row (stride, even)
    int ring, bars, xs, xm, red, ocorr, part, ent, zero, total;  // byte offsets; total = size
};
__host__ __device__ inline SmemPlan smem_plan(int kind, int B, int W, int S, int nkb, bool outl) {
    SmemPlan p;
    const int KB = kind_kblock(kind), XB = kind == kKindF16 ? 2 : 1;
    const int tb = kind_tile_bytes(kind);
    p.kbr = (nkb + S - 1) / S;
    const int xr = p.kbr * KB * XB;
    p.cstride = ((xr + 127) & ~127) + (kind == kKindI4 ? 16 : 64);
    p.nxr = ((p.kbr * KB + kXBlock - 1) / kXBlock + 2 + 1) & ~1;
    int o = 0;
    p.ring = o; o += W * kStages * tb;
    p.bars = o; o += W * kStages * 8 + 16;
    p.xs = o;   o += (2 * B * p.cstride + 15) & ~15;
    p.xm = o;   o += kind == kKindF16 ? 0 : B * p.nxr * 8;
    p.red = o;  o += W * 128 * 4;
    p.ocorr = o; o += 128 * 4;
    p.part = o; o += 128 * 4;
    p.ent = o;  o += outl ? kEntCap * 8 + 32 * 4 : 0;
    p.zero = o; o += 32;
    p.total = o;
    return p;
}


// BT: exact batch 1..4, or 8 for a runtime batch of 5..8 (two MMA column blocks).
template <int KIND, int BT>
__global__ void __launch_bounds__(512, 2) gemv_tc_kernel(const GemvArgs a) {
    constexpr int KB = KIND == kKindI4 ? 128 : (KIND == kKindI8 ? 64 : 32);
    constexpr int XB = KIND == kKindF16 ? 2 : 1;
    constexpr int NB = BT > 4 ? 2 : 1;
    constexpr int G = (KIND == kKindI4 && BT <= 2) ? 2 : 1;  // tiles whose results share one MMA accumulator
    constexpr int SB = KIND == kKindI4 ? 64 : 0;
    constexpr int TB = kTileBytes + SB;  // staged bytes per tile
    extern __shared__ __align__(128) unsigned char smem[];

    const int B = BT > 4 ? a.B : BT;
    const int W = blockDim.x >> 5;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
    const int S = a.S, s = blockIdx.x, T = blockIdx.y;
    const int nkb = a.nkb;
    const int kb0 = (int)((long long)s * nkb / S), kb1 = (int)((long long)(s + 1) * nkb / S);
    const int k0 = kb0 * KB, k1 = kb1 * KB;
    const bool has_out = KIND == kKindI4 && a.row_ptr != nullptr;
    const SmemPlan P = smem_plan(KIND, B, W, S, nkb, has_out);
    const uint32_t sbase = smem_u32(smem);
    const uint32_t ring = sbase + P.ring + warp * kStages * TB;
    const uint32_t wbar = sbase + P.bars + warp * kStages * 8;
    const uint32_t xbar = sbase + P.bars + W * kStages * 8, ebar = xbar + 8;
    const uint32_t xs = sbase + P.xs, zero = sbase + P.zero;
    const int cs = P.cstride;
    const int xb0 = k0 / kXBlock, xb0a = xb0 & ~1;  // meta copies start on an even block (16 bytes)
    const float2* xms = reinterpret_cast<const float2*>(smem + P.xm);
    float* red = reinterpret_cast<float*>(smem + P.red);
    float* ocorr = reinterpret_cast<float*>(smem + P.ocorr);
    float* part = reinterpret_cast<float*>(smem + P.part);
    const uint2* ent_s = reinterpret_cast<const uint2*>(smem + P.ent);
    uint32_t* rp_s = reinterpret_cast<uint32_t*>(smem + P.ent + kEntCap * 8);

    // this warp's tiles: kb = kb0 + warp + i * W, i < nt
    const int nt = kb0 + warp < kb1 ? (kb1 - kb0 - warp + W - 1) / W : 0;
    const uint8_t* wsrc = a.w + ((size_t)T * nkb + kb0 + warp) * TB;
    const size_t wstep = (size_t)W * TB;

    if (lane == 0)
        for (int i = 0; i < kStages; i++) mbar_init(wbar + 8 * i, 1);
    if (tid == 0) {
        mbar_init(xbar, 1);
        mbar_init(ebar, 1);
    }
    if (tid < 8) reinterpret_cast<uint32_t*>(smem + P.zero)[tid] = 0u;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    __syncthreads();
    pdl_launch_dependents();

    // ---- weight ring: the first kStages tiles of this warp (immutable data: no dependency) ----
    auto issue = [&](int i) {  // lane 0 only
        const uint32_t st = ring + (i % kStages) * TB, bar = wbar + 8 * (i % kStages);
        mbar_expect_tx(bar, TB);
        bulk_g2s(st, wsrc + (size_t)i * wstep, TB, bar);  // INT4: nibbles and scale words in one copy
    };
    if (lane == 0)
        for (int i = 0; i < kStages && i < nt; i++) issue(i);

    // ---- outlier CSR bounds of the row tile (rows 16T..16T+15 are one contiguous entry range) ----
    uint32_t e_lo = 0, e_hi = 0, rpv = 0;
    if (has_out) {
        const int r0 = T * 16, r1 = min(T * 16 + 16, a.N);
        if (tid == 0) {
            e_lo = __ldg(a.row_ptr + r0);
            e_hi = __ldg(a.row_ptr + r1);
        }
        if (tid <= 16) rpv = __ldg(a.row_ptr + min(r0 + tid, r1));
    }

    // ---- x of this CTA's k-range, its meta and the outlier entries: bulk copies ----
    pdl_wait();
    if (tid == 0) {
        const unsigned char* xq = reinterpret_cast<const unsigned char*>(a.xq);
        const uint32_t xbytes = (uint32_t)((k1 - k0) * XB);
        const int nmeta = KIND == kKindF16 ? 0 : (((k1 + kXBlock - 1) / kXBlock - xb0a + 1) & ~1);
        mbar_expect_tx(xbar, 2 * B * xbytes + (uint32_t)(B * nmeta * 8));
        for (int c = 0; c < 2 * B; c++) bulk_g2s(xs + c * cs, xq + ((size_t)c * a.Kp + k0) * XB, xbytes, xbar);
        for (int b = 0; b < B && nmeta > 0; b++)
            bulk_g2s(sbase + P.xm + b * P.nxr * 8, a.xm + (size_t)b * a.nxbs + xb0a, nmeta * 8, xbar);
        if (has_out) {
            const uint32_t lo = e_lo & ~1u;
            const uint32_t n = min((e_hi - lo + 1) & ~1u, (uint32_t)kEntCap);  // entries buffer has 2 pad slots
            mbar_expect_tx(ebar, n * 8);
            if (n) bulk_g2s(sbase + P.ent, a.ent + lo, n * 8, ebar);
        }
    }
    bool ok = mbar_wait(xbar, 0);
    ok = __all_sync(0xffffffffu, ok);
    if (!ok && lane == 0) atomicOr(a.err, kErrWaitX);

    // ---- main loop: tiles from the ring, A fragments straight from the staged bytes ----
    float acc[NB][2];
    float fd[NB][4];
#pragma unroll
    for (int nb = 0; nb < NB; nb++) {
        acc[nb][0] = acc[nb][1] = 0.f;
        fd[nb][0] = fd[nb][1] = fd[nb][2] = fd[nb][3] = 0.f;
    }
    // column packing (INT4, batch 1-2): column 2*slot + limb, slot = u * BT + b for tile u of a group
    const int slot_g = g >> 1, u_g = slot_g / (BT > 4 ? 4 : BT), b_g = slot_g % (BT > 4 ? 4 : BT);
    const bool xg_valid = G == 2 ? (u_g < G) : (g < 2 * B);
    const int col_g = G == 2 ? 2 * b_g + (g & 1) : g;
    const int u_t = t / (BT > 4 ? 4 : BT), b_t = t % (BT > 4 ? 4 : BT);

    int i = 0, fail_at = 0;
    while (ok && i < nt) {
        uint4 wa[G], wb[G];
        uint2 scw = make_uint2(0u, 0u);
        int kbu[G];
#pragma unroll
        for (int u = 0; u < G; u++) {
            kbu[u] = kb0 + warp + (i + u) * W;
            wa[u] = wb[u] = make_uint4(0u, 0u, 0u, 0u);
            if (i + u < nt) {
                const int st = (i + u) % kStages;
                const bool w_ok = mbar_wait(wbar + 8 * st, ((i + u) / kStages) & 1);
                if (!__all_sync(0xffffffffu, w_ok)) {
                    ok = false;
                    fail_at = i + u;
                    break;
                }
                const uint32_t sa = ring + st * TB + lane * 16;
                wa[u] = lds128(sa);
                wb[u] = lds128(sa + 512);
                if (KIND == kKindI4 && (G == 1 || u == u_t)) scw = lds64(ring + st * TB + kTileBytes + 8 * g);
                __syncwarp();
                if (lane == 0 && i + u + kStages < nt) {
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // reads done before the refill
                    issue(i + u + kStages);
                }
            }
        }
        if (!ok) {
            if (lane == 0) atomicOr(a.err, kErrWaitRing);
            break;
        }
        if (KIND == kKindI4) {
            int dl[NB][4], dh[NB][4];
#pragma unroll
            for (int nb = 0; nb < NB; nb++)
#pragma unroll
                for (int q = 0; q < 4; q++) dl[nb][q] = dh[nb][q] = 0;
#pragma unroll
            for (int u = 0; u < G; u++) {
                uint32_t X[NB][8];
#pragma unroll
                for (int nb = 0; nb < NB; nb++) {
                    const bool v = G == 2 ? (xg_valid && u == u_g && i + u < nt) : (col_g + 8 * nb < 2 * B);
                    const uint32_t xa = v ? xs + (col_g + 8 * nb) * cs + (uint32_t)(kbu[u] - kb0) * 128u + 32u * t
                                          : zero;
                    const uint4 v0 = lds128(xa), v1 = lds128(v ? xa + 16 : zero + 16);
                    X[nb][0] = v0.x, X[nb][1] = v0.y, X[nb][2] = v0.z, X[nb][3] = v0.w;
                    X[nb][4] = v1.x, X[nb][5] = v1.y, X[nb][6] = v1.z, X[nb][7] = v1.w;
                }
                const uint32_t ra[4] = {wa[u].x, wa[u].y, wa[u].z, wa[u].w};
                const uint32_t rb[4] = {wb[u].x, wb[u].y, wb[u].z, wb[u].w};
#pragma unroll
                for (int j = 0; j < 2; j++) {
                    const uint32_t a0 = ra[2 * j] & 0x0F0F0F0Fu, a1 = rb[2 * j] & 0x0F0F0F0Fu;
                    const uint32_t a2 = ra[2 * j + 1] & 0x0F0F0F0Fu, a3 = rb[2 * j + 1] & 0x0F0F0F0Fu;
                    const uint32_t h0 = ra[2 * j] & 0xF0F0F0F0u, h1 = rb[2 * j] & 0xF0F0F0F0u;
                    const uint32_t h2 = ra[2 * j + 1] & 0xF0F0F0F0u, h3 = rb[2 * j + 1] & 0xF0F0F0F0u;
#pragma unroll
                    for (int nb = 0; nb < NB; nb++) {
                        imma_16832_u8s8(dl[nb], a0, a1, a2, a3, X[nb][4 * j], X[nb][4 * j + 2]);
                        imma_16832_u8s8(dh[nb], h0, h1, h2, h3, X[nb][4 * j + 1], X[nb][4 * j + 3]);
                    }
                }
            }
            // epilogue: lane t owns slot t (G == 2) or batch t (+4): tile u_t, batch b_t
            const bool ev = G == 2 ? (u_t < G && i + u_t < nt) : true;
            const int kbe = G == 2 ? (u_t == 0 ? kbu[0] : kbu[G - 1]) : kbu[0];
            const float2 s0 = __half22float2(*reinterpret_cast<const __half2*>(&scw.x));
            const float2 s1 = __half22float2(*reinterpret_cast<const __half2*>(&scw.y));
#pragma unroll
            for (int nb = 0; nb < NB; nb++) {
                const int b = G == 2 ? b_t : t + 4 * nb;
                if (ev && b < B) {
                    const float2 m = xms[b * P.nxr + (kbe - xb0a)];
                    const float sx = m.x * 0.0625f;  // S below is 16 * sum q X
                    const int S0 = (dl[nb][0] * 16 + dh[nb][0]) * 128 + (dl[nb][1] * 16 + dh[nb][1]);
                    const int S1 = (dl[nb][2] * 16 + dh[nb][2]) * 128 + (dl[nb][3] * 16 + dh[nb][3]);
                    acc[nb][0] = fmaf(s0.x, (float)S0 * sx, fmaf(s0.y, m.y, acc[nb][0]));
                    acc[nb][1] = fmaf(s1.x, (float)S1 * sx, fmaf(s1.y, m.y, acc[nb][1]));
                }
            }
        } else if (KIND == kKindI8) {
            uint32_t X[NB][4];
#pragma unroll
            for (int nb = 0; nb < NB; nb++) {
                const bool v = g + 8 * nb < 2 * B;
                const uint4 v0 = lds128(v ? xs + (g + 8 * nb) * cs + (uint32_t)(kbu[0] - kb0) * 64u + 16u * t : zero);
                X[nb][0] = v0.x, X[nb][1] = v0.y, X[nb][2] = v0.z, X[nb][3] = v0.w;
            }
            int d[NB][4];
#pragma unroll
            for (int nb = 0; nb < NB; nb++) d[nb][0] = d[nb][1] = d[nb][2] = d[nb][3] = 0;
            const uint32_t ra[4] = {wa[0].x, wa[0].y, wa[0].z, wa[0].w};
            const uint32_t rb[4] = {wb[0].x, wb[0].y, wb[0].z, wb[0].w};
#pragma unroll
            for (int m = 0; m < 2; m++)
#pragma unroll
                for (int nb = 0; nb < NB; nb++)
                    imma_16832_s8s8(d[nb], ra[2 * m], rb[2 * m], ra[2 * m + 1], rb[2 * m + 1], X[nb][2 * m],
                                    X[nb][2 * m + 1]);
            const int xbl = (kbu[0] * 64) / kXBlock - xb0a;
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
                    lds128(v ? xs + (g + 8 * nb) * cs + ((uint32_t)(kbu[0] - kb0) * 32u + 8u * t) * 2u : zero);
                mma_16816(fd[nb], wa[0].x, wb[0].x, wa[0].y, wb[0].y, v0.x, v0.y);
                mma_16816(fd[nb], wa[0].z, wb[0].z, wa[0].w, wb[0].w, v0.z, v0.w);
            }
        }
        i += G;
    }
    if (!ok && lane == 0) {
        // never leave with copies in flight into this warp's ring: bounded waits on what was issued
        const int issued = min(nt, fail_at + kStages);
        for (int j = fail_at; j < issued; j++) mbar_wait(wbar + 8 * (j % kStages), (j / kStages) & 1);
    }
    if (KIND == kKindF16) {
#pragma unroll
        for (int nb = 0; nb < NB; nb++) {
            acc[nb][0] = fd[nb][0] + fd[nb][1];  // hi + lo column of batch row t + 4 nb
            acc[nb][1] = fd[nb][2] + fd[nb][3];
        }
    }
    if (G == 2) {
        // BT == 1: lanes t = 0, 1 hold tiles 0, 1 of batch 0; BT == 2: lanes t, t ^ 2 hold batch t & 1
        const int off = BT == 1 ? 1 : 2;
        acc[0][0] += __shfl_xor_sync(0xffffffffu, acc[0][0], off);
        acc[0][1] += __shfl_xor_sync(0xffffffffu, acc[0][1], off);
    }

    // ---- warp partials -> shared memory ----
    float* rw = red + warp * 128;
#pragma unroll
    for (int nb = 0; nb < NB; nb++) {
        const int b = G == 2 ? b_t : t + 4 * nb;
        const bool own = G == 2 ? (t < BT) : true;
        if (own && b < B) {
            rw[g * 8 + b] = acc[nb][0];
            rw[(g + 8) * 8 + b] = acc[nb][1];
        }
    }
    if (has_out && tid <= 16) rp_s[tid] = rpv;
    __syncthreads();

    // ---- outlier correction: sum over the row's entries of (v - dequant(q)) * x[col] ----
    if (has_out) {
        const bool eok = __all_sync(0xffffffffu, mbar_wait(ebar, 0));  // always: no copy left in flight
        if (!eok && lane == 0) atomicOr(a.err, kErrWaitEnt);
        const int tpr = 2 * W;  // threads per row: aligned lane groups of 8, 16 or 32
        const int ri = tid / tpr, sub = tid % tpr;
        const uint32_t lo = rp_s[0] & ~1u;  // the entry copy starts on an even index (16 bytes)
        const uint32_t rb = rp_s[ri] - lo, re = rp_s[ri + 1] - lo;
        float o[NB * 4];
#pragma unroll
        for (int b = 0; b < NB * 4; b++) o[b] = 0.f;
        if (ok && eok) {
            for (uint32_t e = rb + sub; e < re; e += tpr) {
                const uint2 en = e < (uint32_t)kEntCap ? ent_s[e] : __ldg(a.ent + lo + e);
                const int col = (int)en.x;
                if (col >= k0 && col < k1) {
                    const int kk = col - k0;
                    const int xbl = col / kXBlock - xb0a;
                    const float corr = __uint_as_float(en.y);
#pragma unroll
                    for (int b = 0; b < NB * 4; b++) {
                        if (b < B) {
                            const int X = (int)(int8_t)smem[P.xs + (2 * b) * cs + kk] * 128 +
                                          (int)(int8_t)smem[P.xs + (2 * b + 1) * cs + kk];
                            o[b] = fmaf(corr, (float)X * xms[b * P.nxr + xbl].x, o[b]);
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int b = 0; b < NB * 4; b++) {
            if (b < B) {
                for (int off = tpr >> 1; off > 0; off >>= 1) o[b] += __shfl_xor_sync(0xffffffffu, o[b], off);
                if (sub == 0) ocorr[ri * 8 + b] = o[b];
            }
        }
        __syncthreads();
    }

    // ---- reduction: warps in order, then k-splits (cluster ranks) in order ----
    const int rr = tid >> 3, bb = tid & 7;
    float p = 0.f;
    if (tid < 128 && bb < B) {
        for (int w = 0; w < W; w++) p += red[w * 128 + tid];
        if (has_out) p += ocorr[tid];
    }
    const float oscale = KIND == kKindI8 ? a.i8_scale : 1.f;
    const int row = T * 16 + rr;
    if (S == 1) {
        if (tid < 128 && bb < B && row < a.N) {
            const size_t o = (size_t)bb * a.N + row;
            const float os = KIND == kKindI8 && a.row_scale ? a.row_scale[row] : oscale;
            a.y[o] = a.resid ? a.resid[o] + p * os : p * os;
        }
    } else {
        if (tid < 128) part[tid] = p;
        cluster_sync_all();
        if (s == 0 && tid < 128 && bb < B) {
            for (int r = 1; r < S; r++) p += ld_dsmem_f32(part + tid, (uint32_t)r);
            if (row < a.N) {
                const size_t o = (size_t)bb * a.N + row;
                const float os = KIND == kKindI8 && a.row_scale ? a.row_scale[row] : oscale;
                a.y[o] = a.resid ? a.resid[o] + p * os : p * os;
            }
        }
        cluster_sync_all();  // remote shared memory stays valid until rank 0 has read it
    }
}

// ---- host-side planning ----
static int num_sms() {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
}

template <int KIND, int BT>
static cudaError_t prepare_kernel(int dev) {
    static std::mutex mu;
    static unsigned done_mask = 0;  // devices whose attribute is set (device ids < 32)
    std::lock_guard<std::mutex> lk(mu);
    if (dev < 32 && ((done_mask >> dev) & 1u)) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(gemv_tc_kernel<KIND, BT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         227 * 1024);
    if (e == cudaSuccess && dev < 32) done_mask |= 1u << dev;
    return e;
}

template <int KIND, int BT>
static int occupancy(int W, int smem) {
    static std::mutex mu;
    static std::map<std::tuple<int, int, int>, int> cache;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(mu);
    auto key = std::make_tuple(dev, W, smem);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, gemv_tc_kernel<KIND, BT>, W * 32, smem) != cudaSuccess) {
        cudaGetLastError();
        n = 0;
    }
    cache[key] = n;
    return n;
}

struct GemvPlan {
    int W = 0, S = 0, smem = 0;
};

// Chooses warps per CTA (W) and k-splits per row tile (S, a thread block cluster): all CTAs
// resident in one wave if possible, enough warps in flight, few splits, several tiles per warp.
template <int KIND, int BT>
static GemvPlan plan_gemv(int nT, int nkb, int B, bool outl) {
    const int sms = num_sms();
    GemvPlan best;
    double best_score = -1.0;
    for (int S : {1, 2, 4, 8}) {
        if (S > nkb) break;
        const int kbr = (nkb + S - 1) / S;
        for (int W : {16, 8, 4}) {
            if (W > kbr && W != 4) continue;  // keep every warp busy (the smallest CTA excepted)
            const SmemPlan sp = smem_plan(KIND, B, W, S, nkb, outl);
            if (sp.total > 227 * 1024) continue;
            const int occ = occupancy<KIND, BT>(W, sp.total);
            if (occ <= 0) continue;
            const long long ctas = (long long)nT * S, slots = (long long)occ * sms;
            const long long waves = (ctas + slots - 1) / slots;
            const double eff_w = waves == 1 ? 1.0 : (double)ctas / (double)(waves * slots);
            const double active = (double)std::min(ctas, slots) * W;
            const double eff_p = std::min(1.0, active / 2500.0);
            const double tpw = (double)kbr / W;
            const double eff_o = tpw / (tpw + 1.0);
            double pen = 1.0;
            for (int q = S; q > 1; q >>= 1) pen *= 0.97;
            const double score = eff_w * eff_p * eff_o * pen;
            if (score > best_score) {
                best_score = score;
                best.W = W;
                best.S = S;
                best.smem = sp.total;
            }
        }
    }
    return best;
}

template <int KIND, int BT>
static cudaError_t launch_tc_t(const GemvArgs& in, bool pdl, cudaStream_t st) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaError_t e = prepare_kernel<KIND, BT>(dev);
    if (e != cudaSuccess) return e;
    if (in.nT > 65535) return cudaErrorInvalidConfiguration;
    const GemvPlan pl = plan_gemv<KIND, BT>(in.nT, in.nkb, in.B, KIND == kKindI4 && in.row_ptr != nullptr);
    if (pl.W == 0) return cudaErrorInvalidConfiguration;
    GemvArgs a = in;
    a.S = pl.S;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(pl.S, in.nT, 1);
    cfg.blockDim = dim3(pl.W * 32, 1, 1);
    cfg.dynamicSmemBytes = pl.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (pdl) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        na++;
    }
    if (pl.S > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = pl.S;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = 1;
        na++;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, gemv_tc_kernel<KIND, BT>, a);
}

template <int KIND>
static cudaError_t launch_tc_kind(const GemvArgs& a, bool pdl, cudaStream_t st) {
    switch (a.B) {
        case 1: return launch_tc_t<KIND, 1>(a, pdl, st);
        case 2: return launch_tc_t<KIND, 2>(a, pdl, st);
        case 3: return launch_tc_t<KIND, 3>(a, pdl, st);
        case 4: return launch_tc_t<KIND, 4>(a, pdl, st);
        default: return launch_tc_t<KIND, 8>(a, pdl, st);
    }
}

cudaError_t launch_gemv_tc(int kind, const GemvArgs& a, bool pdl, cudaStream_t st) {
    if (a.B < 1 || a.B > kMaxBatch) return cudaErrorInvalidValue;
    switch (kind) {
        case kKindI4: return launch_tc_kind<kKindI4>(a, pdl, st);
        case kKindI8: return launch_tc_kind<kKindI8>(a, pdl, st);
        default: return launch_tc_kind<kKindF16>(a, pdl, st);
    }
}

// ------------------------------------------------------------------------------------------
// Generic kernels over the raw .pox layout, for shapes the tiled path does not take
// (group sizes that are not a multiple of 128, cols not a multiple of the k-block).
// One warp per row; exact dequantized values (mul then add, no FMA) times x in f32.
// ------------------------------------------------------------------------------------------
__global__ void gemv_i4_generic_kernel(GemvGenericArgs a) {
    const int warps = blockDim.x >> 5;
    const int row = blockIdx.x * warps + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= a.N) return;
    const uint8_t* prow = a.raw + (size_t)row * ((a.K + 1) / 2);
    const uint8_t* srow = a.raw_scales + (size_t)row * a.groups * 4;
    for (int b = 0; b < a.B; b++) {
        float s = 0.f;
        for (int c = lane; c < a.K; c += 32) {
            const int grp = c / a.gs;
            const uint32_t sm = (uint32_t)srow[grp * 4] | ((uint32_t)srow[grp * 4 + 1] << 8) |
                                ((uint32_t)srow[grp * 4 + 2] << 16) | ((uint32_t)srow[grp * 4 + 3] << 24);
            const float sc = half_bits_to_float(sm), mn = half_bits_to_float(sm >> 16);
            const uint8_t byte = prow[c >> 1];
            const uint32_t q = (c & 1) ? (byte >> 4) : (byte & 15);
            const float w = __fadd_rn(mn, __fmul_rn((float)q, sc));
            s = fmaf(w, a.x[(size_t)b * a.K + c], s);
        }
        s = warp_sum(s);
        if (a.row_ptr != nullptr) {
            float o = 0.f;
            for (uint32_t e = a.row_ptr[row] + lane; e < a.row_ptr[row + 1]; e += 32) {
                const uint2 en = a.entries[e];
                o = fmaf(__uint_as_float(en.y), a.x[(size_t)b * a.K + en.x], o);
            }
            s += warp_sum(o);
        }
        if (lane == 0) a.y[(size_t)b * a.N + row] = s;
    }
}

__global__ void gemv_i8_generic_kernel(GemvGenericArgs a) {
    const int warps = blockDim.x >> 5;
    const int row = blockIdx.x * warps + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= a.N) return;
    const int8_t* qrow = reinterpret_cast<const int8_t*>(a.raw) + (size_t)row * a.K;
    const float sc = a.row_scale ? a.row_scale[row] : a.i8_scale;
    for (int b = 0; b < a.B; b++) {
        float s = 0.f;
        for (int c = lane; c < a.K; c += 32)
            s = fmaf(__fmul_rn((float)qrow[c], sc), a.x[(size_t)b * a.K + c], s);
        s = warp_sum(s);
        if (lane == 0) a.y[(size_t)b * a.N + row] = s;
    }
}

__global__ void gemv_f16_generic_kernel(GemvGenericArgs a) {
    const int warps = blockDim.x >> 5;
    const int row = blockIdx.x * warps + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= a.N) return;
    const __half* wrow = reinterpret_cast<const __half*>(a.raw) + (size_t)row * a.K;
    for (int b = 0; b < a.B; b++) {
        float s = 0.f;
        for (int c = lane; c < a.K; c += 32) s = fmaf(__half2float(wrow[c]), a.x[(size_t)b * a.K + c], s);
        s = warp_sum(s);
        if (lane == 0) a.y[(size_t)b * a.N + row] = s;
    }
}

cudaError_t launch_gemv_generic(int kind, const GemvGenericArgs& a, cudaStream_t st) {
    const int warps = 8;
    dim3 grid((a.N + warps - 1) / warps);
    if (kind == kKindI4) gemv_i4_generic_kernel<<<grid, warps * 32, 0, st>>>(a);
    else if (kind == kKindI8) gemv_i8_generic_kernel<<<grid, warps * 32, 0, st>>>(a);
    else gemv_f16_generic_kernel<<<grid, warps * 32, 0, st>>>(a);
    return cudaGetLastError();
}

// ------------------------------------------------------------------------------------------
// Upload-time re-tiling. Output word o of the tile sequence decomposes as
// o = ((T * nkb + kb) * 2 + s) * 128 + lane * 4 + w, i.e. the byte layout of TileLayout.
// ------------------------------------------------------------------------------------------
template <int KIND>
__global__ void repack_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ out, TileLayout L,
                              size_t total) {
    for (size_t o = blockIdx.x * (size_t)blockDim.x + threadIdx.x; o < total; o += (size_t)gridDim.x * blockDim.x) {
        const int w = (int)(o & 3), lane = (int)((o >> 2) & 31), s = (int)((o >> 7) & 1);
        const size_t tile = o >> 8;
        const int T = (int)(tile / L.nkb), kb = (int)(tile % L.nkb);
        const int g = lane >> 2, t = lane & 3;
        const size_t row = (size_t)T * 16 + g + 8 * s;
        uint32_t word = 0;
        if (row < (size_t)L.N) {
            if (KIND == kKindI4) {
                // 8 nibbles k0..k0+7 (k0 = 128 kb + 32 t + 8 w): .pox byte j holds k 2j (low), 2j+1
                // (high); the tile byte i holds k0+i (low) and k0+4+i (high)
                const uint32_t v =
                    *reinterpret_cast<const uint32_t*>(src + row * (size_t)(L.K / 2) + (size_t)kb * 64 + 16 * t + 4 * w);
#pragma unroll
                for (int i = 0; i < 4; i++)
                    word |= (((v >> (4 * i)) & 15u) | (((v >> (4 * (i + 4))) & 15u) << 4)) << (8 * i);
            } else if (KIND == kKindI8) {
                word = *reinterpret_cast<const uint32_t*>(src + row * (size_t)L.K + (size_t)kb * 64 + 16 * t + 4 * w);
            } else {
                word = *reinterpret_cast<const uint32_t*>(src + (row * (size_t)L.K + (size_t)kb * 32 + 8 * t + 2 * w) * 2);
            }
        }
        *reinterpret_cast<uint32_t*>(out + tile * L.tb + (o & 255) * 4) = word;
    }
}

// INT4 scale words: word 2 g + s after the nibbles of tile (T, kb) = (f16 scale | f16 min << 16) of
// row 16 T + g + 8 s and the group holding k-block kb.
__global__ void repack_i4_scales_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ tiles, TileLayout L,
                                        int groups, int gs, size_t total) {
    for (size_t o = blockIdx.x * (size_t)blockDim.x + threadIdx.x; o < total; o += (size_t)gridDim.x * blockDim.x) {
        const int j = (int)(o & 15);
        const size_t tile = o >> 4;
        const int T = (int)(tile / L.nkb), kb = (int)(tile % L.nkb);
        const size_t row = (size_t)T * 16 + (j >> 1) + 8 * (j & 1);
        uint32_t v = 0;
        if (row < (size_t)L.N) {
            const int grp = kb * 128 / gs;
            v = *reinterpret_cast<const uint32_t*>(src + (row * groups + grp) * 4);
        }
        *reinterpret_cast<uint32_t*>(tiles + tile * L.tb + kTileBytes + j * 4) = v;
    }
}

// ------------------------------------------------------------------------------------------
// Dequantization (verification path): bit-exact with the reference (mul, then add).
// ------------------------------------------------------------------------------------------
__global__ void dequant_i4_tiled_kernel(const uint8_t* __restrict__ tiles, float* __restrict__ out, TileLayout L) {
    const size_t total = (size_t)L.N * L.K;
    for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total;
         idx += (size_t)gridDim.x * blockDim.x) {
        const size_t row = idx / L.K;
        const int k = (int)(idx % L.K);
        const int T = (int)(row / 16), ri = (int)(row % 16), g = ri & 7, s = ri >> 3;
        const int kb = k / 128, kin = k % 128, t = kin / 32, rem = kin % 32, w = rem / 8, p = rem % 8;
        const size_t tile = (size_t)T * L.nkb + kb;
        const uint8_t byte = tiles[tile * L.tb + s * 512 + (4 * g + t) * 16 + 4 * w + (p & 3)];
        const uint32_t q = (p < 4) ? (byte & 15u) : (byte >> 4);
        const uint32_t sm = *reinterpret_cast<const uint32_t*>(tiles + tile * L.tb + kTileBytes + (2 * g + s) * 4);
        const float scl = half_bits_to_float(sm), mn = half_bits_to_float(sm >> 16);
        out[idx] = __fadd_rn(mn, __fmul_rn((float)q, scl));
    }
}

__global__ void dequant_i4_raw_kernel(const uint8_t* __restrict__ raw, const uint8_t* __restrict__ scales,
                                      float* __restrict__ out, int N, int K, int groups, int gs) {
    const size_t total = (size_t)N * K;
    const size_t row_bytes = (size_t)(K + 1) / 2;
    for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total;
         idx += (size_t)gridDim.x * blockDim.x) {
        const size_t row = idx / K;
        const int c = (int)(idx % K);
        const int grp = c / gs;
        const uint8_t* p = scales + (row * groups + grp) * 4;
        const float sc = half_bits_to_float(p[0] | (p[1] << 8));
        const float mn = half_bits_to_float(p[2] | (p[3] << 8));
        const uint8_t byte = raw[row * row_bytes + (c >> 1)];
        const uint32_t q = (c & 1) ? (byte >> 4) : (byte & 15u);
        out[idx] = __fadd_rn(mn, __fmul_rn((float)q, sc));
    }
}

__global__ void dequant_i8_tiled_kernel(const uint8_t* __restrict__ tiles, float scale,
                                        const float* __restrict__ row_scale, float* __restrict__ out, TileLayout L) {
    const size_t total = (size_t)L.N * L.K;
    for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total;
         idx += (size_t)gridDim.x * blockDim.x) {
        const size_t row = idx / L.K;
        const int k = (int)(idx % L.K);
        const int T = (int)(row / 16), ri = (int)(row % 16), g = ri & 7, s = ri >> 3;
        const int kb = k / 64, kin = k % 64, t = kin / 16, j = kin % 16;
        const size_t tile = (size_t)T * L.nkb + kb;
        const int8_t q = (int8_t)tiles[tile * L.tb + s * 512 + (4 * g + t) * 16 + j];
        out[idx] = __fmul_rn((float)q, row_scale ? row_scale[row] : scale);
    }
}

__global__ void dequant_i8_raw_kernel(const uint8_t* __restrict__ raw, float scale, const float* __restrict__ row_scale,
                                      float* __restrict__ out, size_t total, int K) {
    for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total;
         idx += (size_t)gridDim.x * blockDim.x)
        out[idx] = __fmul_rn((float)(int8_t)raw[idx], row_scale ? row_scale[idx / K] : scale);
}

__global__ void apply_outliers_kernel(const uint32_t* __restrict__ row_ptr, const uint2* __restrict__ entries,
                                      const uint16_t* __restrict__ vals, float* __restrict__ out, int N, int K) {
    for (int row = blockIdx.x * blockDim.y + threadIdx.y; row < N; row += gridDim.x * blockDim.y) {
        for (uint32_t e = row_ptr[row] + threadIdx.x; e < row_ptr[row + 1]; e += blockDim.x)
            out[(size_t)row * K + entries[e].x] = half_bits_to_float(vals[e]);
    }
}

// ------------------------------------------------------------------------------------------
// Host-side launchers
// ------------------------------------------------------------------------------------------
static dim3 grid_for(size_t total) {
    size_t blocks = (total + 255) / 256;
    const size_t cap = (size_t)num_sms() * 32;
    if (blocks > cap) blocks = cap;
    if (blocks == 0) blocks = 1;
    return dim3((unsigned)blocks);
}

cudaError_t launch_repack(int kind, const uint8_t* src, uint8_t* tiles, int N, int K, cudaStream_t st) {
    const TileLayout L(kind, N, K);
    const size_t total = L.tiles() * 256;
    if (kind == kKindI4) repack_kernel<kKindI4><<<grid_for(total), 256, 0, st>>>(src, tiles, L, total);
    else if (kind == kKindI8) repack_kernel<kKindI8><<<grid_for(total), 256, 0, st>>>(src, tiles, L, total);
    else repack_kernel<kKindF16><<<grid_for(total), 256, 0, st>>>(src, tiles, L, total);
    return cudaGetLastError();
}

cudaError_t launch_repack_i4_scales(const uint8_t* src, uint8_t* tiles, int N, int K, int gs, cudaStream_t st) {
    const TileLayout L(kKindI4, N, K);
    const size_t total = L.tiles() * 16;
    const int groups = (K + gs - 1) / gs;
    repack_i4_scales_kernel<<<grid_for(total), 256, 0, st>>>(src, tiles, L, groups, gs, total);
    return cudaGetLastError();
}

cudaError_t launch_dequant_i4(bool tiled, const void* w, const void* scales, float* out, int N, int K, int groups,
                              int gs, cudaStream_t st) {
    const size_t total = (size_t)N * K;
    if (tiled)
        dequant_i4_tiled_kernel<<<grid_for(total), 256, 0, st>>>((const uint8_t*)w, out, TileLayout(kKindI4, N, K));
    else
        dequant_i4_raw_kernel<<<grid_for(total), 256, 0, st>>>((const uint8_t*)w, (const uint8_t*)scales, out, N, K,
                                                               groups, gs);
    return cudaGetLastError();
}

cudaError_t launch_dequant_i8(bool tiled, const void* w, float scale, const float* row_scale, float* out, int N, int K,
                              cudaStream_t st) {
    const size_t total = (size_t)N * K;
    if (tiled)
        dequant_i8_tiled_kernel<<<grid_for(total), 256, 0, st>>>((const uint8_t*)w, scale, row_scale, out,
                                                                 TileLayout(kKindI8, N, K));
    else
        dequant_i8_raw_kernel<<<grid_for(total), 256, 0, st>>>((const uint8_t*)w, scale, row_scale, out, total, K);
    return cudaGetLastError();
}

cudaError_t launch_apply_outliers(const uint32_t* row_ptr, const uint2* entries, const uint16_t* vals, float* out,
                                  int N, int K, cudaStream_t st) {
    dim3 block(32, 8);
    dim3 grid((N + 7) / 8 < 4096 ? (N + 7) / 8 : 4096);
    apply_outliers_kernel<<<grid, block, 0, st>>>(row_ptr, entries, vals, out, N, K);
    return cudaGetLastError();
}

}  // namespace pox
