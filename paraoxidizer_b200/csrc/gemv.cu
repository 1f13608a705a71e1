// gemv.cu -- weight-only quantized GEMV (INT4 affine groups, INT8 per-tensor, F16) for the decode
// hot path on B200 (sm_100a), with the sparse outlier correction fused into the epilogue.
//
// Replaces quant::gemv_int4 / gemv_int8 (crates/paraoxidizer-quant/src/kernels.rs:177-255), the
// Metal gemv_int4_kernel (crates/paraoxidizer-runtime/src/metal_backend.rs:11-54) and the F16
// projection of project_tensor (crates/paraoxidizer-runtime/src/engine.rs:235-250).
//
// Streaming design (HBM-bound at batch <= 8):
//  * Weights are re-tiled at upload into 1 KiB tiles (16 rows x one k-block) ordered
//    chunk-major, so the GEMV is one contiguous byte stream cut into items (one row tile x one
//    chunk of 8 k-blocks = 8 KiB). A persistent grid of one CTA per SM takes a contiguous range
//    of items.
//  * One producer thread streams the range with cp.async.bulk (TMA bulk copies) into a 16-stage
//    shared-memory ring, completion signalled on mbarriers; 8 consumer warps each own every 8th
//    item (two ring slots per warp: double buffering).
//  * Nibbles / int8 / f16 become exact f16 MMA A fragments in registers (exponent-bias trick);
//    mma.sync m16n8k16 does the q*x products with f32 accumulation. x (f32) enters as two f16
//    columns, hi = f16(x) and lo = f16(x - hi), so products keep ~22 bits of x.
//  * INT4: per 128-k block the MMA gives S = sum q*x; the epilogue adds scale*S + min*sum(x),
//    i.e. sum (min + q*scale) * x regrouped.
//  * Split-K partial sums go to a per-tensor scratch buffer; the warp that finishes the last
//    chunk of a row tile (atomic counter) sums the partials in chunk order (deterministic),
//    applies the outlier CSR correction y += sum (v - dequant(q)) * x[c] and writes y.
//  * Every mbarrier wait is bounded (clock64 budget): on expiry the kernel raises an error flag
//    and returns instead of hanging.
//  * Programmatic dependent launch: the producer starts streaming weights before the previous
//    kernel in the stream has finished; consumers wait (griddepcontrol.wait) before reading x.
#include <algorithm>

#include "common.cuh"
#include "gemv.cuh"

namespace pox {

template <int KIND>
struct KindTraits;
template <>
struct KindTraits<kKindI4> {
    static constexpr int KB = 128;
};
template <>
struct KindTraits<kKindI8> {
    static constexpr int KB = 64;
};
template <>
struct KindTraits<kKindF16> {
    static constexpr int KB = 32;
};

constexpr int kConsumerWarps = 8;
constexpr int kStreamThreads = (kConsumerWarps + 1) * 32;
constexpr int kItemBytes = kChunkTiles * kTileBytesL;  // 8 KiB
constexpr int kItemScaleBytes = kChunkTiles * 64;      // 512 B (INT4)
constexpr long long kWaitCycles = 4000000000LL;        // ~2 s at 2 GHz

// ---- PTX wrappers -------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
// Bounded wait on the phase of the given parity. false = the budget ran out.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    const long long t0 = clock64();
    for (;;) {
        uint32_t ok;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n"
            " selp.u32 %0, 1, 0, p;\n}"
            : "=r"(ok)
            : "r"(bar), "r"(parity)
            : "memory");
        if (ok) return true;
        if (clock64() - t0 > kWaitCycles) return false;
    }
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
            "r"(dst),
        "l"(src), "r"(bytes), "r"(bar), "l"(policy)
        : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 r;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(a));
    return r;
}
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t r;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(r) : "r"(a));
    return r;
}
__device__ __forceinline__ uint2 lds64a(uint32_t a) {
    uint2 r;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "r"(a));
    return r;
}
__device__ __forceinline__ void consumer_bar() { asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32)); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

constexpr int kGroupItems = 4;           // items per bulk copy (one ring group)
constexpr int kEntryCapG = 256;          // outlier entries staged per ring group (2 KiB)
constexpr int kXBlock = 128;             // k per x quantization block (integer path)
constexpr int kXLimbMax = 16383;         // |X| bound of the 15-bit x quantization

// Shared-memory plan of the streaming kernel (bytes). ring groups x kGroupItems blobs.
struct StreamSmem {
    size_t ring, ering, bars, meta, xs, xb, red, total;
    int xstride;  // bytes per staged x column
};
__host__ __device__ inline StreamSmem stream_smem(int kind, int B, int groups, int span) {
    StreamSmem s;
    const int ck = kChunkTiles * kind_kblock(kind);
    const size_t stride = (kind == kKindI4 ? kChunkTiles * 64 : 0) + (size_t)kChunkTiles * kTileBytesL;
    s.ring = (size_t)groups * kGroupItems * stride;
    s.ering = kind == kKindI4 ? (size_t)groups * kEntryCapG * 8 : 0;
    s.bars = (size_t)2 * groups * 8;
    s.meta = (size_t)groups * (kGroupItems + 1) * 8;
    if (kind == kKindF16) {
        s.xstride = (span * ck + 16) * 2;        // f16 hi / lo columns
        s.xs = (size_t)2 * B * s.xstride;
        s.xb = 0;
    } else {
        s.xstride = span * ck + 32;              // int8 hi / lo limb columns (permuted per 32 k)
        s.xs = ((size_t)2 * B * s.xstride + 15) & ~(size_t)15;
        s.xb = (size_t)2 * B * ((span * ck + kXBlock - 1) / kXBlock) * 4;  // per-block scale, sum(x)
    }
    s.red = (size_t)kConsumerWarps * 16 * kMaxBatch * 4;
    s.total = s.ring + s.ering + s.bars + s.meta + s.xs + s.xb + s.red;
    return s;
}

// Byte position of window offset kk inside a limb column: per 32 k, lane t's four k of each
// half (k 4t..4t+3 and 16+4t..16+4t+3) are adjacent, so one LDS.64 yields both B registers.
__device__ __forceinline__ int limb_pos(int kk) {
    const int r = kk & 31;
    return (kk & ~31) + 8 * ((r & 15) >> 2) + 4 * (r >> 4) + (r & 3);
}

// Reduction of one row tile by the warp that delivered its last chunk: partial sums of all
// chunks in chunk order (deterministic), written to y.
template <int KIND>
__device__ void reduce_row_tile(const StreamArgs& a, const TileLayout& L, int T) {
    const int lane = threadIdx.x & 31;
    const int B = a.B;
    for (int i = lane; i < 16 * B; i += 32) {
        const int ri = i / B, b = i % B;
        const int row = T * 16 + ri;
        const float* p = a.partial + ((size_t)T * L.nchunks * 16 + ri) * kMaxBatch + b;
        float s = 0.f;
#pragma unroll 8
        for (int c = 0; c < L.nchunks; c++) s += __ldcg(p + (size_t)c * 16 * kMaxBatch);
        if (row < a.N) a.y[(size_t)b * a.N + row] = KIND == kKindI8 ? s * a.i8_scale : s;
    }
    if (lane == 0) a.counters[T] = 0u;  // self-cleaning for the next launch
}

template <int KIND, int NB>
__global__ void __launch_bounds__(kStreamThreads, 1) gemv_stream_kernel(StreamArgs a) {
    constexpr int KB = KindTraits<KIND>::KB;
    constexpr int CK = kChunkTiles * KB;  // k per chunk
    constexpr int SB = KIND == kKindI4 ? kChunkTiles * 64 : 0;  // scale bytes leading a blob
    constexpr uint32_t STRIDE = SB + kChunkTiles * kTileBytesL;
    extern __shared__ __align__(128) unsigned char smem[];

    const TileLayout L(KIND, a.N, a.K);
    const int NG = a.ring;  // ring groups
    const int B = a.B;
    const StreamSmem sp = stream_smem(KIND, B, NG, a.span);
    unsigned char* ring = smem;
    uint2* ering = reinterpret_cast<uint2*>(smem + sp.ring);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + sp.ring + sp.ering);
    uint2* meta = reinterpret_cast<uint2*>(smem + sp.ring + sp.ering + sp.bars);  // [NG][kGroupItems+1]
    unsigned char* xs = smem + sp.ring + sp.ering + sp.bars + sp.meta;
    float* xblk = reinterpret_cast<float*>(smem + sp.ring + sp.ering + sp.bars + sp.meta + sp.xs);
    float* redall = reinterpret_cast<float*>(smem + sp.ring + sp.ering + sp.bars + sp.meta + sp.xs + sp.xb);

    const int items = L.items();
    const int G = gridDim.x;
    const int i0 = (int)((long long)blockIdx.x * items / G);
    const int i1 = (int)((long long)(blockIdx.x + 1) * items / G);
    const int n = i1 - i0;
    const int ngroups = (n + kGroupItems - 1) / kGroupItems;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + NG);
    const bool outl = KIND == kKindI4 && a.item_ptr != nullptr;

    if (tid == 0) {
        for (int s = 0; s < NG; s++) {
            mbar_init(full0 + 8 * s, 2);  // blob copy + outlier-entry copy
            mbar_init(empty0 + 8 * s, kGroupItems);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    pdl_launch_dependents();
    if (n <= 0) return;

    if (warp == kConsumerWarps) {
        // ---------------- producer warp: lane 0 issues the copies ----------------
        const uint64_t pol = policy_evict_first();
        auto issue_blobs = [&](int g) {
            const int gs = g % NG;
            const int m = min(kGroupItems, n - g * kGroupItems);
            const uint32_t bytes = (uint32_t)m * STRIDE;
            mbar_arrive_expect_tx(full0 + 8 * gs, bytes);
            bulk_g2s(smem_u32(ring + (size_t)gs * kGroupItems * STRIDE),
                     a.blobs + (size_t)(i0 + g * kGroupItems) * STRIDE, bytes, full0 + 8 * gs, pol);
        };
        // outlier offsets of items [i0, i1]: one warp-wide load per 32 items
        uint32_t ipv = 0;
        int ip_base = -1;
        auto ip_at = [&](int li) -> uint32_t {  // warp-collective, li in [0, n]
            const int base = li & ~31;
            if (base != ip_base) {
                ip_base = base;
                ipv = base + lane <= n ? __ldg(a.item_ptr + i0 + base + lane) : 0u;
            }
            return __shfl_sync(0xffffffffu, ipv, li & 31);
        };
        auto issue_entries = [&](int g) {  // warp-collective
            const int gs = g % NG;
            const int m = min(kGroupItems, n - g * kGroupItems);
            uint32_t e[kGroupItems + 1];
#pragma unroll
            for (int j = 0; j <= kGroupItems; j++) {
                const int li = g * kGroupItems + (j < m ? j : m);
                e[j] = outl ? ip_at(li) : 0u;
            }
            // li is clamped to the group's end, so e[j] == e[m] for j >= m
            if (lane == 0) {
                uint32_t bytes = 0, estart = e[0] & ~1u;
                if (outl && e[kGroupItems] > e[0]) {
                    uint32_t cnt = e[kGroupItems] - estart;
                    if (cnt > (uint32_t)kEntryCapG) cnt = kEntryCapG;
                    cnt = (cnt + 1) & ~1u;
                    bytes = cnt * 8;
                }
                uint2* mg = meta + gs * (kGroupItems + 1);
#pragma unroll
                for (int j = 0; j < kGroupItems; j++) mg[j] = make_uint2(e[j], e[j + 1]);
                mg[kGroupItems] = make_uint2(estart, estart + bytes / 8);
                if (bytes) {
                    mbar_arrive_expect_tx(full0 + 8 * gs, bytes);
                    bulk_g2s(smem_u32(ering + (size_t)gs * kEntryCapG), a.entries + estart, bytes, full0 + 8 * gs,
                             pol);
                } else {
                    mbar_arrive(full0 + 8 * gs);
                }
            }
        };
        int issued = 0;
        bool abort = false;
        const int first = min(NG, ngroups);
        if (lane == 0)
            for (int g = 0; g < first; g++) issue_blobs(g);  // weights first: no dependency
        for (int g = 0; g < first; g++) issue_entries(g);
        issued = first;
        for (int g = first; g < ngroups && !abort; g++) {
            int ok = 1;
            if (lane == 0) {
                if (!mbar_wait(empty0 + 8 * (g % NG), ((g / NG) - 1) & 1)) {
                    atomicOr(a.err, kErrTimeoutEmpty);
                    ok = 0;
                } else {
                    issue_blobs(g);
                }
            }
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) {
                abort = true;
                // the blob copy was not issued: complete the phase's entry arrival anyway so the
                // bounded drain below never waits on a half-armed barrier
                break;
            }
            issue_entries(g);
            issued = g + 1;
        }
        if (lane == 0) {
            // never leave with copies in flight: wait (bounded) for the last use of every group
            for (int g = issued - 1; g >= 0 && g >= issued - NG; g--) mbar_wait(full0 + 8 * (g % NG), (g / NG) & 1);
        }
        return;
    }

    // ---------------- consumers ----------------
    const int g = lane >> 2, t = lane & 3;
    const int c_first = i0 / L.nT, c_last = (i1 - 1) / L.nT;
    const int kw0 = c_first * CK;
    const int kw1 = min(a.K, (c_last + 1) * CK);
    const int kw = kw1 - kw0;
    pdl_wait();  // x (and the scratch of a previous launch) are visible from here on
    const int nxb = (kw + kXBlock - 1) / kXBlock;           // x blocks in the window
    const int xbs = (a.span * CK + kXBlock - 1) / kXBlock;  // x-block stride per limb column
    if (KIND == kKindF16) {
        for (int b = 0; b < B; b++) {
            const float* xb = a.x + (size_t)b * a.K + kw0;
            __half* hi = reinterpret_cast<__half*>(xs + (size_t)(2 * b) * sp.xstride);
            __half* lo = reinterpret_cast<__half*>(xs + (size_t)(2 * b + 1) * sp.xstride);
            for (int k = tid * 2; k < kw; k += kConsumerWarps * 64) {
                const float2 v = *reinterpret_cast<const float2*>(xb + k);
                const __half h0 = __float2half_rn(v.x), h1 = __float2half_rn(v.y);
                const __half l0 = __float2half_rn(v.x - __half2float(h0));
                const __half l1 = __float2half_rn(v.y - __half2float(h1));
                *reinterpret_cast<__half2*>(hi + k) = __halves2half2(h0, h1);
                *reinterpret_cast<__half2*>(lo + k) = __halves2half2(l0, l1);
            }
        }
    } else {
        // 15-bit quantization of x per 128-k block: X = rint(x * 16383 / max|x|) split into two
        // exact int8 limbs (X = 128 hi + lo); the integer MMAs then compute sum q*X exactly.
        for (int i = warp; i < B * nxb; i += kConsumerWarps) {
            const int b = i / nxb, bl = i % nxb;
            const int kk = bl * kXBlock + lane * 4;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (kk < kw) v = *reinterpret_cast<const float4*>(a.x + (size_t)b * a.K + kw0 + kk);
            float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            const float inv = m > 0.f ? (float)kXLimbMax / m : 0.f;
            const float sc = m > 0.f ? m / (float)kXLimbMax : 0.f;
            const int X0 = __float2int_rn(v.x * inv), X1 = __float2int_rn(v.y * inv);
            const int X2 = __float2int_rn(v.z * inv), X3 = __float2int_rn(v.w * inv);
            const uint32_t hi = ((uint32_t)(X0 >> 7) & 0xFFu) | (((uint32_t)(X1 >> 7) & 0xFFu) << 8) |
                                (((uint32_t)(X2 >> 7) & 0xFFu) << 16) | (((uint32_t)(X3 >> 7) & 0xFFu) << 24);
            const uint32_t lo = ((uint32_t)X0 & 0x7Fu) | (((uint32_t)X1 & 0x7Fu) << 8) | (((uint32_t)X2 & 0x7Fu) << 16) |
                                (((uint32_t)X3 & 0x7Fu) << 24);
            if (kk < kw) {
                const int pos = limb_pos(kk);
                *reinterpret_cast<uint32_t*>(xs + (size_t)(2 * b) * sp.xstride + pos) = hi;
                *reinterpret_cast<uint32_t*>(xs + (size_t)(2 * b + 1) * sp.xstride + pos) = lo;
            }
            float sum = (v.x + v.y) + (v.z + v.w);
            sum = warp_sum(sum);
            if (lane == 0) {
                xblk[(2 * b) * xbs + bl] = sc;
                xblk[(2 * b + 1) * xbs + bl] = sum;
            }
        }
    }
    consumer_bar();

    float* red = redall + warp * 16 * kMaxBatch;
    const uint32_t xs_base = smem_u32(xs);
    const int ncols = 2 * B;
    int done_items = 0;
    for (int i = warp; i < n; i += kConsumerWarps) {
        const int gi = i / kGroupItems, gs = gi % NG, j4 = i % kGroupItems;
        if (!mbar_wait(full0 + 8 * gs, (gi / NG) & 1)) {
            atomicOr(a.err, kErrTimeoutFull);
            break;
        }
        const int item = i0 + i;
        const int c = item / L.nT, T = item - c * L.nT;
        const int kc = L.kch(c);
        const uint32_t st = smem_u32(ring + ((size_t)gs * kGroupItems + j4) * STRIDE);
        uint4 ta[kChunkTiles], tb[kChunkTiles];
        uint32_t sg[kChunkTiles], sg8[kChunkTiles];
#pragma unroll
        for (int j = 0; j < kChunkTiles; j++) {
            if (j < kc) {
                ta[j] = lds128(st + SB + j * kTileBytesL + lane * 16);
                tb[j] = lds128(st + SB + j * kTileBytesL + 512 + lane * 16);
                if (KIND == kKindI4) {
                    sg[j] = lds32(st + j * 64 + g * 4);
                    sg8[j] = lds32(st + j * 64 + (g + 8) * 4);
                }
            }
        }
        // outlier entries of this item: staged in the group's entry buffer up to its end
        uint32_t e0 = 0, e1 = 0, es = 0, ee = 0;
        uint2 oen[2] = {make_uint2(0u, 0u), make_uint2(0u, 0u)};
        if (outl) {
            const uint2 mi = meta[gs * (kGroupItems + 1) + j4];
            const uint2 mg = meta[gs * (kGroupItems + 1) + kGroupItems];
            e0 = mi.x, e1 = mi.y, es = mg.x, ee = mg.y;
#pragma unroll
            for (int q = 0; q < 2; q++) {
                const uint32_t e = e0 + lane + 32u * q;
                if (e < e1 && e < ee) oen[q] = lds64a(smem_u32(ering + (size_t)gs * kEntryCapG + (e - es)));
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty0 + 8 * gs);  // the group refills once its items are read

        float acc[NB][2];
#pragma unroll
        for (int nb = 0; nb < NB; nb++) acc[nb][0] = acc[nb][1] = 0.f;
        float dacc[NB][4];
#pragma unroll
        for (int nb = 0; nb < NB; nb++) dacc[nb][0] = dacc[nb][1] = dacc[nb][2] = dacc[nb][3] = 0.f;
#pragma unroll
        for (int j = 0; j < kChunkTiles; j++) {
            if (j < kc) {
                const int kb = c * kChunkTiles + j;
                const int kk0 = kb * KB - kw0;  // window offset of this tile
                const uint32_t ra[4] = {ta[j].x, ta[j].y, ta[j].z, ta[j].w};
                const uint32_t rb[4] = {tb[j].x, tb[j].y, tb[j].z, tb[j].w};
                if (KIND == kKindF16) {
                    const uint32_t xk = xs_base + 2u * (uint32_t)(kk0 + 4 * t);
#pragma unroll
                    for (int jj = 0; jj < 2; jj++) {
#pragma unroll
                        for (int nb = 0; nb < NB; nb++) {
                            const int col = g + 8 * nb;
                            uint2 b0 = make_uint2(0u, 0u);
                            if (col < ncols) b0 = lds64a(xk + (uint32_t)(col * sp.xstride) + 2u * 16u * jj);
                            mma_16816(dacc[nb], ra[2 * jj], rb[2 * jj], ra[2 * jj + 1], rb[2 * jj + 1], b0.x, b0.y);
                        }
                    }
                } else {
                    int d[NB][4];
#pragma unroll
                    for (int nb = 0; nb < NB; nb++) d[nb][0] = d[nb][1] = d[nb][2] = d[nb][3] = 0;
                    constexpr int MM = KIND == kKindI4 ? 4 : 2;  // k32 MMAs per tile
#pragma unroll
                    for (int m = 0; m < MM; m++) {
                        uint32_t a0, a1, a2, a3;
                        if (KIND == kKindI4) {
                            a0 = ra[m] & 0x0F0F0F0Fu;
                            a1 = rb[m] & 0x0F0F0F0Fu;
                            a2 = (ra[m] >> 4) & 0x0F0F0F0Fu;
                            a3 = (rb[m] >> 4) & 0x0F0F0F0Fu;
                        } else {
                            a0 = ra[2 * m];
                            a1 = rb[2 * m];
                            a2 = ra[2 * m + 1];
                            a3 = rb[2 * m + 1];
                        }
                        const uint32_t xk = xs_base + (uint32_t)(kk0 + 32 * m + 8 * t);
#pragma unroll
                        for (int nb = 0; nb < NB; nb++) {
                            const int col = g + 8 * nb;
                            uint2 b0 = make_uint2(0u, 0u);
                            if (col < ncols) b0 = lds64a(xk + (uint32_t)(col * sp.xstride));
                            if (KIND == kKindI4) imma_16832_u8s8(d[nb], a0, a1, a2, a3, b0.x, b0.y);
                            else imma_16832_s8s8(d[nb], a0, a1, a2, a3, b0.x, b0.y);
                        }
                    }
                    const int bl = kk0 / kXBlock;
                    float fg = 1.f, fm = 0.f, fg8 = 1.f, fm8 = 0.f;
                    if (KIND == kKindI4) {
                        const float2 s0 = __half22float2(*reinterpret_cast<const __half2*>(&sg[j]));
                        const float2 s1 = __half22float2(*reinterpret_cast<const __half2*>(&sg8[j]));
                        fg = s0.x, fm = s0.y, fg8 = s1.x, fm8 = s1.y;
                    }
#pragma unroll
                    for (int nb = 0; nb < NB; nb++) {
                        const int b = t + 4 * nb;
                        if (b < B) {
                            const float sx = xblk[(2 * b) * xbs + bl];
                            const float S0 = (float)(d[nb][0] * 128 + d[nb][1]) * sx;
                            const float S1 = (float)(d[nb][2] * 128 + d[nb][3]) * sx;
                            if (KIND == kKindI4) {
                                const float sum = xblk[(2 * b + 1) * xbs + bl];
                                acc[nb][0] = fmaf(fg, S0, fmaf(fm, sum, acc[nb][0]));
                                acc[nb][1] = fmaf(fg8, S1, fmaf(fm8, sum, acc[nb][1]));
                            } else {
                                acc[nb][0] += S0;
                                acc[nb][1] += S1;
                            }
                        }
                    }
                }
            }
        }
        if (KIND == kKindF16) {
#pragma unroll
            for (int nb = 0; nb < NB; nb++) {
                acc[nb][0] = dacc[nb][0] + dacc[nb][1];
                acc[nb][1] = dacc[nb][2] + dacc[nb][3];
            }
        }
        // outlier correction of this item: sum (v - dequant(q)) * x[c], x from the limbs
        if (outl && e1 > e0) {
            for (int q = lane; q < 16 * kMaxBatch; q += 32) red[q] = 0.f;
            __syncwarp();
            for (uint32_t e = e0 + lane; e < e1; e += 32) {
                const uint32_t r = e - e0;
                uint2 en = r < 32u ? oen[0] : oen[1];
                if (r >= 64u || e >= ee) en = __ldg(a.entries + e);
                const int ri = (int)(en.x & 15u);
                const int kx = (int)(en.x >> 4) - kw0;
                const float corr = __uint_as_float(en.y);
                const int pos = limb_pos(kx);
                for (int b = 0; b < B; b++) {
                    const int X = (int)(int8_t)xs[(size_t)(2 * b) * sp.xstride + pos] * 128 +
                                  (int)(int8_t)xs[(size_t)(2 * b + 1) * sp.xstride + pos];
                    const float xv = (float)X * xblk[(2 * b) * xbs + kx / kXBlock];
                    atomicAdd(red + ri * kMaxBatch + b, corr * xv);
                }
            }
            __syncwarp();
#pragma unroll
            for (int nb = 0; nb < NB; nb++) {
                const int b = t + 4 * nb;
                if (b < B) {
                    acc[nb][0] += red[g * kMaxBatch + b];
                    acc[nb][1] += red[(g + 8) * kMaxBatch + b];
                }
            }
            __syncwarp();
        }
        // partial sums of this (row tile, chunk): fire-and-forget stores
        float* P = a.partial + ((size_t)T * L.nchunks + c) * 16 * kMaxBatch;
#pragma unroll
        for (int nb = 0; nb < NB; nb++) {
            const int b = t + 4 * nb;
            if (b < B) {
                __stcg(P + g * kMaxBatch + b, acc[nb][0]);
                __stcg(P + (g + 8) * kMaxBatch + b, acc[nb][1]);
            }
        }
        done_items++;
    }

    // ---- publish this warp's partials; the last contributor of a row tile reduces it ----
    __threadfence();
    __syncwarp();
    for (int j0 = 0; j0 < done_items; j0 += 32) {
        const int j = j0 + lane;
        bool last = false;
        int T = 0;
        if (j < done_items) {
            const int item = i0 + warp + kConsumerWarps * j;
            T = item % L.nT;
            last = atomicAdd(a.counters + T, 1u) == (unsigned)L.nchunks - 1;
        }
        unsigned m = __ballot_sync(0xffffffffu, last);
        if (m) __threadfence();
        while (m) {
            const int src = __ffs(m) - 1;
            m &= m - 1;
            reduce_row_tile<KIND>(a, L, __shfl_sync(0xffffffffu, T, src));
        }
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
    for (int b = 0; b < a.B; b++) {
        float s = 0.f;
        for (int c = lane; c < a.K; c += 32)
            s = fmaf(__fmul_rn((float)qrow[c], a.i8_scale), a.x[(size_t)b * a.K + c], s);
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

// ------------------------------------------------------------------------------------------
// Upload-time re-tiling into item blobs (one thread per output 32-bit word). Word o of the
// (T, kb)-ordered tile sequence: o = ((T * nkb + kb) * 2 + s) * 128 + lane * 4 + w
// (s = row half g / g+8, w = word of the lane's 16 bytes).
// ------------------------------------------------------------------------------------------
template <int KIND>
__global__ void repack_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ blobs, TileLayout L,
                              size_t total) {
    for (size_t o = blockIdx.x * (size_t)blockDim.x + threadIdx.x; o < total; o += (size_t)gridDim.x * blockDim.x) {
        const int w = (int)(o & 3), lane = (int)((o >> 2) & 31), s = (int)((o >> 7) & 1);
        const size_t tl = o >> 8;
        const int T = (int)(tl / L.nkb), kb = (int)(tl % L.nkb);
        const int g = lane >> 2, t = lane & 3;
        const size_t row = (size_t)T * 16 + g + 8 * s;
        uint32_t word = 0;
        if (row < (size_t)L.N) {
            if (KIND == kKindI4) {
                const size_t row_bytes = (size_t)(L.K + 1) / 2;
#pragma unroll
                for (int p = 0; p < 8; p++) {
                    // word w feeds the k32 MMA w: even nibbles are k 4t..4t+3 (A registers 0/1),
                    // odd nibbles k 16+4t..16+4t+3 (A registers 2/3); (v & 0x0F0F0F0F) and
                    // (v >> 4 & 0x0F0F0F0F) are then the u8 fragments
                    const int k = kb * 128 + 32 * w + ((p & 1) ? 16 : 0) + 4 * t + (p >> 1);
                    const uint8_t byte = src[row * row_bytes + (k >> 1)];
                    const uint32_t nib = (k & 1) ? (byte >> 4) : (byte & 15u);
                    word |= nib << (4 * p);
                }
            } else if (KIND == kKindI8) {
                // word 2m: k 32m+4t..+3, word 2m+1: k 32m+16+4t..+3 (s8 fragments of the k32 MMA m)
                const int k = kb * 64 + 16 * w + 4 * t;
                word = *reinterpret_cast<const uint32_t*>(src + row * L.K + k);
            } else {
                const int k = kb * 32 + 16 * (w >> 1) + 4 * t + 2 * (w & 1);
                word = *reinterpret_cast<const uint32_t*>(src + (row * L.K + k) * 2);
            }
        }
        *reinterpret_cast<uint32_t*>(blobs + L.tile_off(T, kb) + s * 512 + lane * 16 + w * 4) = word;
    }
}

// INT4 scales into the blobs: per tile 16 rows of (f16 scale | f16 min << 16); a group spanning
// several 128-k blocks is repeated in each.
__global__ void repack_i4_scales_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ blobs, TileLayout L,
                                        int groups, int gs, size_t total) {
    for (size_t o = blockIdx.x * (size_t)blockDim.x + threadIdx.x; o < total; o += (size_t)gridDim.x * blockDim.x) {
        const int ri = (int)(o & 15);
        const size_t tl = o >> 4;
        const int T = (int)(tl / L.nkb), kb = (int)(tl % L.nkb);
        const size_t row = (size_t)T * 16 + ri;
        uint32_t v = 0;
        if (row < (size_t)L.N) {
            const int grp = kb * 128 / gs;
            const uint8_t* p = src + (row * groups + grp) * 4;
            v = (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
        }
        *reinterpret_cast<uint32_t*>(blobs + L.scale_off(T, kb) + ri * 4) = v;
    }
}

// ------------------------------------------------------------------------------------------
// Dequantization (verification path): bit-exact with the reference.
// ------------------------------------------------------------------------------------------
__global__ void dequant_i4_tiled_kernel(const uint8_t* __restrict__ blobs, float* __restrict__ out, TileLayout L) {
    const size_t total = (size_t)L.N * L.K;
    for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total;
         idx += (size_t)gridDim.x * blockDim.x) {
        const size_t row = idx / L.K;
        const int k = (int)(idx % L.K);
        const int T = (int)(row / 16);
        const int ri = (int)(row % 16), g = ri & 7, s = ri >> 3;
        const int kb = k / 128, kin = k % 128;
        const int w = kin / 32, r = kin % 32, half = r >> 4, t = (r & 15) >> 2, i = r & 3;
        const int lane = g * 4 + t;
        const int p = 2 * i + half;
        const uint32_t word = *reinterpret_cast<const uint32_t*>(blobs + L.tile_off(T, kb) + s * 512 + lane * 16 + w * 4);
        const uint32_t q = (word >> (4 * p)) & 15u;
        const uint32_t sm = *reinterpret_cast<const uint32_t*>(blobs + L.scale_off(T, kb) + ri * 4);
        const float sc = half_bits_to_float(sm), mn = half_bits_to_float(sm >> 16);
        out[idx] = __fadd_rn(mn, __fmul_rn((float)q, sc));
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

__global__ void dequant_i8_tiled_kernel(const uint8_t* __restrict__ blobs, float scale, float* __restrict__ out,
                                        TileLayout L) {
    const size_t total = (size_t)L.N * L.K;
    for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total;
         idx += (size_t)gridDim.x * blockDim.x) {
        const size_t row = idx / L.K;
        const int k = (int)(idx % L.K);
        const int T = (int)(row / 16);
        const int ri = (int)(row % 16), g = ri & 7, s = ri >> 3;
        const int kb = k / 64, kin = k % 64;
        const int w = kin / 16, rem = kin % 16, t = rem / 4, kk = rem % 4;
        const int lane = g * 4 + t;
        const uint32_t word = *reinterpret_cast<const uint32_t*>(blobs + L.tile_off(T, kb) + s * 512 + lane * 16 + w * 4);
        const int8_t q = (int8_t)((word >> (8 * kk)) & 0xFFu);
        out[idx] = __fmul_rn((float)q, scale);
    }
}

__global__ void dequant_i8_raw_kernel(const uint8_t* __restrict__ raw, float scale, float* __restrict__ out,
                                      size_t total) {
    for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total;
         idx += (size_t)gridDim.x * blockDim.x)
        out[idx] = __fmul_rn((float)(int8_t)raw[idx], scale);
}

__global__ void apply_outliers_kernel(const uint32_t* __restrict__ row_ptr, const uint2* __restrict__ entries,
                                      const uint16_t* __restrict__ vals, float* __restrict__ out, int N, int K) {
    for (int row = blockIdx.x * blockDim.y + threadIdx.y; row < N; row += gridDim.x * blockDim.y) {
        for (uint32_t e = row_ptr[row] + threadIdx.x; e < row_ptr[row + 1]; e += blockDim.x)
            out[(size_t)row * K + entries[e].x] = half_bits_to_float(vals[e]);
    }
}

__global__ void apply_outliers_items_kernel(const uint32_t* __restrict__ item_ptr, const uint2* __restrict__ entries,
                                            const uint16_t* __restrict__ vals, float* __restrict__ out, int nT,
                                            int items, int K) {
    for (int item = blockIdx.x * blockDim.y + threadIdx.y; item < items; item += gridDim.x * blockDim.y) {
        const int T = item % nT;
        for (uint32_t e = item_ptr[item] + threadIdx.x; e < item_ptr[item + 1]; e += blockDim.x) {
            const uint2 en = entries[e];
            const size_t row = (size_t)T * 16 + (en.x & 15u);
            out[row * K + (en.x >> 4)] = half_bits_to_float(vals[e]);
        }
    }
}

// ------------------------------------------------------------------------------------------
// Host-side launchers
// ------------------------------------------------------------------------------------------
static int num_sms() {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
}

size_t stream_scratch_bytes(int kind, int N, int K) {
    const TileLayout L(kind, N, K);
    return (size_t)L.nT * L.nchunks * 16 * kMaxBatch * 4 + (size_t)L.nT * 4;
}

template <int KIND, int NB>
static cudaError_t launch_stream_t(const StreamArgs& a, int grid, size_t smem, bool pdl, cudaStream_t st) {
    auto kern = gemv_stream_kernel<KIND, NB>;
    static int attr_dev = -1;  // the attribute is per device: set once per device in use
    int dev = 0;
    cudaGetDevice(&dev);
    if (attr_dev != dev) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e != cudaSuccess) return e;
        attr_dev = dev;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(kStreamThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, a);
}

cudaError_t launch_gemv_stream(int kind, const StreamArgs& in, bool pdl, cudaStream_t st) {
    StreamArgs a = in;
    if (a.B < 1 || a.B > kMaxBatch) return cudaErrorInvalidValue;
    const TileLayout L(kind, a.N, a.K);
    const int items = L.items();
    const int grid = items < num_sms() ? items : num_sms();
    // widest x window any CTA stages (chunks)
    int span = 1;
    for (int c = 0; c < grid; c++) {
        const int i0 = (int)((long long)c * items / grid), i1 = (int)((long long)(c + 1) * items / grid);
        if (i1 > i0) span = std::max(span, (i1 - 1) / L.nT - i0 / L.nT + 1);
    }
    a.span = span;
    a.ring = 4;  // ring groups of kGroupItems items
    StreamSmem sp = stream_smem(kind, a.B, a.ring, span);
    while (sp.total > 227 * 1024 && a.ring > 2) {
        a.ring -= 1;
        sp = stream_smem(kind, a.B, a.ring, span);
    }
    if (sp.total > 227 * 1024) return cudaErrorInvalidConfiguration;
    const bool two = a.B > 4;
    switch (kind) {
        case kKindI4:
            return two ? launch_stream_t<kKindI4, 2>(a, grid, sp.total, pdl, st)
                       : launch_stream_t<kKindI4, 1>(a, grid, sp.total, pdl, st);
        case kKindI8:
            return two ? launch_stream_t<kKindI8, 2>(a, grid, sp.total, pdl, st)
                       : launch_stream_t<kKindI8, 1>(a, grid, sp.total, pdl, st);
        default:
            return two ? launch_stream_t<kKindF16, 2>(a, grid, sp.total, pdl, st)
                       : launch_stream_t<kKindF16, 1>(a, grid, sp.total, pdl, st);
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

static dim3 grid_for(size_t total) {
    size_t blocks = (total + 255) / 256;
    const size_t cap = (size_t)num_sms() * 32;
    if (blocks > cap) blocks = cap;
    if (blocks == 0) blocks = 1;
    return dim3((unsigned)blocks);
}

cudaError_t launch_repack(int kind, const uint8_t* src, uint8_t* blobs, int N, int K, cudaStream_t st) {
    const TileLayout L(kind, N, K);
    const size_t total = (size_t)L.nT * L.nkb * 256;
    if (kind == kKindI4) repack_kernel<kKindI4><<<grid_for(total), 256, 0, st>>>(src, blobs, L, total);
    else if (kind == kKindI8) repack_kernel<kKindI8><<<grid_for(total), 256, 0, st>>>(src, blobs, L, total);
    else repack_kernel<kKindF16><<<grid_for(total), 256, 0, st>>>(src, blobs, L, total);
    return cudaGetLastError();
}

cudaError_t launch_repack_i4_scales(const uint8_t* src, uint8_t* blobs, int N, int K, int gs, cudaStream_t st) {
    const TileLayout L(kKindI4, N, K);
    const size_t total = (size_t)L.nT * L.nkb * 16;
    const int groups = (K + gs - 1) / gs;
    repack_i4_scales_kernel<<<grid_for(total), 256, 0, st>>>(src, blobs, L, groups, gs, total);
    return cudaGetLastError();
}

cudaError_t launch_dequant_i4(bool tiled, const void* w, const void* raw_scales, float* out, int N, int K,
                              int groups, int gs, cudaStream_t st) {
    const size_t total = (size_t)N * K;
    if (tiled)
        dequant_i4_tiled_kernel<<<grid_for(total), 256, 0, st>>>((const uint8_t*)w, out, TileLayout(kKindI4, N, K));
    else
        dequant_i4_raw_kernel<<<grid_for(total), 256, 0, st>>>((const uint8_t*)w, (const uint8_t*)raw_scales, out, N,
                                                               K, groups, gs);
    return cudaGetLastError();
}

cudaError_t launch_dequant_i8(bool tiled, const void* w, float scale, float* out, int N, int K, cudaStream_t st) {
    const size_t total = (size_t)N * K;
    if (tiled)
        dequant_i8_tiled_kernel<<<grid_for(total), 256, 0, st>>>((const uint8_t*)w, scale, out,
                                                                 TileLayout(kKindI8, N, K));
    else
        dequant_i8_raw_kernel<<<grid_for(total), 256, 0, st>>>((const uint8_t*)w, scale, out, total);
    return cudaGetLastError();
}

cudaError_t launch_apply_outliers(const uint32_t* row_ptr, const uint2* entries, const uint16_t* vals, float* out,
                                  int N, int K, cudaStream_t st) {
    dim3 block(32, 8);
    dim3 grid((N + 7) / 8 < 4096 ? (N + 7) / 8 : 4096);
    apply_outliers_kernel<<<grid, block, 0, st>>>(row_ptr, entries, vals, out, N, K);
    return cudaGetLastError();
}

cudaError_t launch_apply_outliers_items(const uint32_t* item_ptr, const uint2* entries, const uint16_t* vals,
                                        float* out, int N, int K, cudaStream_t st) {
    const TileLayout L(kKindI4, N, K);
    dim3 block(32, 8);
    const int items = L.items();
    dim3 grid((items + 7) / 8 < 4096 ? (items + 7) / 8 : 4096);
    apply_outliers_items_kernel<<<grid, block, 0, st>>>(item_ptr, entries, vals, out, L.nT, items, K);
    return cudaGetLastError();
}

}  // namespace pox
