/*
 * pox_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C, single-threaded restatement of ParaOxidizer's CPU decode hot path, against which
 * the CUDA backend's results are compared. Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline leg (and `bench.py --impl reference`) may load it; the product library never
 * links or calls it.
 *
 * Parity pin: the reference is Rust and cannot be built or run in this environment (no cargo,
 * no network), so no output of the reference itself exists here. This restatement is pinned
 * against every known-answer test that the reference's own test suite holds for this path
 * (tests/test_quant_and_security.rs:14-111, paged_cache.rs:223-250, the fidelity bounds of
 * tests/test_model_degradation.rs) and its f16 conversion against an independent IEEE
 * implementation (numpy), see tests/test_oracle_known_answers.py. Bit-level agreement with
 * the Rust binary beyond those tests is therefore argued from the source, not measured.
 *
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off -fno-fast-math): no FMA contraction and
 * IEEE f32 arithmetic on SSE, the same evaluation rules as the Rust code (which never
 * contracts a*b+c and never reassociates float sums).
 *
 * Every function cites the reference file:line it restates (paths relative to the
 * reference repository root).
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORACLE_OK 0
#define ORACLE_ERR 1

/* ------------------------------------------------------------------------------------------
 * binary16 conversions. The reference uses the `half` crate 2.7.1 (Cargo.lock), whose
 * f16::from_f32 is IEEE 754 round-to-nearest-even with overflow to infinity and NaN kept
 * quiet with the top mantissa bits preserved; f16::to_f32 is exact. Restated from the IEEE
 * 754 definition.
 * ---------------------------------------------------------------------------------------- */
uint16_t pox_oracle_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t exp = (x >> 23) & 0xFFu;
    uint32_t man = x & 0x7FFFFFu;
    if (exp == 0xFFu) {
        if (man == 0) return (uint16_t)(sign | 0x7C00u);
        return (uint16_t)(sign | 0x7C00u | 0x0200u | (man >> 13));
    }
    if (exp == 0) return (uint16_t)sign; /* f32 subnormals are far below the f16 range */
    int32_t he = (int32_t)exp - 127 + 15;
    if (he >= 31) return (uint16_t)(sign | 0x7C00u);
    if (he >= 1) {
        uint32_t hm = man >> 13;
        uint32_t rem = man & 0x1FFFu;
        uint32_t out = ((uint32_t)he << 10) + hm;
        if (rem > 0x1000u || (rem == 0x1000u && (hm & 1u))) out += 1; /* may carry into inf */
        return (uint16_t)(sign | out);
    }
    /* result is an f16 subnormal (or zero): value = m * 2^(E-23), unit 2^-24 */
    uint32_t m = man | 0x800000u;
    int32_t s = 14 - he; /* >= 14 */
    if (s > 24) return (uint16_t)sign;
    uint32_t hm = m >> s;
    uint32_t rem = m & ((1u << s) - 1u);
    uint32_t half = 1u << (s - 1);
    if (rem > half || (rem == half && (hm & 1u))) hm += 1;
    return (uint16_t)(sign | hm);
}

float pox_oracle_f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t exp = ((uint32_t)h >> 10) & 0x1Fu;
    uint32_t man = (uint32_t)h & 0x3FFu;
    uint32_t out;
    if (exp == 0x1Fu) {
        out = sign | 0x7F800000u | (man << 13);
    } else if (exp == 0) {
        if (man == 0) {
            out = sign;
        } else { /* normalise the subnormal */
            int e = -1;
            do { man <<= 1; e++; } while (!(man & 0x400u));
            man &= 0x3FFu;
            out = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else {
        out = sign | ((exp - 15 + 127) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &out, 4);
    return f;
}

void pox_oracle_f32_to_f16_array(const float* in, uint16_t* out, size_t n) {
    for (size_t i = 0; i < n; i++) out[i] = pox_oracle_f32_to_f16(in[i]);
}

void pox_oracle_f16_to_f32_array(const uint16_t* in, float* out, size_t n) {
    for (size_t i = 0; i < n; i++) out[i] = pox_oracle_f16_to_f32(in[i]);
}

/* Rust `v.round().clamp(lo, hi) as uN/iN`: round half away from zero, clamp (NaN passes
 * through clamp), then a saturating cast that maps NaN to 0. */
static int32_t rust_round_clamp_cast(float v, float lo, float hi) {
    if (isnan(v)) return 0;
    float r = roundf(v);
    if (r < lo) r = lo;
    if (r > hi) r = hi;
    return (int32_t)r;
}

static uint16_t rd_u16(const uint8_t* p) { return (uint16_t)(p[0] | ((uint16_t)p[1] << 8)); }
static uint32_t rd_u32(const uint8_t* p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
static void wr_u16(uint8_t* p, uint16_t v) { p[0] = (uint8_t)v; p[1] = (uint8_t)(v >> 8); }
static void wr_u32(uint8_t* p, uint32_t v) {
    p[0] = (uint8_t)v; p[1] = (uint8_t)(v >> 8); p[2] = (uint8_t)(v >> 16); p[3] = (uint8_t)(v >> 24);
}

/* ------------------------------------------------------------------------------------------
 * crates/paraoxidizer-quant/src/kernels.rs:26-82 quantize_int4_group.
 * packed_out: (numel + num_groups) / 2 bytes at most (each group starts a fresh byte);
 * scales_out: num_groups * 4 bytes. Returns the number of packed bytes written.
 * ---------------------------------------------------------------------------------------- */
size_t pox_oracle_quantize_int4_group(const float* w, size_t numel, size_t group_size,
                                      uint8_t* packed_out, uint8_t* scales_out) {
    size_t num_groups = (numel + group_size - 1) / group_size;
    size_t np = 0;
    for (size_t g = 0; g < num_groups; g++) {
        size_t start = g * group_size;
        size_t end = start + group_size < numel ? start + group_size : numel;
        float mn = INFINITY, mx = -INFINITY;
        for (size_t i = start; i < end; i++) {
            float v = w[i];
            if (v < mn) mn = v;
            if (v > mx) mx = v;
        }
        if (fabsf(mx - mn) < 1e-8f) mx = mn + 1e-4f; /* kernels.rs:50-52 */
        float scale = (mx - mn) / 15.0f;
        float min_offset = mn;
        wr_u16(scales_out + g * 4, pox_oracle_f32_to_f16(scale));
        wr_u16(scales_out + g * 4 + 2, pox_oracle_f32_to_f16(min_offset));
        size_t len = end - start;
        for (size_t i = 0; i < len; i += 2) {
            uint8_t q0 = (uint8_t)rust_round_clamp_cast((w[start + i] - min_offset) / scale, 0.0f, 15.0f);
            uint8_t q1 = 0;
            if (i + 1 < len)
                q1 = (uint8_t)rust_round_clamp_cast((w[start + i + 1] - min_offset) / scale, 0.0f, 15.0f);
            packed_out[np++] = (uint8_t)((q0 & 0x0F) | ((q1 & 0x0F) << 4)); /* pack_i4 :15-17 */
        }
    }
    return np;
}

/* kernels.rs:85-128 dequantize_int4_group: out = min + q*scale (mul, then add; two f32
 * roundings, no FMA). Stops early when the packed bytes run out, like the reference. */
int pox_oracle_dequantize_int4_group(const uint8_t* packed, size_t packed_len,
                                     const uint8_t* scales, size_t scale_len,
                                     size_t group_size, size_t numel, float* out, size_t out_len) {
    if (out_len < numel) return ORACLE_ERR;
    size_t num_groups = (numel + group_size - 1) / group_size;
    size_t pidx = 0;
    for (size_t g = 0; g < num_groups; g++) {
        size_t start = g * group_size;
        size_t end = start + group_size < numel ? start + group_size : numel;
        if (g * 4 + 4 > scale_len) return ORACLE_ERR; /* Cursor::read_u16 fails: Err */
        float scale = pox_oracle_f16_to_f32(rd_u16(scales + g * 4));
        float mn = pox_oracle_f16_to_f32(rd_u16(scales + g * 4 + 2));
        size_t cur = start;
        while (cur < end) {
            if (pidx >= packed_len) break;
            uint8_t b = packed[pidx++];
            float t0 = (float)(b & 0x0F) * scale;
            out[cur] = mn + t0;
            cur++;
            if (cur < end) {
                float t1 = (float)((b >> 4) & 0x0F) * scale;
                out[cur] = mn + t1;
                cur++;
            }
        }
    }
    return ORACLE_OK;
}

/* kernels.rs:131-154 quantize_int8_symmetric: one per-tensor f32 scale (4 bytes LE). */
void pox_oracle_quantize_int8_symmetric(const float* w, size_t n, uint8_t* q_out, uint8_t* scale_out) {
    float max_abs = 0.0f;
    for (size_t i = 0; i < n; i++) {
        float a = fabsf(w[i]);
        if (a > max_abs) max_abs = a;
    }
    if (max_abs < 1e-8f) max_abs = 1e-4f;
    float scale = max_abs / 127.0f;
    for (size_t i = 0; i < n; i++)
        q_out[i] = (uint8_t)(int8_t)rust_round_clamp_cast(w[i] / scale, -127.0f, 127.0f);
    uint32_t sb;
    memcpy(&sb, &scale, 4);
    wr_u32(scale_out, sb);
}

/* kernels.rs:157-173 dequantize_int8_symmetric */
int pox_oracle_dequantize_int8_symmetric(const uint8_t* q, size_t n, const uint8_t* scale_data,
                                         size_t scale_len, float* out, size_t out_len) {
    if (scale_len < 4) return ORACLE_ERR;
    uint32_t sb = rd_u32(scale_data);
    float scale;
    memcpy(&scale, &sb, 4);
    for (size_t i = 0; i < n && i < out_len; i++) out[i] = (float)(int8_t)q[i] * scale;
    return ORACLE_OK;
}

/* Per-output-channel INT8 (an f16 scale per output row; the reference's .pox INT8 is per tensor,
 * kernels.rs:131-154): the reference's rules applied to each row -- max_abs of the
 * row (floor 1e-4 below 1e-8), scale = max_abs / 127 (f32), stored as f16 (round to nearest even);
 * q = round(w / s) clamped to +-127 with s = the f16 scale read back as f32, so that q * s is the
 * value the stored table dequantizes to. scale_out: rows x 2 bytes LE. */
void pox_oracle_quantize_int8_rows(const float* w, size_t rows, size_t cols, uint8_t* q_out, uint8_t* scale_out) {
    for (size_t r = 0; r < rows; r++) {
        const float* wr = w + r * cols;
        float max_abs = 0.0f;
        for (size_t c = 0; c < cols; c++) {
            float a = fabsf(wr[c]);
            if (a > max_abs) max_abs = a;
        }
        if (max_abs < 1e-8f) max_abs = 1e-4f;
        const uint16_t sh = pox_oracle_f32_to_f16(max_abs / 127.0f);
        const float s = pox_oracle_f16_to_f32(sh);
        for (size_t c = 0; c < cols; c++)
            q_out[r * cols + c] = (uint8_t)(int8_t)rust_round_clamp_cast(wr[c] / s, -127.0f, 127.0f);
        wr_u16(scale_out + 2 * r, sh);
    }
}

/* dequantization of the per-row layout: q * scale_r (one f32 multiply, as dequantize_int8_symmetric). */
int pox_oracle_dequantize_int8_rows(const uint8_t* q, size_t rows, size_t cols, const uint8_t* scale_data,
                                    size_t scale_len, float* out) {
    if (scale_len < 2 * rows) return ORACLE_ERR;
    for (size_t r = 0; r < rows; r++) {
        const float s = pox_oracle_f16_to_f32(rd_u16(scale_data + 2 * r));
        for (size_t c = 0; c < cols; c++) out[r * cols + c] = (float)(int8_t)q[r * cols + c] * s;
    }
    return ORACLE_OK;
}

/* gemv_int8's arithmetic (kernels.rs:229-255: sum += ((q as f32) * scale) * x[c], sequential per row)
 * with the row's own scale. */
int pox_oracle_gemv_int8_rows(const uint8_t* q, size_t rows, size_t cols, const uint8_t* scale_data,
                              size_t scale_len, const float* x, float* y) {
    if (scale_len < 2 * rows) return ORACLE_ERR;
    for (size_t r = 0; r < rows; r++) {
        const uint8_t* qr = q + r * cols;
        const float s = pox_oracle_f16_to_f32(rd_u16(scale_data + 2 * r));
        float sum = 0.0f;
        for (size_t c = 0; c < cols; c++) {
            float t = (float)(int8_t)qr[c] * s;
            sum += t * x[c];
        }
        y[r] = sum;
    }
    return ORACLE_OK;
}

/* kernels.rs:293-316 dot_product_simd, non-aarch64 order: four strided accumulators summed
 * as ((s0+s1)+s2)+s3, then the scalar tail. */
float pox_oracle_dot_x86(const float* a, const float* b, size_t len) {
    float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
    size_t i = 0;
    while (i + 4 <= len) {
        s0 += a[i] * b[i];
        s1 += a[i + 1] * b[i + 1];
        s2 += a[i + 2] * b[i + 2];
        s3 += a[i + 3] * b[i + 3];
        i += 4;
    }
    float total = s0 + s1 + s2 + s3;
    while (i < len) { total += a[i] * b[i]; i++; }
    return total;
}

/* kernels.rs:262-291 dot_product_simd, aarch64 NEON order: two 4-lane FMA accumulators on an
 * 8-wide stride (vfmaq is a fused multiply-add), lane-wise add, horizontal add
 * ((l0+l1)+(l2+l3)) as vaddvq_f32 reduces pairwise, then the unfused scalar tail. */
float pox_oracle_dot_neon(const float* a, const float* b, size_t len) {
    float s0[4] = {0, 0, 0, 0}, s1[4] = {0, 0, 0, 0};
    size_t i = 0;
    while (i + 8 <= len) {
        for (int l = 0; l < 4; l++) {
            s0[l] = fmaf(a[i + l], b[i + l], s0[l]);
            s1[l] = fmaf(a[i + 4 + l], b[i + 4 + l], s1[l]);
        }
        i += 8;
    }
    float c[4];
    for (int l = 0; l < 4; l++) c[l] = s0[l] + s1[l];
    float total = (c[0] + c[1]) + (c[2] + c[3]);
    while (i < len) { total += a[i] * b[i]; i++; }
    return total;
}

/* ------------------------------------------------------------------------------------------
 * crates/paraoxidizer-quant/src/outlier.rs
 * ---------------------------------------------------------------------------------------- */

/* outlier.rs:57-85 extract_and_zero_outliers. mean and std in f32 with sequential sums
 * (Rust's f32 Sum is a left fold), `powi(2)` is x*x, strict `>` against k*std, indices
 * ascending, values rounded to f16, extracted slots zeroed. Returns the count (0 == None). */
size_t pox_oracle_extract_and_zero_outliers(float* w, size_t n, float sigma_mult,
                                            uint32_t* idx_out, uint16_t* val_out) {
    if (n == 0) return 0;
    float sum = -0.0f;
    for (size_t i = 0; i < n; i++) sum += w[i];
    float mean = sum / (float)n;
    float var_sum = -0.0f;
    for (size_t i = 0; i < n; i++) {
        float d = w[i] - mean;
        var_sum += d * d;
    }
    float std_dev = sqrtf(var_sum / (float)n);
    float threshold = sigma_mult * std_dev;
    size_t cnt = 0;
    for (size_t i = 0; i < n; i++) {
        if (fabsf(w[i] - mean) > threshold) {
            idx_out[cnt] = (uint32_t)i;
            val_out[cnt] = pox_oracle_f32_to_f16(w[i]);
            cnt++;
            w[i] = 0.0f;
        }
    }
    return cnt;
}

/* outlier.rs:99-110 to_bytes: count:u32 | indices:u32[count] | values:f16[count], LE */
size_t pox_oracle_outliers_to_bytes(const uint32_t* idx, const uint16_t* val, size_t count, uint8_t* out) {
    wr_u32(out, (uint32_t)count);
    for (size_t i = 0; i < count; i++) wr_u32(out + 4 + 4 * i, idx[i]);
    for (size_t i = 0; i < count; i++) wr_u16(out + 4 + 4 * count + 2 * i, val[i]);
    return 4 + 6 * count;
}

/* outlier.rs:112-127 from_bytes. Fewer than 4 bytes -> empty table (OK); a count that runs
 * past the buffer -> Err. Returns the count, or -1 on Err. */
long pox_oracle_outliers_from_bytes(const uint8_t* b, size_t len, uint32_t* idx, uint16_t* val, size_t cap) {
    if (len < 4) return 0;
    size_t count = rd_u32(b);
    if (4 + 6 * count > len) return -1;
    if (count > cap) return -1;
    for (size_t i = 0; i < count; i++) idx[i] = rd_u32(b + 4 + 4 * i);
    for (size_t i = 0; i < count; i++) val[i] = rd_u16(b + 4 + 4 * count + 2 * i);
    return (long)count;
}

/* outlier.rs:88-95 apply_to */
void pox_oracle_outliers_apply(const uint32_t* idx, const uint16_t* val, size_t count, float* deq, size_t n) {
    for (size_t i = 0; i < count; i++)
        if (idx[i] < n) deq[idx[i]] = pox_oracle_f16_to_f32(val[i]);
}

/* ------------------------------------------------------------------------------------------
 * kernels.rs:177-226 gemv_int4: per row, dequantize into a scratch row, replace outlier slots
 * by scanning the whole table in order (the last entry for a slot wins), then
 * dot_product_simd(row, x). `neon` selects the aarch64 dot order instead of the x86 one.
 * Note the scratch row is reused across rows, as in the reference.
 * ---------------------------------------------------------------------------------------- */
int pox_oracle_gemv_int4(const uint8_t* packed, size_t packed_len, const uint8_t* scales,
                         size_t scale_len, size_t group_size, size_t rows, size_t cols,
                         const uint32_t* out_idx, const uint16_t* out_val, size_t out_count,
                         const float* x, size_t x_len, float* y, size_t y_len, int neon) {
    if (x_len < cols || y_len < rows) return ORACLE_ERR;
    float* row = (float*)calloc(cols ? cols : 1, sizeof(float));
    if (!row) return ORACLE_ERR;
    size_t row_packed = (cols + 1) / 2;
    size_t gpr = (cols + group_size - 1) / group_size;
    size_t row_scale = gpr * 4;
    for (size_t r = 0; r < rows; r++) {
        size_t ws = r * row_packed;
        size_t we = ws + row_packed < packed_len ? ws + row_packed : packed_len;
        size_t ss = r * row_scale;
        size_t se = ss + row_scale < scale_len ? ss + row_scale : scale_len;
        if (ws > we || ss > se) { free(row); return ORACLE_ERR; } /* slice start out of range: panic */
        if (pox_oracle_dequantize_int4_group(packed + ws, we - ws, scales + ss, se - ss, group_size,
                                             cols, row, cols) != ORACLE_OK) {
            free(row);
            return ORACLE_ERR;
        }
        if (out_count) {
            uint32_t ro = (uint32_t)(r * cols);
            for (size_t i = 0; i < out_count; i++) {
                uint32_t id = out_idx[i];
                if (id >= ro && id < ro + (uint32_t)cols) row[id - ro] = pox_oracle_f16_to_f32(out_val[i]);
            }
        }
        y[r] = neon ? pox_oracle_dot_neon(row, x, cols) : pox_oracle_dot_x86(row, x, cols);
    }
    free(row);
    return ORACLE_OK;
}

/* kernels.rs:229-255 gemv_int8: sum += ((q as f32) * scale) * x[c], sequential per row */
int pox_oracle_gemv_int8(const uint8_t* q, size_t q_len, const uint8_t* scale_data, size_t scale_len,
                         size_t rows, size_t cols, const float* x, size_t x_len, float* y, size_t y_len) {
    if (x_len < cols || y_len < rows || q_len < rows * cols) return ORACLE_ERR;
    if (scale_len < 4) return ORACLE_ERR;
    uint32_t sb = rd_u32(scale_data);
    float scale;
    memcpy(&scale, &sb, 4);
    for (size_t r = 0; r < rows; r++) {
        const uint8_t* qr = q + r * cols;
        float sum = 0.0f;
        for (size_t c = 0; c < cols; c++) {
            float t = (float)(int8_t)qr[c] * scale;
            sum += t * x[c];
        }
        y[r] = sum;
    }
    return ORACLE_OK;
}

/* engine.rs:235-250: F16 projection (embedding-style weights and lm_head):
 * sum += w * x[c] sequentially, w = f16 -> f32. */
void pox_oracle_gemv_f16(const uint16_t* w, size_t rows, size_t cols, const float* x, float* y) {
    for (size_t r = 0; r < rows; r++) {
        const uint16_t* wr = w + r * cols;
        float sum = 0.0f;
        for (size_t c = 0; c < cols; c++) sum += pox_oracle_f16_to_f32(wr[c]) * x[c];
        y[r] = sum;
    }
}

/* ------------------------------------------------------------------------------------------
 * crates/paraoxidizer-runtime/src/engine.rs decode-step pieces
 * ---------------------------------------------------------------------------------------- */

/* engine.rs:294-350 rms_norm_with_weight (F16 weight, or none when w == NULL) */
void pox_oracle_rms_norm(float* x, size_t n, const uint16_t* w, float eps) {
    if (n == 0) return;
    float sum_sq = -0.0f;
    for (size_t i = 0; i < n; i++) sum_sq += x[i] * x[i];
    float rms = sqrtf(sum_sq / (float)n + eps);
    float inv = 1.0f / rms;
    for (size_t i = 0; i < n; i++) x[i] *= inv;
    if (w)
        for (size_t i = 0; i < n; i++) x[i] *= pox_oracle_f16_to_f32(w[i]);
}

/* engine.rs:353-408 apply_rope: interleaved pairs (2i, 2i+1), f32 angle = pos * 1/theta^(2i/d) */
void pox_oracle_rope(float* q, size_t nq, float* k, size_t nkv, size_t head_dim, size_t pos, float rope_theta) {
    if (head_dim < 2) return;
    size_t half = head_dim / 2;
    float* cs = (float*)malloc(half * sizeof(float));
    float* sn = (float*)malloc(half * sizeof(float));
    float theta = rope_theta > 1.0f ? rope_theta : 1.0f; /* f32::max(1.0) */
    for (size_t i = 0; i < half; i++) {
        float exponent = (float)(2 * i) / (float)head_dim;
        float freq = 1.0f / powf(theta, exponent);
        float angle = (float)pos * freq;
        cs[i] = 1.0f;
        sn[i] = 0.0f;
        if (isfinite(angle)) { cs[i] = cosf(angle); sn[i] = sinf(angle); }
    }
    for (size_t h = 0; h < nq; h++) {
        float* v = q + h * head_dim;
        for (size_t i = 0; i < half; i++) {
            float a = v[2 * i], b = v[2 * i + 1];
            v[2 * i] = a * cs[i] - b * sn[i];
            v[2 * i + 1] = a * sn[i] + b * cs[i];
        }
    }
    for (size_t h = 0; h < nkv; h++) {
        float* v = k + h * head_dim;
        for (size_t i = 0; i < half; i++) {
            float a = v[2 * i], b = v[2 * i + 1];
            v[2 * i] = a * cs[i] - b * sn[i];
            v[2 * i + 1] = a * sn[i] + b * cs[i];
        }
    }
    free(cs);
    free(sn);
}

/* engine.rs:580-641 GQA attention of one token over positions 0..=pos.
 * kc/vc: this layer's cache, [pos][kv_head][head_dim] f32. out: [nq][head_dim] (zeroed here). */
void pox_oracle_attention(const float* q, const float* kc, const float* vc, size_t nq, size_t nkv,
                          size_t head_dim, size_t pos, float* out) {
    float scale = 1.0f / sqrtf((float)head_dim > 1.0f ? (float)head_dim : 1.0f);
    size_t hpk = nq / (nkv ? nkv : 1);
    if (hpk == 0) hpk = 1;
    float* scores = (float*)malloc((pos + 1) * sizeof(float));
    memset(out, 0, nq * head_dim * sizeof(float));
    for (size_t hq = 0; hq < nq; hq++) {
        size_t hkv = (hq / hpk) % nkv; /* KvCache::get_k folds the head with % num_kv_heads */
        const float* qv = q + hq * head_dim;
        float mx = -INFINITY;
        for (size_t t = 0; t <= pos; t++) {
            const float* kv = kc + (t * nkv + hkv) * head_dim;
            float dot = 0.0f;
            for (size_t d = 0; d < head_dim; d++) dot += qv[d] * kv[d];
            float s = dot * scale;
            if (s > mx) mx = s;
            scores[t] = s;
        }
        if (!isfinite(mx)) mx = 0.0f;
        float sum_exp = 0.0f;
        for (size_t t = 0; t <= pos; t++) {
            float e = expf(scores[t] - mx);
            if (!isfinite(e)) e = 0.0f;
            scores[t] = e;
            sum_exp += e;
        }
        float inv = sum_exp > 1e-9f ? 1.0f / sum_exp : 0.0f;
        for (size_t t = 0; t <= pos; t++) scores[t] *= inv;
        float* o = out + hq * head_dim;
        for (size_t t = 0; t <= pos; t++) {
            float wgt = scores[t];
            const float* vv = vc + (t * nkv + hkv) * head_dim;
            for (size_t d = 0; d < head_dim; d++) o[d] += wgt * vv[d];
        }
    }
    free(scores);
}

/* engine.rs:671-677 SwiGLU: silu(g) * u with silu(g) = g / (1 + exp(-g)) */
void pox_oracle_swiglu(const float* gate, const float* up, float* out, size_t n) {
    for (size_t i = 0; i < n; i++) {
        float g = gate[i];
        float s = g / (1.0f + expf(-g));
        out[i] = s * up[i];
    }
}

/* sampler.rs:55-65 greedy argmax: the first index holding the maximum (strict `>`) */
uint32_t pox_oracle_argmax(const float* logits, size_t n) {
    size_t best = 0;
    float bv = -INFINITY;
    for (size_t i = 0; i < n; i++)
        if (logits[i] > bv) { bv = logits[i]; best = i; }
    return (uint32_t)best;
}

/* ------------------------------------------------------------------------------------------
 * engine.rs:411-716 forward_token for a Llama-architecture model whose projections are INT4
 * (with optional outlier tables), embedding/lm_head/norms F16. The KV cache is the
 * reference's contiguous f32 cache (engine.rs:10-84), [layer][pos][kv_head][dim]; with
 * kv_f16 != 0 K and V are rounded to f16 on store, which is what the fp16 paged cache of the
 * CUDA backend holds.
 * ---------------------------------------------------------------------------------------- */
typedef struct {
    const uint8_t* packed;
    size_t packed_len;
    const uint8_t* scales;
    size_t scale_len;
    const uint32_t* out_idx;
    const uint16_t* out_val;
    size_t out_count;
    size_t rows, cols, group_size;
} pox_oracle_i4_tensor;

typedef struct {
    size_t hidden, inter, layers, n_heads, n_kv_heads, vocab, max_seq;
    float rms_eps, rope_theta;
    int kv_f16;
    const uint16_t* embed;        /* [vocab][hidden] f16 */
    const uint16_t* lm_head;      /* [vocab][hidden] f16 */
    const uint16_t* final_norm;   /* [hidden] f16 */
    const uint16_t* const* attn_norm; /* [layers] -> [hidden] */
    const uint16_t* const* mlp_norm;
    const pox_oracle_i4_tensor* proj; /* [layers][7]: q,k,v,o,gate,up,down */
    float* k_cache;               /* [layers][max_seq][nkv][hd] */
    float* v_cache;
} pox_oracle_model;

static void proj_i4(const pox_oracle_i4_tensor* t, const float* x, float* y) {
    pox_oracle_gemv_int4(t->packed, t->packed_len, t->scales, t->scale_len, t->group_size, t->rows,
                         t->cols, t->out_idx, t->out_val, t->out_count, x, t->cols, y, t->rows, 0);
}

static float round_f16(float v) { return pox_oracle_f16_to_f32(pox_oracle_f32_to_f16(v)); }

int pox_oracle_forward_token(const pox_oracle_model* m, uint32_t token, size_t pos, float* logits) {
    size_t H = m->hidden, hd = H / (m->n_heads ? m->n_heads : 1);
    size_t qd = m->n_heads * hd, kvd = m->n_kv_heads * hd;
    if (pos >= m->max_seq) return ORACLE_ERR;
    float* x = (float*)malloc(H * sizeof(float));
    float* nx = (float*)malloc(H * sizeof(float));
    float* q = (float*)malloc(qd * sizeof(float));
    float* k = (float*)malloc(kvd * sizeof(float));
    float* v = (float*)malloc(kvd * sizeof(float));
    float* att = (float*)malloc(qd * sizeof(float));
    float* o = (float*)malloc(H * sizeof(float));
    float* g = (float*)malloc(m->inter * sizeof(float));
    float* u = (float*)malloc(m->inter * sizeof(float));
    float* s = (float*)malloc(m->inter * sizeof(float));
    size_t tok = token % m->vocab;
    for (size_t i = 0; i < H; i++) x[i] = pox_oracle_f16_to_f32(m->embed[tok * H + i]);
    int sig = 0;
    for (size_t i = 0; i < H; i++) if (fabsf(x[i]) > 1e-6f) { sig = 1; break; }
    if (!sig) { /* engine.rs:518-524 */
        float val = sinf((float)tok * 0.17f) * 0.1f;
        for (size_t i = 0; i < H; i++) x[i] = val;
    }
    for (size_t l = 0; l < m->layers; l++) {
        const pox_oracle_i4_tensor* P = m->proj + l * 7;
        memcpy(nx, x, H * sizeof(float));
        pox_oracle_rms_norm(nx, H, m->attn_norm[l], m->rms_eps);
        proj_i4(&P[0], nx, q);
        proj_i4(&P[1], nx, k);
        proj_i4(&P[2], nx, v);
        pox_oracle_rope(q, m->n_heads, k, m->n_kv_heads, hd, pos, m->rope_theta);
        float* kc = m->k_cache + l * m->max_seq * kvd;
        float* vc = m->v_cache + l * m->max_seq * kvd;
        for (size_t i = 0; i < kvd; i++) {
            kc[pos * kvd + i] = m->kv_f16 ? round_f16(k[i]) : k[i];
            vc[pos * kvd + i] = m->kv_f16 ? round_f16(v[i]) : v[i];
        }
        pox_oracle_attention(q, kc, vc, m->n_heads, m->n_kv_heads, hd, pos, att);
        proj_i4(&P[3], att, o);
        for (size_t i = 0; i < H; i++) x[i] += o[i];
        memcpy(nx, x, H * sizeof(float));
        pox_oracle_rms_norm(nx, H, m->mlp_norm[l], m->rms_eps);
        proj_i4(&P[4], nx, g);
        proj_i4(&P[5], nx, u);
        pox_oracle_swiglu(g, u, s, m->inter);
        proj_i4(&P[6], s, o);
        for (size_t i = 0; i < H; i++) x[i] += o[i];
    }
    pox_oracle_rms_norm(x, H, m->final_norm, m->rms_eps);
    pox_oracle_gemv_f16(m->lm_head, m->vocab, H, x, logits);
    for (size_t i = 0; i < m->vocab; i++)
        if (!isfinite(logits[i])) logits[i] = 0.0f;
    free(x); free(nx); free(q); free(k); free(v); free(att); free(o); free(g); free(u); free(s);
    return ORACLE_OK;
}
