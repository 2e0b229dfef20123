/*
 * qraf_oracle.c — CPU restatement of QRAF's quantized matvec path.
 *
 * TEST INFRASTRUCTURE ONLY: the parity checker for the CUDA kernels.  Nothing
 * in the product links or calls this file.  See qraf_oracle.h for the contract.
 *
 * Must be compiled with -ffp-contract=off (no FMA contraction) and without
 * -ffast-math: the reference's Linux build (GCC, x86-64, -O3, no -march) emits
 * separate fp32 multiply and add instructions, and bit-parity depends on it.
 */
#include "qraf_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ── fp16 helpers ───────────────────────────────────────────────────────── */

/* Follows src/tensor/dtype.cpp:9-37: exact decode, subnormals normalised by a
 * shift loop, exponent 31 kept as inf/nan with the mantissa carried over. */
float qo_fp16_to_fp32(uint16_t h) {
    uint32_t sign = (h >> 15) & 1u;
    uint32_t e = (h >> 10) & 0x1Fu;
    uint32_t m = h & 0x3FFu;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign << 31;
        } else {
            int ee = 1;
            while (!(m & 0x400u)) { m <<= 1; ee--; }
            m &= 0x3FFu;
            bits = (sign << 31) | ((uint32_t)(ee + 112) << 23) | (m << 13);
        }
    } else if (e == 31) {
        bits = (sign << 31) | 0x7F800000u | (m << 13);
    } else {
        bits = (sign << 31) | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* Follows src/tensor/dtype.cpp:39-59: the mantissa is TRUNCATED (m >> 13, no
 * rounding); unbiased exponent > 15 (including NaN) encodes as signed inf;
 * exponent <= -15 flushes to signed zero (no fp16 subnormals are produced). */
uint16_t qo_fp32_to_fp16(float f) {
    uint32_t bits;
    memcpy(&bits, &f, 4);
    uint32_t sign = (bits >> 31) & 1u;
    int32_t e = (int32_t)((bits >> 23) & 0xFFu) - 127;
    uint32_t m = bits & 0x7FFFFFu;
    if (e > 15) return (uint16_t)((sign << 15) | 0x7C00u);
    if (e > -15) return (uint16_t)((sign << 15) | ((uint32_t)(e + 15) << 10) | (m >> 13));
    return (uint16_t)(sign << 15);
}

/* ── layout ─────────────────────────────────────────────────────────────── */

size_t qo_block_bytes(uint32_t dtype, int bs) {
    if (dtype == QO_DTYPE_Q8_0) return 4u + (size_t)bs;           /* quantize.cpp:107 */
    if (dtype == QO_DTYPE_Q4_0) return 2u + (size_t)(bs / 2);     /* quantize.cpp:146 */
    return 0;
}

size_t qo_row_bytes(uint32_t dtype, int bs, uint32_t K) {
    size_t nb = ((size_t)K + (size_t)bs - 1) / (size_t)bs;        /* backend.cpp:138 */
    return nb * qo_block_bytes(dtype, bs);
}

/* std::min(a, b) / std::max(a, b) as the reference evaluates them
 * ((b < a) ? b : a and (a < b) ? b : a): with a NaN second argument these
 * return the FIRST argument, which is what makes NaN inputs clamp the way the
 * reference clamps them. */
static inline float ref_min(float a, float b) { return (b < a) ? b : a; }
static inline float ref_max(float a, float b) { return (a < b) ? b : a; }

/* ── quantizers ─────────────────────────────────────────────────────────── */

/* Follows src/tensor/quantize.cpp:105-140.  Per block: max |x| over the
 * block's valid elements; scale = max/127; inv = 1/scale (0 when scale is 0);
 * q = round_half_away(clamp(x*inv, -127, 127)).  Output is zero-initialised, so
 * the bytes of a ragged last block past `count` stay 0. */
size_t qo_quantize_q8_0(const float* data, size_t count, int bs, uint8_t* out) {
    size_t nb = (count + (size_t)bs - 1) / (size_t)bs;
    size_t bb = 4u + (size_t)bs;
    memset(out, 0, nb * bb);
    uint8_t* o = out;
    for (size_t b = 0; b < nb; b++) {
        size_t off = b * (size_t)bs;
        size_t rem = count - off;
        int n = (int)(rem < (size_t)bs ? rem : (size_t)bs);
        float max_abs = 0.0f;
        for (int i = 0; i < n; i++) {
            float a = fabsf(data[off + i]);
            if (a > max_abs) max_abs = a;
        }
        float scale = max_abs / 127.0f;
        float inv = (scale > 0.0f) ? 1.0f / scale : 0.0f;
        memcpy(o, &scale, 4);
        int8_t* q = (int8_t*)(o + 4);
        for (int i = 0; i < n; i++) {
            float v = data[off + i] * inv;
            v = ref_max(-127.0f, ref_min(127.0f, v));
            q[i] = (int8_t)roundf(v);
        }
        o += bb;
    }
    return nb * bb;
}

/* Follows src/tensor/quantize.cpp:144-183.  scale = max/7; inv is taken from
 * the fp32 scale, the stored scale is the truncating fp16 encoding; each value
 * is rounded THEN clamped to [-8, 7]; byte i holds element 2i in its low nibble
 * and element 2i+1 in its high nibble (nibble = q + 8).  With an odd number of
 * valid elements the last one is not stored (only n/2 bytes are packed). */
size_t qo_quantize_q4_0(const float* data, size_t count, int bs, uint8_t* out) {
    size_t nb = (count + (size_t)bs - 1) / (size_t)bs;
    size_t bb = 2u + (size_t)(bs / 2);
    memset(out, 0, nb * bb);
    uint8_t* o = out;
    for (size_t b = 0; b < nb; b++) {
        size_t off = b * (size_t)bs;
        size_t rem = count - off;
        int n = (int)(rem < (size_t)bs ? rem : (size_t)bs);
        float max_abs = 0.0f;
        for (int i = 0; i < n; i++) {
            float a = fabsf(data[off + i]);
            if (a > max_abs) max_abs = a;
        }
        float scale = max_abs / 7.0f;
        float inv = (scale > 0.0f) ? 1.0f / scale : 0.0f;
        uint16_t s16 = qo_fp32_to_fp16(scale);
        memcpy(o, &s16, 2);
        uint8_t* q = o + 2;
        for (int i = 0; i < n / 2; i++) {
            float v0 = data[off + 2 * i] * inv;
            float v1 = data[off + 2 * i + 1] * inv;
            v0 = ref_max(-8.0f, ref_min(7.0f, roundf(v0)));
            v1 = ref_max(-8.0f, ref_min(7.0f, roundf(v1)));
            uint8_t lo = (uint8_t)((int)v0 + 8) & 0x0F;
            uint8_t hi = (uint8_t)((int)v1 + 8) & 0x0F;
            q[i] = (uint8_t)(lo | (hi << 4));
        }
        o += bb;
    }
    return nb * bb;
}

/* ── dequantizers ───────────────────────────────────────────────────────── */

void qo_dequantize_block_q8_0(const void* block, float* out, int bs) {   /* quantize.cpp:17-28 */
    const uint8_t* p = (const uint8_t*)block;
    float scale;
    memcpy(&scale, p, 4);
    const int8_t* q = (const int8_t*)(p + 4);
    for (int i = 0; i < bs; i++) out[i] = (float)q[i] * scale;
}

void qo_dequantize_block_q4_0(const void* block, float* out, int bs) {   /* quantize.cpp:35-51 */
    const uint8_t* p = (const uint8_t*)block;
    uint16_t s16;
    memcpy(&s16, p, 2);
    float scale = qo_fp16_to_fp32(s16);
    const uint8_t* q = p + 2;
    for (int i = 0; i < bs / 2; i++) {
        int lo = (q[i] & 0x0F) - 8;
        int hi = ((q[i] >> 4) & 0x0F) - 8;
        out[2 * i] = (float)lo * scale;
        out[2 * i + 1] = (float)hi * scale;
    }
}

/* ── dot products ───────────────────────────────────────────────────────── */

/* Follows src/tensor/quantize.cpp:187-210.  Operation order is the parity
 * contract: block_sum accumulates fl(q*x) sequentially from 0; then
 * total = fl(total + fl(block_sum*scale)), sequentially over blocks. */
float qo_dot_q8_0_f32(const void* q8, const float* x, size_t count, int bs) {
    const uint8_t* p = (const uint8_t*)q8;
    float total = 0.0f;
    size_t nb = (count + (size_t)bs - 1) / (size_t)bs;
    for (size_t b = 0; b < nb; b++) {
        float scale;
        memcpy(&scale, p, 4);
        p += 4;
        const int8_t* q = (const int8_t*)p;
        size_t off = b * (size_t)bs;
        size_t rem = count - off;
        int n = (int)(rem < (size_t)bs ? rem : (size_t)bs);
        float block_sum = 0.0f;
        for (int i = 0; i < n; i++) {
            float prod = (float)q[i] * x[off + i];
            block_sum = block_sum + prod;
        }
        float part = block_sum * scale;
        total = total + part;
        p += bs;
    }
    return total;
}

/* Follows src/tensor/quantize.cpp:212-239 (same order; low nibble is element
 * 2i, high nibble element 2i+1, both biased by 8; scale decoded from fp16). */
float qo_dot_q4_0_f32(const void* q4, const float* x, size_t count, int bs) {
    const uint8_t* p = (const uint8_t*)q4;
    float total = 0.0f;
    size_t nb = (count + (size_t)bs - 1) / (size_t)bs;
    for (size_t b = 0; b < nb; b++) {
        uint16_t s16;
        memcpy(&s16, p, 2);
        float scale = qo_fp16_to_fp32(s16);
        p += 2;
        size_t off = b * (size_t)bs;
        size_t rem = count - off;
        int n = (int)(rem < (size_t)bs ? rem : (size_t)bs);
        float block_sum = 0.0f;
        for (int i = 0; i < n / 2; i++) {
            uint8_t packed = p[i];
            int lo = (packed & 0x0F) - 8;
            int hi = ((packed >> 4) & 0x0F) - 8;
            float p0 = (float)lo * x[off + 2 * i];
            block_sum = block_sum + p0;
            float p1 = (float)hi * x[off + 2 * i + 1];
            block_sum = block_sum + p1;
        }
        float part = block_sum * scale;
        total = total + part;
        p += bs / 2;
    }
    return total;
}

/* ── matvec ─────────────────────────────────────────────────────────────── */

/* Follows src/nn/backend.cpp:131-199, scalar branch (the one Linux runs):
 * rows are row_bytes apart and each output is one dot over K elements. */
void qo_matvec_q(const void* w, uint32_t dtype, int bs, uint32_t N, uint32_t K,
                 const float* x, float* y) {
    const uint8_t* base = (const uint8_t*)w;
    if (dtype == QO_DTYPE_Q8_0) {
        size_t rb = qo_row_bytes(dtype, bs, K);
        for (uint32_t i = 0; i < N; i++) y[i] = qo_dot_q8_0_f32(base + (size_t)i * rb, x, K, bs);
    } else if (dtype == QO_DTYPE_Q4_0) {
        size_t rb = qo_row_bytes(dtype, bs, K);
        for (uint32_t i = 0; i < N; i++) y[i] = qo_dot_q4_0_f32(base + (size_t)i * rb, x, K, bs);
    } else {
        memset(y, 0, (size_t)N * sizeof(float));
    }
}

void qo_matmul_q(const void* w, uint32_t dtype, int bs, uint32_t N, uint32_t K,
                 uint32_t M, const float* x, float* y) {
    for (uint32_t m = 0; m < M; m++)
        qo_matvec_q(w, dtype, bs, N, K, x + (size_t)m * K, y + (size_t)m * N);
}

void qo_block_partials(const void* w, uint32_t dtype, int bs, uint32_t N, uint32_t K,
                       const float* x, float* out) {
    size_t nb = ((size_t)K + (size_t)bs - 1) / (size_t)bs;
    size_t rb = qo_row_bytes(dtype, bs, K);
    size_t bb = qo_block_bytes(dtype, bs);
    for (uint32_t r = 0; r < N; r++) {
        const uint8_t* p = (const uint8_t*)w + (size_t)r * rb;
        for (size_t b = 0; b < nb; b++, p += bb) {
            size_t off = b * (size_t)bs;
            size_t rem = (size_t)K - off;
            int n = (int)(rem < (size_t)bs ? rem : (size_t)bs);
            float block_sum = 0.0f;
            float scale;
            if (dtype == QO_DTYPE_Q8_0) {
                memcpy(&scale, p, 4);
                const int8_t* q = (const int8_t*)(p + 4);
                for (int i = 0; i < n; i++) {
                    float prod = (float)q[i] * x[off + i];
                    block_sum = block_sum + prod;
                }
            } else {
                uint16_t s16;
                memcpy(&s16, p, 2);
                scale = qo_fp16_to_fp32(s16);
                const uint8_t* q = p + 2;
                for (int i = 0; i < n / 2; i++) {
                    float p0 = (float)((q[i] & 0x0F) - 8) * x[off + 2 * i];
                    block_sum = block_sum + p0;
                    float p1 = (float)(((q[i] >> 4) & 0x0F) - 8) * x[off + 2 * i + 1];
                    block_sum = block_sum + p1;
                }
            }
            out[(size_t)r * nb + b] = block_sum * scale;
        }
    }
}

void qo_matvec_q_f64(const void* w, uint32_t dtype, int bs, uint32_t N, uint32_t K,
                     const float* x, double* y) {
    size_t nb = ((size_t)K + (size_t)bs - 1) / (size_t)bs;
    size_t rb = qo_row_bytes(dtype, bs, K);
    size_t bb = qo_block_bytes(dtype, bs);
    for (uint32_t r = 0; r < N; r++) {
        const uint8_t* p = (const uint8_t*)w + (size_t)r * rb;
        double total = 0.0;
        for (size_t b = 0; b < nb; b++, p += bb) {
            size_t off = b * (size_t)bs;
            size_t rem = (size_t)K - off;
            int n = (int)(rem < (size_t)bs ? rem : (size_t)bs);
            double s = 0.0;
            if (dtype == QO_DTYPE_Q8_0) {
                float scale;
                memcpy(&scale, p, 4);
                const int8_t* q = (const int8_t*)(p + 4);
                for (int i = 0; i < n; i++) s += (double)q[i] * (double)x[off + i];
                total += s * (double)scale;
            } else {
                uint16_t s16;
                memcpy(&s16, p, 2);
                const uint8_t* q = p + 2;
                for (int i = 0; i < n / 2; i++) {
                    s += (double)((q[i] & 0x0F) - 8) * (double)x[off + 2 * i];
                    s += (double)(((q[i] >> 4) & 0x0F) - 8) * (double)x[off + 2 * i + 1];
                }
                total += s * (double)qo_fp16_to_fp32(s16);
            }
        }
        y[r] = total;
    }
}

/* Integer limb partials (the FAST kernels' integer path; see qraf_oracle.h).
 * Not a restatement of reference code: the reference has no integer path.  The
 * dot it reconstructs, sum_b scale_b * c_b * sum_j 2^(8(3-j)) D_j, approximates
 * dot_q*_0_f32 (quantize.cpp:187-239) with X_i carrying 30 bits of each block's
 * range.  Per block: t = fl(max|x| * (1 + 2^-8)), e with t < 2^e (frexpf; 128 when
 * t overflows), c = 2^(e-30), X_i = rint(x_i 2^(30-e)) (half to even), and the
 * balanced base-256 digits of X_i, -128 <= L_j <= 127, most significant first. */
void qo_limb_partials(const void* w, uint32_t dtype, uint32_t N, uint32_t K, const float* x, int32_t* D,
                      float* c) {
    const size_t nb = (size_t)K / 32;
    const size_t rb = qo_row_bytes(dtype, 32, K);
    const size_t bb = qo_block_bytes(dtype, 32);
    int32_t* L = (int32_t*)malloc(sizeof(int32_t) * 4 * 32 * (nb ? nb : 1));
    for (size_t b = 0; b < nb; b++) {
        const float* xb = x + 32 * b;
        float amax = 0.0f;
        int bad = 0;
        for (int i = 0; i < 32; i++) {
            float a = fabsf(xb[i]);
            if (!isfinite(xb[i])) bad = 1;
            else if (a > amax) amax = a;
        }
        int e = 0;
        int live = amax > 0.0f && !bad;
        if (live) {
            const float t = amax * 1.00390625f;
            if (isinf(t)) e = 128;
            else frexpf(t, &e);   /* t = m * 2^e, m in [0.5, 1) */
        }
        c[b] = bad ? NAN : (live ? ldexpf(1.0f, e - 30) : 0.0f);
        for (int i = 0; i < 32; i++) {
            long X = live ? lrintf(ldexpf(xb[i], 30 - e)) : 0;   /* exact scaling, round half to even */
            int32_t* l = L + (b * 32 + (size_t)i) * 4;
            for (int j = 3; j >= 0; j--) {   /* balanced digits, least significant first */
                long d = X & 0xFF;
                if (d >= 128) d -= 256;
                l[j] = (int32_t)d;
                X = (X - d) / 256;
            }
        }
    }
    for (uint32_t r = 0; r < N; r++) {
        const uint8_t* row = (const uint8_t*)w + (size_t)r * rb;
        for (size_t b = 0; b < nb; b++) {
            const uint8_t* p = row + b * bb;
            int32_t d[4] = {0, 0, 0, 0};
            for (int i = 0; i < 32; i++) {
                int q;
                if (dtype == QO_DTYPE_Q8_0) q = (int)((const int8_t*)(p + 4))[i];
                else q = (int)((i & 1) ? ((p[2 + i / 2] >> 4) & 0x0F) : (p[2 + i / 2] & 0x0F)) - 8;
                const int32_t* l = L + (b * 32 + (size_t)i) * 4;
                for (int j = 0; j < 4; j++) d[j] += q * l[j];
            }
            for (int j = 0; j < 4; j++) D[((size_t)r * nb + b) * 4 + (size_t)j] = d[j];
        }
    }
    free(L);
}

/* RMSNorm in place, src/nn/ops.cpp:107-118 (rms_norm_inplace, the Linux path of
 * dispatch_rms_norm): a running fp32 sum of fl(x*x), fl(fl(ss / size) + eps),
 * r = fl(1 / sqrt), then x = fl(fl(x * r) * w). */
void qo_rms_norm(float* x, const float* w, int size, float eps) {
    float ss = 0.0f;
    for (int i = 0; i < size; i++) {
        const float sq = x[i] * x[i];
        ss = ss + sq;
    }
    ss = ss / (float)size + eps;
    const float r = 1.0f / sqrtf(ss);
    for (int i = 0; i < size; i++) {
        const float t = x[i] * r;
        x[i] = t * w[i];
    }
}

