/*
 * oracle/quant.c -- CPU restatement of the GGUF Q8_0 / Q4_K block formats.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product path links or calls this file; it is the
 * checker that tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg compare the CUDA
 * kernels against.
 *
 * The arithmetic of these formats lives in ggml (fork betweentwomidnights/ggml @ 922875a6,
 * upstream v0.16.0), which is not vendored with the reference.  Its call sites in the reference:
 *   - dequant to f32 per row: src/lora.h:52-74 (read_to_f32 -> type traits to_float)
 *   - quantized rows are produced along ne[0] = in, only when in % block == 0:
 *     tools/sa3-quantize.cpp:75-85
 * The published algorithm restated here (and pinned against gguf-py 0.19.0's
 * gguf.quants.Q8_0 / Q4_K, which states bit-exactness with ggml-quants.c, by
 * tests/golden/gen_golden.py):
 *   Q8_0  block of 32: f16 d, 32 x int8 q.  d = amax/127, q = roundf(x/d) (half away from 0),
 *         value = q * (float)d.                                       34 bytes / 32 values
 *   Q4_K  super-block of 256: f16 d, f16 dmin, 12 bytes of 6-bit (scale, min) pairs for
 *         8 sub-blocks of 32, 128 bytes of 4-bit q.  value = (d*sc)*q - (dmin*m).
 *                                                                      144 bytes / 256 values
 * The Q4_K *encoder* below is this project's own (any valid encoding works: only the decoder
 * has to be bit-exact).  The Q8_0 encoder follows the published reference rounding exactly.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

/* ---- IEEE half <-> single, round-to-nearest-even (the conversion numpy and F16C use) ---- */
static uint16_t f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t absx = x & 0x7fffffffu;
    if (absx >= 0x7f800000u) {                        /* inf or nan */
        return (uint16_t)(sign | 0x7c00u | (absx > 0x7f800000u ? 0x200u : 0u));
    }
    if (absx >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);   /* rounds to inf */
    if (absx < 0x38800000u) {                         /* result is subnormal or zero */
        if (absx < 0x33000000u) return (uint16_t)sign;             /* < 2^-25: rounds to 0 */
        const uint32_t mant = (absx & 0x7fffffu) | 0x800000u;
        const int exp = (int)(absx >> 23);             /* 102 .. 112 */
        const int shift = 126 - exp;                   /* 14 .. 24 */
        uint32_t h = mant >> shift;
        const uint32_t rem = mant & ((1u << shift) - 1u);
        const uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (h & 1u))) h += 1;
        return (uint16_t)(sign | h);
    }
    uint32_t h = ((absx >> 13) - (112u << 10));        /* rebias exponent 127 -> 15 */
    const uint32_t rem = absx & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1;
    return (uint16_t)(sign | h);
}

static float f16_to_f32(uint16_t h) {
    const uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t mant = h & 0x3ffu;
    uint32_t x;
    if (exp == 0) {
        if (mant == 0) {
            x = sign;
        } else {                                       /* normalise a subnormal */
            int e = -1;
            do { e++; mant <<= 1; } while ((mant & 0x400u) == 0);
            x = sign | ((uint32_t)(127 - 15 - e) << 23) | ((mant & 0x3ffu) << 13);
        }
    } else if (exp == 31) {
        x = sign | 0x7f800000u | (mant << 13);
    } else {
        x = sign | ((exp + 112u) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

float oracle_f16_to_f32(uint16_t h) { return f16_to_f32(h); }
uint16_t oracle_f32_to_f16(float f) { return f32_to_f16(f); }

/* ---------------------------------------- Q8_0 ---------------------------------------- */
enum { QK8 = 32, Q8_BYTES = 34, QKK = 256, Q4K_BYTES = 144 };

/* Quantize n values (n % 32 == 0) into n/32 blocks of 34 bytes. */
void oracle_quantize_q8_0(const float* x, uint8_t* out, int64_t n) {
    for (int64_t b = 0; b < n / QK8; ++b) {
        const float* xb = x + b * QK8;
        uint8_t* ob = out + b * Q8_BYTES;
        float amax = 0.0f;
        for (int j = 0; j < QK8; ++j) amax = fmaxf(amax, fabsf(xb[j]));
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        const uint16_t dh = f32_to_f16(d);
        memcpy(ob, &dh, 2);
        for (int j = 0; j < QK8; ++j) {
            const float v = xb[j] * id;
            ob[2 + j] = (uint8_t)(int8_t)roundf(v);     /* roundf: half away from zero */
        }
    }
}

void oracle_dequantize_q8_0(const uint8_t* in, float* y, int64_t n) {
    for (int64_t b = 0; b < n / QK8; ++b) {
        const uint8_t* ib = in + b * Q8_BYTES;
        uint16_t dh;
        memcpy(&dh, ib, 2);
        const float d = f16_to_f32(dh);
        for (int j = 0; j < QK8; ++j) y[b * QK8 + j] = (float)(int8_t)ib[2 + j] * d;
    }
}

/* ---------------------------------------- Q4_K ---------------------------------------- */
/* 6-bit (scale, min) unpack of sub-block j (0..7) from the 12-byte field. */
static void q4k_scale_min(const uint8_t* s, int j, uint8_t* sc, uint8_t* mn) {
    if (j < 4) {
        *sc = s[j] & 63u;
        *mn = s[j + 4] & 63u;
    } else {
        *sc = (uint8_t)((s[j + 4] & 0x0fu) | ((s[j - 4] >> 6) << 4));
        *mn = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
    }
}

void oracle_q4k_scale_min(const uint8_t* block, int j, uint8_t* sc, uint8_t* mn) {
    q4k_scale_min(block + 4, j, sc, mn);
}

void oracle_dequantize_q4_k(const uint8_t* in, float* y, int64_t n) {
    for (int64_t b = 0; b < n / QKK; ++b) {
        const uint8_t* ib = in + b * Q4K_BYTES;
        uint16_t dh, mh;
        memcpy(&dh, ib, 2);
        memcpy(&mh, ib + 2, 2);
        const float d = f16_to_f32(dh), dmin = f16_to_f32(mh);
        const uint8_t* sc12 = ib + 4;
        const uint8_t* qs = ib + 16;
        float* yb = y + b * QKK;
        for (int sb = 0; sb < 8; ++sb) {
            uint8_t sc, mn;
            q4k_scale_min(sc12, sb, &sc, &mn);
            const float d1 = d * (float)sc, m1 = dmin * (float)mn;
            const uint8_t* q = qs + (sb / 2) * 32;
            const int shift = (sb & 1) ? 4 : 0;
            for (int l = 0; l < 32; ++l) yb[sb * 32 + l] = d1 * (float)((q[l] >> shift) & 0x0f) - m1;
        }
    }
}

/* This project's own Q4_K encoder: per sub-block affine fit over [min(0,x), max(x)], then the
 * 8 scales / mins are quantized to 6 bits against the super-block d / dmin (stored as f16, and
 * the f16-rounded values are the ones used to pick q, so decode(encode(x)) is self-consistent). */
void oracle_quantize_q4_k(const float* x, uint8_t* out, int64_t n) {
    for (int64_t b = 0; b < n / QKK; ++b) {
        const float* xb = x + b * QKK;
        uint8_t* ob = out + b * Q4K_BYTES;
        float scale[8], minv[8];
        float max_scale = 0.0f, max_min = 0.0f;
        for (int sb = 0; sb < 8; ++sb) {
            float lo = 0.0f, hi = -INFINITY;
            for (int l = 0; l < 32; ++l) {
                lo = fminf(lo, xb[sb * 32 + l]);
                hi = fmaxf(hi, xb[sb * 32 + l]);
            }
            if (hi < lo) hi = lo;
            scale[sb] = (hi - lo) / 15.0f;
            minv[sb] = -lo;
            max_scale = fmaxf(max_scale, scale[sb]);
            max_min = fmaxf(max_min, minv[sb]);
        }
        const uint16_t dh = f32_to_f16(max_scale / 63.0f);
        const uint16_t mh = f32_to_f16(max_min / 63.0f);
        const float d = f16_to_f32(dh), dmin = f16_to_f32(mh);
        uint8_t sc[8], mn[8];
        for (int sb = 0; sb < 8; ++sb) {
            int s = d > 0.0f ? (int)lrintf(scale[sb] / d) : 0;
            int m = dmin > 0.0f ? (int)lrintf(minv[sb] / dmin) : 0;
            sc[sb] = (uint8_t)(s < 0 ? 0 : s > 63 ? 63 : s);
            mn[sb] = (uint8_t)(m < 0 ? 0 : m > 63 ? 63 : m);
        }
        memcpy(ob, &dh, 2);
        memcpy(ob + 2, &mh, 2);
        uint8_t* s12 = ob + 4;
        for (int j = 0; j < 4; ++j) {
            s12[j] = (uint8_t)(sc[j] | ((sc[j + 4] >> 4) << 6));
            s12[j + 4] = (uint8_t)(mn[j] | ((mn[j + 4] >> 4) << 6));
            s12[j + 8] = (uint8_t)((sc[j + 4] & 0x0f) | ((mn[j + 4] & 0x0f) << 4));
        }
        uint8_t* qs = ob + 16;
        memset(qs, 0, 128);
        for (int sb = 0; sb < 8; ++sb) {
            const float d1 = d * (float)sc[sb], m1 = dmin * (float)mn[sb];
            for (int l = 0; l < 32; ++l) {
                int q = d1 > 0.0f ? (int)lrintf((xb[sb * 32 + l] + m1) / d1) : 0;
                q = q < 0 ? 0 : q > 15 ? 15 : q;
                qs[(sb / 2) * 32 + l] |= (uint8_t)(q << ((sb & 1) ? 4 : 0));
            }
        }
    }
}

/* Row norms of a dequantized [out][in] matrix with f64 accumulation, as
 * src/train_lora.h:141-155 (train_row_norms) and :160-174 (train_row_norm_sq, + in*eps). */
void oracle_row_norm_sq(const float* w, int64_t in, int64_t out, float eps, float* nsq, float* norm) {
    for (int64_t o = 0; o < out; ++o) {
        double s = 0.0;
        for (int64_t i = 0; i < in; ++i) {
            const float v = w[o * in + i];
            s += (double)v * v;
        }
        if (nsq) nsq[o] = (float)(s + (double)in * eps);
        if (norm) norm[o] = (float)sqrt(s);
    }
}
