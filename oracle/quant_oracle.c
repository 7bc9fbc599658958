/* CPU oracle (plain C) for the GGML block-quant matvec/matmul.
 *
 * TEST INFRASTRUCTURE ONLY: loaded through ctypes by tests/ (and by bench.py's
 * cpu_baseline leg) as a checker for large cases.  It is never linked into
 * or called by the CUDA library.
 *
 * Restates engine/dequant.py:27-167 of the reference (block layouts :6-9,
 * Q8_0 :75-78, Q4_0 :62-66, Q4_K :97-120, Q5_K :122-144, Q6_K :146-167) with
 * the same f32 rounding: every product is exact in f32, and Q4_K/Q5_K round
 * once at the subtraction of the minimum term.  matvec/matmul accumulate the
 * decoded f32 weights in double precision -- the numeric oracle of the GEMV
 * and MoE paths, ``dequantize(raw) @ x`` in float64.
 */
#include <stdint.h>
#include <string.h>
#include <stdlib.h>

static float half_bits_to_float(uint16_t h)
{
    /* exact fp16 -> f32 widening, subnormals included */
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t expo = (h >> 10) & 31u, mant = h & 1023u, bits;
    if (expo == 0) {
        if (mant == 0) {
            bits = sign;
        } else {
            int e = 113;                  /* 127 - 14 */
            while (!(mant & 1024u)) { mant <<= 1; --e; }
            bits = sign | ((uint32_t)e << 23) | ((mant & 1023u) << 13);
        }
    } else if (expo == 31) {
        bits = sign | 0x7f800000u | (mant << 13);
    } else {
        bits = sign | ((expo + 112u) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static float rd16(const uint8_t *p) { return half_bits_to_float((uint16_t)(p[0] | (p[1] << 8))); }

static void k_scale_min(const uint8_t *s, int g, int *sc, int *mn)
{
    if (g < 4) { *sc = s[g] & 63; *mn = s[g + 4] & 63; }
    else {
        *sc = (s[g + 4] & 15) | ((s[g - 4] >> 6) << 4);
        *mn = (s[g + 4] >> 4) | ((s[g] >> 6) << 4);
    }
}

static int block_values(int t) { return (t == 12 || t == 13 || t == 14) ? 256 : 32; }
static int block_bytes(int t)
{
    switch (t) { case 2: return 18; case 8: return 34; case 12: return 144; case 13: return 176; case 14: return 210; }
    return 0;
}

static void decode_block(int t, const uint8_t *b, float *o)
{
    if (t == 8) {
        float d = rd16(b);
        for (int i = 0; i < 32; ++i) o[i] = (float)(int8_t)b[2 + i] * d;
    } else if (t == 2) {
        float d = rd16(b);
        for (int i = 0; i < 16; ++i) {
            o[i] = ((float)(b[2 + i] & 15) - 8.0f) * d;
            o[i + 16] = ((float)(b[2 + i] >> 4) - 8.0f) * d;
        }
    } else if (t == 12 || t == 13) {
        float d = rd16(b), dmin = rd16(b + 2);
        const uint8_t *s = b + 4;
        const uint8_t *qh = b + 16;
        const uint8_t *qs = b + (t == 12 ? 16 : 48);
        for (int g = 0; g < 8; ++g) {
            int sc, mn;
            k_scale_min(s, g, &sc, &mn);
            volatile float step = d * (float)sc;     /* exact */
            volatile float low = dmin * (float)mn;   /* exact */
            for (int j = 0; j < 32; ++j) {
                int byte = qs[(g / 2) * 32 + j];
                int q = (g & 1) ? (byte >> 4) : (byte & 15);
                if (t == 13) q |= ((qh[j] >> g) & 1) << 4;
                volatile float prod = (float)q * step;  /* exact */
                o[g * 32 + j] = prod - low;             /* the single rounding */
            }
        }
    } else if (t == 14) {
        const uint8_t *ql = b, *qh = b + 128;
        const int8_t *sc = (const int8_t *)(b + 192);
        float d = rd16(b + 208);
        for (int h = 0; h < 2; ++h)
            for (int u = 0; u < 4; ++u)
                for (int j = 0; j < 32; ++j) {
                    int lo = ql[64 * h + 32 * (u & 1) + j];
                    lo = (u < 2) ? (lo & 15) : (lo >> 4);
                    int hi = (qh[32 * h + j] >> (2 * u)) & 3;
                    volatile float a = (float)((lo | (hi << 4)) - 32) * d;   /* exact */
                    o[128 * h + 32 * u + j] = a * (float)sc[8 * h + 2 * u + j / 16];
                }
    }
}

/* Decode ``nblocks`` consecutive blocks; returns 0, or -1 for an unknown type. */
int oracle_dequant(int t, const uint8_t *raw, float *out, long long nblocks)
{
    int bv = block_values(t), bb = block_bytes(t);
    if (!bb) return -1;
    for (long long i = 0; i < nblocks; ++i) decode_block(t, raw + i * bb, out + i * bv);
    return 0;
}

/* y[t][r] = sum_c W[r][c] * x[t][c] in double; x is [tokens][cols]. */
int oracle_matmul_f64(int t, const uint8_t *raw, const float *x, double *y,
                      int rows, int cols, int tokens)
{
    int bv = block_values(t), bb = block_bytes(t);
    if (!bb || cols % bv) return -1;
    long long rb = (long long)(cols / bv) * bb;
    float *w = (float *)malloc(sizeof(float) * (size_t)cols);
    if (!w) return -2;
    for (int r = 0; r < rows; ++r) {
        for (int b = 0; b < cols / bv; ++b) decode_block(t, raw + r * rb + (long long)b * bb, w + b * bv);
        for (int k = 0; k < tokens; ++k) {
            double acc = 0.0;
            const float *xk = x + (long long)k * cols;
            for (int c = 0; c < cols; ++c) acc += (double)w[c] * (double)xk[c];
            y[(long long)k * rows + r] = acc;
        }
    }
    free(w);
    return 0;
}
