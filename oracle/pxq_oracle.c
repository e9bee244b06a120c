/*
 * pxq_oracle.c -- CPU restatement of Pixelina's quantized-matmul arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker that the CUDA path is
 * compared against; it is never linked into, called by, or shipped with the
 * product library (pixelina_b200/libpxq.so).  Only tests/, the smoke check
 * in __graft_entry__.py and the cpu_baseline leg of bench.py may load it.
 *
 * Every function restates, in plain scalar C, one function of the reference
 * (paths relative to the Pixelina source tree):
 *
 *   pxo_quantize_row_q8_0   src/kernels_quant.cpp:120-144  quantize_row_q8_0_ref
 *   pxo_quantize_row_q8_K   src/kernels_quant.cpp:80-118   quantize_row_q8_K_ref
 *   pxo_dot_q8_0            src/kernels_quant.cpp:339-365  pix_dot_q8_0
 *   pxo_dot_q5_K            src/kernels_quant.cpp:163-254  pix_dot_q5_K
 *   pxo_dot_q6_K            src/kernels_quant.cpp:256-337  pix_dot_q6_K
 *   pxo_block_dots_q6_K     src/kernels_quant.cpp:256-337  its exact int32 super-block sums
 *   pxo_quant_matmul        src/kernels_quant.cpp:369-412  cpu_quant_matmul
 *   pxo_decode              src/backend_cpu.cpp:24-101     cpu_decode
 *   pxo_weight_bytes        src/model.cpp:87-121           weight_bytes
 *
 * The reference computes its dots with 8-lane AVX2 integer partials and an
 * 8-lane fp32 FMA accumulator, then a fixed horizontal-sum order.  The dots
 * here replay that lane structure with scalars so that their fp32 result is
 * bit-identical to the reference build, not merely close.  The
 * pxo_block_dots_* functions additionally expose the exact int32 block dot
 * products, which every implementation (reference, oracle, CUDA) must agree
 * on exactly.
 *
 * Build: see oracle/Makefile (plain C11, no fast-math, no FP contraction).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define PXO_QK8_0 32
#define PXO_QK_K 256
#define PXO_Q8_0_BYTES 34
#define PXO_Q8_K_BYTES 292
#define PXO_Q5_K_BYTES 176
#define PXO_Q6_K_BYTES 210
#define PXO_TYPE_F32 0
#define PXO_TYPE_F16 1
#define PXO_TYPE_Q8_0 8
#define PXO_TYPE_Q5_K 13
#define PXO_TYPE_Q6_K 14
#define PXO_TYPE_BF16 30

/* ---------------------------------------------------------------- fp16 --- */

/* IEEE binary16 -> binary32, exact (every half is representable). */
float pxo_half_to_float(uint16_t h)
{
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 31u;
    uint32_t man = h & 1023u;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            /* subnormal: man * 2^-24, normalise */
            int e = -1;
            do {
                man <<= 1;
                e++;
            } while (!(man & 1024u));
            man &= 1023u;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 112u) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* binary32 -> binary16 with round-to-nearest-even, the rounding mode the
 * reference requests from F16C (_cvtss_sh(d,_MM_FROUND_TO_NEAREST_INT),
 * src/kernels_quant.cpp:136).  NaNs are quieted keeping the top payload bits,
 * as F16C does. */
uint16_t pxo_float_to_half(float f)
{
    uint32_t x;
    memcpy(&x, &f, 4);
    uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) {
        if (ax == 0x7f800000u) return sign | 0x7c00u;
        return (uint16_t)(sign | 0x7e00u | ((ax >> 13) & 0x3ffu));
    }
    uint32_t e = ax >> 23;
    uint32_t mant = (ax & 0x7fffffu) | (e ? 0x800000u : 0u);
    if (e < 113) {
        /* result is a half subnormal (or zero): units of 2^-24.
         * value = mant * 2^(e-150)  (e==0: mant * 2^-149) */
        uint32_t ee = e ? e : 1;
        uint32_t shift = 126 - ee; /* value / 2^-24 = mant >> shift */
        if (shift > 31) return sign;
        uint32_t q = mant >> shift;
        uint32_t rem = mant & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1u))) q++;
        return (uint16_t)(sign | q);
    }
    /* normal half range (may round up into infinity) */
    uint32_t q = ((e - 112u) << 10) | ((ax >> 13) & 0x3ffu);
    uint32_t rem = ax & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
    if (q >= 0x7c00u) return sign | 0x7c00u;
    return (uint16_t)(sign | q);
}

static uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static void wr16(uint8_t* p, uint16_t v)
{
    p[0] = (uint8_t)(v & 255u);
    p[1] = (uint8_t)(v >> 8);
}

/* ------------------------------------------------------------ quantize --- */

/* src/kernels_quant.cpp:120-144.  Per 32-block: amax = max|x|, d = amax/127
 * (fp32), id = d ? 1/d : 0, stored d = fp16_rne(d), q = roundf(x*id)
 * (rounding half away from zero).  Block layout: {u16 d; i8 qs[32]}. */
void pxo_quantize_row_q8_0(const float* x, uint8_t* y, int64_t k)
{
    const int64_t nb = k / PXO_QK8_0;
    for (int64_t i = 0; i < nb; i++) {
        float amax = 0.0f;
        for (int j = 0; j < PXO_QK8_0; j++) {
            const float v = fabsf(x[i * PXO_QK8_0 + j]);
            amax = amax < v ? v : amax; /* std::max(amax, v) */
        }
        const float d = amax / 127;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        uint8_t* blk = y + i * PXO_Q8_0_BYTES;
        wr16(blk, pxo_float_to_half(d));
        for (int j = 0; j < PXO_QK8_0; j++) {
            const float x0 = x[i * PXO_QK8_0 + j] * id;
            blk[2 + j] = (uint8_t)(int8_t)roundf(x0);
        }
    }
}

/* The reference's nearest_int (src/kernels_quant.cpp:41-48): add 1.5*2^23 and
 * read the low mantissa bits; rounds half to even for |v| < 2^22.
 *
 * The reference is C++ built with -O3 -std=c++17, for which g++ defaults to
 * -ffp-contract=fast; nearest_int is inlined into the FMA-enabled
 * quantize_row_q8_K_ref, so `iscale*x[j] + 12582912.0f` is evaluated as ONE
 * fused multiply-add (checked against the reference build on crafted
 * near-tie inputs, tests/test_oracle.py).  The restatement takes the product
 * and the bias together for that reason. */
static int pxo_nearest_int_fused(float iscale, float xv)
{
    float val = fmaf(iscale, xv, 12582912.0f);
    int32_t i;
    memcpy(&i, &val, 4);
    return (i & 0x007fffff) - 0x00400000;
}

/* src/kernels_quant.cpp:80-118.  Per 256-block: the signed value with the
 * largest |x| (first one on ties), iscale = -127/max, q = min(127,
 * nearest_int(iscale*x)), bsums over 16-element groups, d = 1/iscale.
 * Block layout: {f32 d; i8 qs[256]; i16 bsums[16]} = 292 bytes. */
void pxo_quantize_row_q8_K(const float* x, uint8_t* y, int64_t k)
{
    const int64_t nb = k / PXO_QK_K;
    for (int64_t i = 0; i < nb; i++) {
        uint8_t* blk = y + i * PXO_Q8_K_BYTES;
        float max = 0.0f, amax = 0.0f;
        for (int j = 0; j < PXO_QK_K; j++) {
            float ax = fabsf(x[j]);
            if (ax > amax) {
                amax = ax;
                max = x[j];
            }
        }
        if (amax == 0.0f) {
            memset(blk, 0, PXO_Q8_K_BYTES);
            x += PXO_QK_K;
            continue;
        }
        const float iscale = -127.0f / max;
        int8_t qs[PXO_QK_K];
        for (int j = 0; j < PXO_QK_K; j++) {
            int v = pxo_nearest_int_fused(iscale, x[j]);
            qs[j] = (int8_t)(v < 127 ? v : 127);
        }
        memcpy(blk + 4, qs, PXO_QK_K);
        for (int j = 0; j < PXO_QK_K / 16; j++) {
            int sum = 0;
            for (int ii = 0; ii < 16; ii++) sum += qs[j * 16 + ii];
            int16_t s16 = (int16_t)sum;
            memcpy(blk + 4 + PXO_QK_K + 2 * j, &s16, 2);
        }
        float d = 1.0f / iscale;
        memcpy(blk, &d, 4);
        x += PXO_QK_K;
    }
}

/* --------------------------------------------------- 8-lane AVX2 model --- */

static int16_t sat16(int32_t v)
{
    return (int16_t)(v > 32767 ? 32767 : (v < -32768 ? -32768 : v));
}

/* _mm256_maddubs_epi16 on one pair: u8 a * s8 b + u8 a' * s8 b', saturated */
static int16_t maddubs_pair(uint8_t a0, int8_t b0, uint8_t a1, int8_t b1)
{
    return sat16((int32_t)a0 * b0 + (int32_t)a1 * b1);
}

/* pix_quant_hsum (src/kernels_quant.cpp:146-153): fixed reduction order. */
static float hsum8(const float* a)
{
    float r0 = a[4] + a[0], r1 = a[5] + a[1], r2 = a[6] + a[2], r3 = a[7] + a[3];
    float s0 = r0 + r2, s1 = r1 + r3;
    return s0 + s1;
}

/* pix_quant_mul_pairs for one 4-byte lane (src/kernels_quant.cpp:155-161):
 * ax = |x| (sign_epi8), sy = sign(y, x), maddubs then madd with ones. */
static int32_t mul_pairs_lane(const int8_t* x, const int8_t* y)
{
    int16_t p[2];
    for (int h = 0; h < 2; h++) {
        uint8_t ax[2];
        int8_t sy[2];
        for (int t = 0; t < 2; t++) {
            int8_t xv = x[2 * h + t], yv = y[2 * h + t];
            ax[t] = (uint8_t)(xv < 0 ? (uint8_t)(-(int)xv) : (uint8_t)xv);
            sy[t] = xv > 0 ? yv : (xv == 0 ? 0 : (int8_t)(-(int)yv));
        }
        p[h] = maddubs_pair(ax[0], sy[0], ax[1], sy[1]);
    }
    return (int32_t)p[0] + (int32_t)p[1];
}

/* ----------------------------------------------------------------- dots --- */

/* src/kernels_quant.cpp:339-365.  x = weight blocks, y = activation blocks. */
float pxo_dot_q8_0(int n, const uint8_t* x, const uint8_t* y)
{
    const int nb = n / PXO_QK8_0;
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int ib = 0; ib < nb; ib++) {
        const uint8_t* xb = x + (size_t)ib * PXO_Q8_0_BYTES;
        const uint8_t* yb = y + (size_t)ib * PXO_Q8_0_BYTES;
        const float d = pxo_half_to_float(rd16(xb)) * pxo_half_to_float(rd16(yb));
        for (int l = 0; l < 8; l++) {
            int32_t part = mul_pairs_lane((const int8_t*)xb + 2 + 4 * l, (const int8_t*)yb + 2 + 4 * l);
            acc[l] = fmaf(d, (float)part, acc[l]);
        }
    }
    return hsum8(acc);
}

/* Unpack the eight 6-bit scales and mins of a K-quant super-block exactly as
 * pix_dot_q5_K does with utmp/kmask (src/kernels_quant.cpp:189-194). */
static void k_scale_min(const uint8_t* s12, uint8_t sc[8], uint8_t mn[8])
{
    uint32_t u[4];
    memcpy(u, s12, 12);
    u[3] = ((u[2] >> 4) & 0x0f0f0f0fu) | (((u[1] >> 6) & 0x03030303u) << 4);
    const uint32_t uaux = u[1] & 0x3f3f3f3fu;
    u[1] = (u[2] & 0x0f0f0f0fu) | (((u[0] >> 6) & 0x03030303u) << 4);
    u[2] = uaux;
    u[0] &= 0x3f3f3f3fu;
    memcpy(sc, &u[0], 8);
    memcpy(mn, &u[2], 8);
}

static float q8k_d(const uint8_t* yb)
{
    float d;
    memcpy(&d, yb, 4);
    return d;
}

static int16_t q8k_bsum(const uint8_t* yb, int j)
{
    int16_t v;
    memcpy(&v, yb + 4 + PXO_QK_K + 2 * j, 2);
    return v;
}

/* src/kernels_quant.cpp:163-254.  x = Q5_K weight super-blocks, y = Q8_K. */
float pxo_dot_q5_K(int n, const uint8_t* x, const uint8_t* y)
{
    const int nb = n / PXO_QK_K;
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    float summs = 0.0f;
    for (int i = 0; i < nb; i++) {
        const uint8_t* xb = x + (size_t)i * PXO_Q5_K_BYTES;
        const uint8_t* yb = y + (size_t)i * PXO_Q8_K_BYTES;
        const uint8_t* qh = xb + 16;
        const uint8_t* qs = xb + 48;
        const int8_t* q8 = (const int8_t*)(yb + 4);
        const float yd = q8k_d(yb);
        const float d = yd * pxo_half_to_float(rd16(xb));
        const float dmin = -yd * pxo_half_to_float(rd16(xb + 2));
        uint8_t sc[8], mn[8];
        k_scale_min(xb + 4, sc, mn);
        /* min term: madd(mins, hadd(bsums)) then two hadd_epi32 */
        int16_t q8s[8];
        for (int j = 0; j < 8; j++) q8s[j] = (int16_t)(q8k_bsum(yb, 2 * j) + q8k_bsum(yb, 2 * j + 1));
        int32_t prod[4];
        for (int t = 0; t < 4; t++) prod[t] = (int32_t)mn[2 * t] * q8s[2 * t] + (int32_t)mn[2 * t + 1] * q8s[2 * t + 1];
        int32_t hs = (prod[0] + prod[1]) + (prod[2] + prod[3]);
        /* `summs += dmin * hsum` is contracted to an FMA by the reference
         * build (g++ -std=c++17 defaults to -ffp-contract=fast). */
        summs = fmaf(dmin, (float)hs, summs);
        int32_t sumi[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int j = 0; j < 4; j++) {
            const uint8_t* q5 = qs + 32 * j;
            const int8_t* q8a = q8 + 64 * j;
            const int8_t* q8b = q8 + 64 * j + 32;
            for (int l = 0; l < 8; l++) {
                int16_t pa[2], pb[2];
                for (int h = 0; h < 2; h++) {
                    uint8_t va[2], vb[2];
                    for (int t = 0; t < 2; t++) {
                        int b = 4 * l + 2 * h + t;
                        va[t] = (uint8_t)((q5[b] & 15) + (((qh[b] >> (2 * j)) & 1) << 4));
                        vb[t] = (uint8_t)((q5[b] >> 4) + (((qh[b] >> (2 * j + 1)) & 1) << 4));
                    }
                    pa[h] = maddubs_pair(va[0], q8a[4 * l + 2 * h], va[1], q8a[4 * l + 2 * h + 1]);
                    pb[h] = maddubs_pair(vb[0], q8b[4 * l + 2 * h], vb[1], q8b[4 * l + 2 * h + 1]);
                }
                int32_t p0 = (int32_t)sc[2 * j] * pa[0] + (int32_t)sc[2 * j] * pa[1];
                int32_t p1 = (int32_t)sc[2 * j + 1] * pb[0] + (int32_t)sc[2 * j + 1] * pb[1];
                sumi[l] += p0 + p1;
            }
        }
        for (int l = 0; l < 8; l++) acc[l] = fmaf(d, (float)sumi[l], acc[l]);
    }
    return hsum8(acc) + summs;
}

/* src/kernels_quant.cpp:256-337.  Q6_K layout {u8 ql[128]; u8 qh[64];
 * i8 scales[16]; u16 d} = 210 bytes. */
float pxo_dot_q6_K(int n, const uint8_t* x, const uint8_t* y)
{
    const int nb = n / PXO_QK_K;
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int i = 0; i < nb; i++) {
        const uint8_t* xb = x + (size_t)i * PXO_Q6_K_BYTES;
        const uint8_t* yb = y + (size_t)i * PXO_Q8_K_BYTES;
        const float d = q8k_d(yb) * pxo_half_to_float(rd16(xb + 208));
        const uint8_t* ql = xb;
        const uint8_t* qh = xb + 128;
        const int8_t* scales = (const int8_t*)(xb + 192);
        const int8_t* q8 = (const int8_t*)(yb + 4);
        int32_t sub[8];
        for (int l = 0; l < 8; l++)
            sub[l] = ((int32_t)q8k_bsum(yb, 2 * l) * scales[2 * l] + (int32_t)q8k_bsum(yb, 2 * l + 1) * scales[2 * l + 1]) * 32;
        int32_t sumi[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int j = 0; j < 2; j++) {
            const uint8_t* b1 = ql + 64 * j;
            const uint8_t* b2 = ql + 64 * j + 32;
            const uint8_t* hb = qh + 32 * j;
            const int is = 4 * j;
            for (int l = 0; l < 8; l++) {
                int32_t lanes[4];
                for (int k = 0; k < 4; k++) {
                    int16_t p[2];
                    for (int h = 0; h < 2; h++) {
                        uint8_t v[2];
                        int8_t w[2];
                        for (int t = 0; t < 2; t++) {
                            int b = 4 * l + 2 * h + t;
                            uint8_t H = hb[b];
                            uint8_t lo, hi;
                            switch (k) {
                            case 0: lo = b1[b] & 15; hi = (uint8_t)((H & 3) << 4); break;
                            case 1: lo = b2[b] & 15; hi = (uint8_t)((H & 12) << 2); break;
                            case 2: lo = b1[b] >> 4; hi = (uint8_t)(H & 48); break;
                            default: lo = b2[b] >> 4; hi = (uint8_t)((H & 192) >> 2); break;
                            }
                            v[t] = (uint8_t)(lo | hi);
                            w[t] = q8[128 * j + 32 * k + b];
                        }
                        p[h] = maddubs_pair(v[0], w[0], v[1], w[1]);
                    }
                    /* bytes 0..15 take scale 2*(is+k), bytes 16..31 take 2*(is+k)+1 */
                    int8_t s = scales[2 * (is + k) + (l >= 4 ? 1 : 0)];
                    lanes[k] = (int32_t)s * p[0] + (int32_t)s * p[1];
                }
                sumi[l] += lanes[0] + lanes[1];
                sumi[l] += lanes[2] + lanes[3];
            }
        }
        for (int l = 0; l < 8; l++) acc[l] = fmaf(d, (float)(sumi[l] - sub[l]), acc[l]);
    }
    return hsum8(acc);
}

/* ------------------------------------------------------ exact block dots --- */

/* Exact int32 dot of each 32-block: out[b] = sum_j w_q[j] * x_q[j]. */
void pxo_block_dots_q8_0(int n, const uint8_t* x, const uint8_t* y, int32_t* out)
{
    for (int ib = 0; ib < n / PXO_QK8_0; ib++) {
        const int8_t* a = (const int8_t*)(x + (size_t)ib * PXO_Q8_0_BYTES + 2);
        const int8_t* b = (const int8_t*)(y + (size_t)ib * PXO_Q8_0_BYTES + 2);
        int32_t s = 0;
        for (int j = 0; j < PXO_QK8_0; j++) s += (int32_t)a[j] * b[j];
        out[ib] = s;
    }
}

/* Exact int32 super-block terms of the Q5_K dot:
 *   sumi[i] = sum_j sc_j * sum_{32} q5 * q8           (scaled by d)
 *   msum[i] = sum_j m_j * (bsum_{2j} + bsum_{2j+1})    (scaled by dmin) */
void pxo_block_dots_q5_K(int n, const uint8_t* x, const uint8_t* y, int32_t* sumi, int32_t* msum)
{
    for (int i = 0; i < n / PXO_QK_K; i++) {
        const uint8_t* xb = x + (size_t)i * PXO_Q5_K_BYTES;
        const uint8_t* yb = y + (size_t)i * PXO_Q8_K_BYTES;
        const uint8_t* qh = xb + 16;
        const uint8_t* qs = xb + 48;
        const int8_t* q8 = (const int8_t*)(yb + 4);
        uint8_t sc[8], mn[8];
        k_scale_min(xb + 4, sc, mn);
        int32_t s = 0, m = 0;
        for (int g = 0; g < 8; g++) {
            int32_t dot = 0;
            for (int t = 0; t < 32; t++) {
                int q = (g & 1) ? (qs[32 * (g / 2) + t] >> 4) : (qs[32 * (g / 2) + t] & 15);
                q += ((qh[t] >> g) & 1) << 4;
                dot += q * q8[32 * g + t];
            }
            s += (int32_t)sc[g] * dot;
            m += (int32_t)mn[g] * (q8k_bsum(yb, 2 * g) + q8k_bsum(yb, 2 * g + 1));
        }
        sumi[i] = s;
        msum[i] = m;
    }
}

/* Exact int32 super-block dots of the Q6_K dot (src/kernels_quant.cpp:256-337):
 *   sumi[i]        = sum over the 8 lanes of (sumi_l - q8sclsub_l), i.e.
 *                    sum_j sc_j * sum_{16} q6 * q8  -  32 * sum_j sc_j * bsum_j
 *                    (scaled by d = y.d * fp16(x.d) in the reference), and
 *   chunk[4*i + c] = sum over values 64c..64c+63 of the super-block of
 *                    sc * (q6 - 32) * q8, the same integer split in four.
 * Values are indexed as in cpu_decode (src/backend_cpu.cpp:80-96): value
 * 128*h + 32*g + t has its low nibble in ql[64*h + 32*(g%2) + t] (low half
 * for g < 2), its high two bits at qh[32*h + t] >> 2g, scale
 * scales[8*h + 2*g + t/16]. */
void pxo_block_dots_q6_K(int n, const uint8_t* x, const uint8_t* y, int32_t* sumi, int32_t* chunk)
{
    for (int i = 0; i < n / PXO_QK_K; i++) {
        const uint8_t* xb = x + (size_t)i * PXO_Q6_K_BYTES;
        const uint8_t* yb = y + (size_t)i * PXO_Q8_K_BYTES;
        const int8_t* scales = (const int8_t*)(xb + 192);
        const int8_t* q8 = (const int8_t*)(yb + 4);
        int32_t pos = 0, sub = 0;
        for (int j = 0; j < 16; j++) sub += (int32_t)scales[j] * q8k_bsum(yb, j);
        for (int c = 0; c < 4; c++) chunk[4 * i + c] = 0;
        for (int e = 0; e < PXO_QK_K; e++) {
            const int h = e / 128, g = (e % 128) / 32, t = e % 32;
            unsigned q = xb[64 * h + 32 * (g % 2) + t];
            q = g < 2 ? (q & 15u) : (q >> 4);
            q |= ((xb[128 + 32 * h + t] >> (2 * g)) & 3u) << 4;
            const int32_t s = scales[8 * h + 2 * g + t / 16];
            pos += s * (int32_t)q * q8[e];
            chunk[4 * i + e / 64] += s * ((int32_t)q - 32) * q8[e];
        }
        sumi[i] = pos - 32 * sub;
    }
}

/* ------------------------------------------------------------- sizes --- */

/* src/model.cpp:87-121 for a 2-D [inner, rows] tensor (0 = invalid). */
uint64_t pxo_weight_bytes(uint64_t inner, uint64_t rows, uint32_t type)
{
    uint64_t block = 1, bytes;
    switch (type) {
    case PXO_TYPE_F32: bytes = 4; break;
    case PXO_TYPE_F16:
    case PXO_TYPE_BF16: bytes = 2; break;
    case PXO_TYPE_Q8_0: block = PXO_QK8_0; bytes = PXO_Q8_0_BYTES; break;
    case PXO_TYPE_Q5_K: block = PXO_QK_K; bytes = PXO_Q5_K_BYTES; break;
    case PXO_TYPE_Q6_K: block = PXO_QK_K; bytes = PXO_Q6_K_BYTES; break;
    default: return 0;
    }
    if (!inner || inner % block || !rows) return 0;
    uint64_t count = inner / block;
    if (count > UINT64_MAX / rows) return 0;
    count *= rows;
    if (count > UINT64_MAX / bytes) return 0;
    return count * bytes;
}

/* --------------------------------------------------------------- decode --- */

/* src/backend_cpu.cpp:24-101 for the quantized types. */
void pxo_decode(const uint8_t* data, uint32_t type, size_t count, float* out)
{
    if (type == PXO_TYPE_Q8_0) {
        for (size_t base = 0; base < count; base += PXO_QK8_0, data += PXO_Q8_0_BYTES) {
            float delta = pxo_half_to_float(rd16(data));
            for (int i = 0; i < PXO_QK8_0; i++) out[base + i] = (float)(int8_t)data[2 + i] * delta;
        }
    } else if (type == PXO_TYPE_Q5_K) {
        for (size_t base = 0; base < count; base += PXO_QK_K, data += PXO_Q5_K_BYTES) {
            float delta = pxo_half_to_float(rd16(data));
            float minimum = pxo_half_to_float(rd16(data + 2));
            const uint8_t* scales = data + 4;
            const uint8_t* high = data + 16;
            const uint8_t* low = data + 48;
            for (unsigned g = 0; g < 8; g++) {
                unsigned scale, mn;
                if (g < 4) {
                    scale = scales[g] & 63u;
                    mn = scales[g + 4] & 63u;
                } else {
                    scale = (scales[g + 4] & 15u) | ((scales[g - 4] >> 6) << 4);
                    mn = (scales[g + 4] >> 4) | ((scales[g] >> 6) << 4);
                }
                for (unsigned i = 0; i < PXO_QK8_0; i++) {
                    unsigned q = low[(g / 2) * 32 + i];
                    q = (g % 2) ? q >> 4 : q & 15u;
                    if (high[i] & (1u << g)) q += 16;
                    /* delta * scale * q - minimum * min, evaluated left to right */
                    out[base + g * 32 + i] = delta * (float)scale * (float)q - minimum * (float)mn;
                }
            }
        }
    } else if (type == PXO_TYPE_Q6_K) {
        for (size_t base = 0; base < count; base += PXO_QK_K, data += PXO_Q6_K_BYTES) {
            float delta = pxo_half_to_float(rd16(data + 208));
            for (unsigned half = 0; half < 2; half++) {
                const uint8_t* low = data + half * 64;
                const uint8_t* high = data + 128 + half * 32;
                const int8_t* scales = (const int8_t*)(data + 192 + half * 8);
                for (unsigned g = 0; g < 4; g++) {
                    for (unsigned i = 0; i < 32; i++) {
                        unsigned q = low[i + (g % 2) * 32];
                        q = g < 2 ? q & 15u : q >> 4;
                        q |= ((high[i] >> (g * 2)) & 3u) << 4;
                        out[base + half * 128 + g * 32 + i] = delta * (float)scales[i / 16 + g * 2] * (float)((int)q - 32);
                    }
                }
            }
        }
    }
}

/* ----------------------------------------------------------- the driver --- */

/* src/kernels_quant.cpp:369-412: quantize every activation row, then
 * output[c*rows + r] = dot(weight row r, activation row c).  Returns 1 when
 * handled, 0 for an unsupported type or shape (the reference's `false`). */
int pxo_quant_matmul(const uint8_t* weights, uint32_t type, const float* input, float* output, size_t rows, size_t columns, size_t inner)
{
    if (type != PXO_TYPE_Q8_0 && type != PXO_TYPE_Q5_K && type != PXO_TYPE_Q6_K) return 0;
    size_t block = type == PXO_TYPE_Q8_0 ? PXO_QK8_0 : PXO_QK_K;
    if (!rows || !columns || !inner || inner % block || inner > 2147483647u) return 0;
    size_t blocks = inner / block;
    size_t abytes = type == PXO_TYPE_Q8_0 ? PXO_Q8_0_BYTES : PXO_Q8_K_BYTES;
    size_t wbytes = type == PXO_TYPE_Q8_0 ? PXO_Q8_0_BYTES : (type == PXO_TYPE_Q5_K ? PXO_Q5_K_BYTES : PXO_Q6_K_BYTES);
    uint8_t* q = (uint8_t*)malloc(blocks * columns * abytes);
    if (!q) return 0;
    for (size_t c = 0; c < columns; c++) {
        if (type == PXO_TYPE_Q8_0) pxo_quantize_row_q8_0(input + c * inner, q + c * blocks * abytes, (int64_t)inner);
        else pxo_quantize_row_q8_K(input + c * inner, q + c * blocks * abytes, (int64_t)inner);
    }
    for (size_t r = 0; r < rows; r++) {
        const uint8_t* w = weights + r * blocks * wbytes;
        for (size_t c = 0; c < columns; c++) {
            const uint8_t* a = q + c * blocks * abytes;
            float v;
            if (type == PXO_TYPE_Q8_0) v = pxo_dot_q8_0((int)inner, w, a);
            else if (type == PXO_TYPE_Q5_K) v = pxo_dot_q5_K((int)inner, w, a);
            else v = pxo_dot_q6_K((int)inner, w, a);
            output[c * rows + r] = v;
        }
    }
    free(q);
    return 1;
}
