/*
 * qo_kernels.c -- CPU restatement of qma's numeric kernels (TEST
 * INFRASTRUCTURE: the parity checker for the CUDA engine; see qma_oracle.h).
 *
 * Restated reference functions, each in the reference's operation order:
 *   half_to_float / float_to_half   qma.h:101-152 (AArch64 FCVT semantics)
 *   quantize_row_q8k                q8k.c:34-85
 *   dot_q4_K_q8k                    q8k.c:89-131
 *   dot_q4_K_gateup_q8k             q8k.c:140-207
 *   dot_q6_K_q8k                    q8k.c:210-262
 *   dequantize_row_q4_K / _q6_K     quants.c:29-75
 *   matmul (q8k path)               nn.c:261-345
 * plus the engine's own Q8_0 weight dot, weight quantizers and synthetic
 * weight generator (the reference has none of these).
 */
#include "qma_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------- parallel for --
 * Independent loops (rows of a matmul, expert tasks, recurrent heads) are
 * split over a few pthreads.  Every output element is still computed by one
 * thread in the reference's order, so results do not depend on the count. */
static int g_qo_threads = 1;

void qo_set_threads(int n) { g_qo_threads = n < 1 ? 1 : (n > 64 ? 64 : n); }

typedef struct {
    void (*fn)(void *, int, int);
    void *ctx;
    int i0, i1;
} qo_pfor_job;

static void *qo_pfor_run(void *a)
{
    qo_pfor_job *j = a;
    if (j->i1 > j->i0) j->fn(j->ctx, j->i0, j->i1);
    return NULL;
}

void qo_pfor(int n, void (*fn)(void *, int, int), void *ctx)
{
    int nt = g_qo_threads;
    if (nt > n) nt = n;
    if (nt <= 1) {
        if (n > 0) fn(ctx, 0, n);
        return;
    }
    pthread_t th[64];
    qo_pfor_job jobs[64];
    for (int k = 0; k < nt; k++) {
        jobs[k].fn = fn;
        jobs[k].ctx = ctx;
        jobs[k].i0 = (int)((long)n * k / nt);
        jobs[k].i1 = (int)((long)n * (k + 1) / nt);
    }
    for (int k = 1; k < nt; k++) pthread_create(&th[k], NULL, qo_pfor_run, &jobs[k]);
    qo_pfor_run(&jobs[0]);
    for (int k = 1; k < nt; k++) pthread_join(th[k], NULL);
}

/* ---------------------------------------------------------------- fp16 -- */
float qo_half_to_float(uint16_t h)
{
    uint32_t sign = (uint32_t)(h & 0x8000) << 16;
    uint32_t exp = (h >> 10) & 0x1f;
    uint32_t man = h & 0x3ff;
    uint32_t f;
    if (exp == 0) {
        if (man == 0) {
            f = sign;
        } else {
            exp = 127 - 15 + 1;
            while (!(man & 0x400)) { man <<= 1; exp--; }
            man &= 0x3ff;
            f = sign | (exp << 23) | (man << 13);
        }
    } else if (exp == 0x1f) {
        f = sign | 0x7f800000u | (man << 13);
    } else {
        f = sign | ((exp + (127 - 15)) << 23) | (man << 13);
    }
    float r;
    memcpy(&r, &f, 4);
    return r;
}

/* IEEE binary32 -> binary16, round to nearest, ties to even. */
uint16_t qo_float_to_half(float x)
{
    uint32_t f;
    memcpy(&f, &x, 4);
    const uint32_t sign = (f >> 16) & 0x8000;
    const uint32_t exp = (f >> 23) & 0xff;
    const uint32_t man = f & 0x7fffff;
    if (exp == 0xff) return (uint16_t)(sign | 0x7c00 | (man ? 0x200 : 0));
    int32_t e = (int32_t)exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7c00);
    if (e <= 0) {
        /* subnormal half: value = m * 2^(exp-150), unit 2^-24 */
        const int shift = 126 - (int)exp;
        if (shift > 24) return (uint16_t)sign;
        const uint32_t m = man | 0x800000;
        uint32_t hm = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1);
        const uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (hm & 1))) hm++;
        return (uint16_t)(sign | hm);
    }
    uint32_t hm = man >> 13;
    const uint32_t rem = man & 0x1fff;
    if (rem > 0x1000 || (rem == 0x1000 && (hm & 1))) hm++;
    if (hm == 0x400) {
        hm = 0;
        e++;
        if (e >= 31) return (uint16_t)(sign | 0x7c00);
    }
    return (uint16_t)(sign | ((uint32_t)e << 10) | hm);
}

static inline float h2f_at(const uint8_t *p)
{
    uint16_t h;
    memcpy(&h, p, 2);
    return qo_half_to_float(h);
}

size_t qo_row_bytes(int wtype, int n_in)
{
    switch (wtype) {
    case QO_Q4_K: return (size_t)(n_in / QO_QK_K) * QO_Q4K_BYTES;
    case QO_Q6_K: return (size_t)(n_in / QO_QK_K) * QO_Q6K_BYTES;
    case QO_Q8_0: return (size_t)(n_in / 32) * QO_Q80_BYTES;
    case QO_F32:  return (size_t)n_in * 4;
    default:      return 0;
    }
}

/* ------------------------------------------------------------ Q8_K quant -- */
void qo_q8k_quant(const float *x, int n, int8_t *xq, float *xd, int16_t *xsum)
{
    const int nb = n / QO_QK_K;
    for (int i = 0; i < nb; i++) {
        const float *xs = x + (size_t)i * QO_QK_K;
        int8_t *q = xq + (size_t)i * QO_QK_K;
        int16_t *sp = xsum + (size_t)i * (QO_QK_K / 16);
        float amax = 0.0f;
        for (int j = 0; j < QO_QK_K; j++) {
            const float a = fabsf(xs[j]);
            if (a > amax) amax = a;
        }
        const float s = amax > 0.0f ? amax / 127.0f : 1.0f;
        xd[i] = s;
        const float inv = 1.0f / s;
        for (int j = 0; j < QO_QK_K; j += 16) {
            int sum = 0;
            for (int l = 0; l < 16; l++) {
                float v = roundf(xs[j + l] * inv);   /* FCVTAS: ties away */
                int iv = (int)v;
                if (iv > 127) iv = 127;
                if (iv < -127) iv = -127;
                q[j + l] = (int8_t)iv;
                sum += iv;
            }
            sp[j / 16] = (int16_t)sum;
        }
    }
}

/* --------------------------------------------------------------- Q4_K dot -- */
static inline void scale_min_k4(int j, const uint8_t *q, uint8_t *d, uint8_t *m)
{
    if (j < 4) {
        *d = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *d = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        *m = (q[j + 4] >> 4) | ((q[j - 0] >> 6) << 4);
    }
}

float qo_dot_q4k(const uint8_t *row, const int8_t *xq, const float *xd,
                 const int16_t *xsum, int n, int32_t *isum)
{
    const int nb = n / QO_QK_K;
    float total = 0.0f;
    for (int i = 0; i < nb; i++) {
        const uint8_t *b = row + (size_t)i * QO_Q4K_BYTES;
        const float d = h2f_at(b);
        const float mn = h2f_at(b + 2);
        const uint8_t *sc = b + 4;
        const uint8_t *q = b + 16;
        const float xd_blk = xd[i];
        const int8_t *xp = xq + (size_t)i * QO_QK_K;
        const int16_t *sp = xsum + (size_t)i * (QO_QK_K / 16);
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        float bias = 0.0f;
        int is = 0;
        for (int g = 0; g < 4; g++) {
            uint8_t s1, m1, s2, m2;
            scale_min_k4(is + 0, sc, &s1, &m1);
            scale_min_k4(is + 1, sc, &s2, &m2);
            const float d1 = d * s1, mm1 = mn * m1;
            const float d2 = d * s2, mm2 = mn * m2;
            int32_t pn[4], ph[4];
            for (int l = 0; l < 4; l++) {
                int32_t a = 0, h = 0;
                for (int j = 0; j < 4; j++) {
                    a += (int32_t)(q[4 * l + j] & 0xF) * xp[4 * l + j];
                    a += (int32_t)(q[16 + 4 * l + j] & 0xF) * xp[16 + 4 * l + j];
                    h += (int32_t)(q[4 * l + j] >> 4) * xp[32 + 4 * l + j];
                    h += (int32_t)(q[16 + 4 * l + j] >> 4) * xp[48 + 4 * l + j];
                }
                pn[l] = a;
                ph[l] = h;
            }
            if (isum) {
                isum[(size_t)i * 8 + 2 * g] = pn[0] + pn[1] + pn[2] + pn[3];
                isum[(size_t)i * 8 + 2 * g + 1] = ph[0] + ph[1] + ph[2] + ph[3];
            }
            const float sx0 = (float)(sp[0] + sp[1]);
            const float sx1 = (float)(sp[2] + sp[3]);
            const float f1 = d1 * xd_blk, f2 = d2 * xd_blk;
            for (int l = 0; l < 4; l++) acc[l] = fmaf((float)pn[l], f1, acc[l]);
            for (int l = 0; l < 4; l++) acc[l] = fmaf((float)ph[l], f2, acc[l]);
            bias += (mm1 * sx0 + mm2 * sx1) * xd_blk;
            q += 32;
            xp += 64;
            sp += 4;
            is += 2;
        }
        const float s01 = acc[0] + acc[1];
        const float s23 = acc[2] + acc[3];
        total += (s01 + s23) - bias;
    }
    return total;
}

void qo_gateup_q4k(const uint8_t *g, const uint8_t *u, const int8_t *xq,
                   const float *xd, const int16_t *xsum, int n,
                   float *gate, float *up)
{
    /* dot_q4_K_gateup_q8k performs, per row, exactly the arithmetic of
       dot_q4_K_q8k (same lane partials, same fused multiply-adds, same bias
       and total order); fusing only shares the activation loads. */
    *gate = qo_dot_q4k(g, xq, xd, xsum, n, NULL);
    *up = qo_dot_q4k(u, xq, xd, xsum, n, NULL);
}

/* --------------------------------------------------------------- Q6_K dot -- */
static inline int q6_value(const uint8_t *ql, const uint8_t *qh, int w)
{
    /* w in [0,128) inside one 128-lane half (dequantize_row_q6_K order) */
    const int L = w & 63, hi = w >> 6;
    const int lo4 = hi ? (ql[L] >> 4) : (ql[L] & 0xF);
    const int shift = 2 * ((L >> 5) + 2 * hi);
    const int h2 = (qh[L & 31] >> shift) & 3;
    return (lo4 | (h2 << 4)) - 32;
}

float qo_dot_q6k(const uint8_t *row, const int8_t *xq, const float *xd, int n,
                 int32_t *isum)
{
    const int nb = n / QO_QK_K;
    float total = 0.0f;
    for (int i = 0; i < nb; i++) {
        const uint8_t *b = row + (size_t)i * QO_Q6K_BYTES;
        const uint8_t *ql = b;
        const uint8_t *qh = b + 128;
        const int8_t *sc = (const int8_t *)(b + 192);
        const float d = h2f_at(b + 208);
        const float xd_blk = xd[i];
        const int8_t *xp = xq + (size_t)i * QO_QK_K;
        int32_t acc = 0;
        for (int j = 0; j < 2; j++) {
            for (int g = 0; g < 8; g++) {
                int32_t p = 0;
                for (int l = 0; l < 16; l++)
                    p += q6_value(ql, qh, g * 16 + l) * xp[g * 16 + l];
                acc += p * sc[g];
            }
            ql += 64;
            qh += 32;
            sc += 8;
            xp += 128;
        }
        if (isum) isum[i] = acc;
        total += d * xd_blk * (float)acc;
    }
    return total;
}

/* --------------------------------------------------------------- Q8_0 dot -- */
float qo_dot_q80(const uint8_t *row, const int8_t *xq, const float *xd, int n,
                 int32_t *isum)
{
    const int nsb = n / QO_QK_K;
    float total = 0.0f;
    for (int i = 0; i < nsb; i++) {
        float acc = 0.0f;
        for (int b = 0; b < 8; b++) {
            const uint8_t *blk = row + ((size_t)i * 8 + b) * QO_Q80_BYTES;
            const int8_t *q = (const int8_t *)(blk + 2);
            const int8_t *xp = xq + (size_t)i * QO_QK_K + b * 32;
            int32_t s = 0;
            for (int l = 0; l < 32; l++) s += (int32_t)q[l] * xp[l];
            if (isum) isum[(size_t)i * 8 + b] = s;
            acc += (float)s * h2f_at(blk);
        }
        total += acc * xd[i];
    }
    return total;
}

float qo_dot(const uint8_t *row, int wtype, const int8_t *xq, const float *xd,
             const int16_t *xsum, int n)
{
    if (wtype == QO_Q4_K) return qo_dot_q4k(row, xq, xd, xsum, n, NULL);
    if (wtype == QO_Q6_K) return qo_dot_q6k(row, xq, xd, n, NULL);
    if (wtype == QO_Q8_0) return qo_dot_q80(row, xq, xd, n, NULL);
    return 0.0f;
}

/* ------------------------------------------------------------ dequantize -- */
void qo_dequant_row(const uint8_t *row, int wtype, float *y, int n)
{
    if (wtype == QO_Q4_K) {
        for (int i = 0; i < n / QO_QK_K; i++) {
            const uint8_t *b = row + (size_t)i * QO_Q4K_BYTES;
            const float d = h2f_at(b), mn = h2f_at(b + 2);
            const uint8_t *q = b + 16;
            int is = 0;
            for (int j = 0; j < QO_QK_K; j += 64) {
                uint8_t sc, m;
                scale_min_k4(is + 0, b + 4, &sc, &m);
                const float d1 = d * sc, m1 = mn * m;
                scale_min_k4(is + 1, b + 4, &sc, &m);
                const float d2 = d * sc, m2 = mn * m;
                for (int l = 0; l < 32; l++) *y++ = d1 * (q[l] & 0xF) - m1;
                for (int l = 0; l < 32; l++) *y++ = d2 * (q[l] >> 4) - m2;
                q += 32;
                is += 2;
            }
        }
    } else if (wtype == QO_Q6_K) {
        for (int i = 0; i < n / QO_QK_K; i++) {
            const uint8_t *b = row + (size_t)i * QO_Q6K_BYTES;
            const float d = h2f_at(b + 208);
            const int8_t *sc = (const int8_t *)(b + 192);
            for (int half = 0; half < 2; half++) {
                const uint8_t *ql = b + 64 * half;
                const uint8_t *qh = b + 128 + 32 * half;
                for (int w = 0; w < 128; w++)
                    y[w] = d * sc[8 * half + w / 16] * q6_value(ql, qh, w);
                y += 128;
            }
        }
    } else if (wtype == QO_Q8_0) {
        for (int i = 0; i < n / 32; i++) {
            const uint8_t *b = row + (size_t)i * QO_Q80_BYTES;
            const float d = h2f_at(b);
            const int8_t *q = (const int8_t *)(b + 2);
            for (int l = 0; l < 32; l++) *y++ = d * q[l];
        }
    } else if (wtype == QO_F32) {
        memcpy(y, row, (size_t)n * 4);
    }
}

/* ---------------------------------------------------------------- matmul -- */
void qo_matmul(const float *x, const uint8_t *W, int n_in, int n_out, int T,
               int wtype, float *out)
{
    int8_t *xq = malloc((size_t)T * n_in);
    float *xd = malloc((size_t)T * (n_in / QO_QK_K) * sizeof(float));
    int16_t *xs = malloc((size_t)T * (n_in / 16) * sizeof(int16_t));
    for (int t = 0; t < T; t++)
        qo_q8k_quant(x + (size_t)t * n_in, n_in, xq + (size_t)t * n_in,
                     xd + (size_t)t * (n_in / QO_QK_K), xs + (size_t)t * (n_in / 16));
    const size_t rb = qo_row_bytes(wtype, n_in);
    for (int r = 0; r < n_out; r++) {
        const uint8_t *wr = W + (size_t)r * rb;
        for (int t = 0; t < T; t++)
            out[(size_t)t * n_out + r] =
                qo_dot(wr, wtype, xq + (size_t)t * n_in, xd + (size_t)t * (n_in / QO_QK_K),
                       xs + (size_t)t * (n_in / 16), n_in);
    }
    free(xq);
    free(xd);
    free(xs);
}

/* ------------------------------------------------------------ quantizers --
 * The engine's own weight quantizers (the reference ships none).  They are
 * written with plain IEEE single operations (no fused multiply-add, exact
 * division, roundf ties away from zero) so the CUDA synthetic generator
 * reproduces them bit for bit. */
static inline int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

void qo_quantize_q4k(const float *x, uint8_t *blk)
{
    float scale[8], mins[8];
    float max_scale = 0.0f, max_min = 0.0f;
    for (int j = 0; j < 8; j++) {
        float mn = x[32 * j], mx = x[32 * j];
        for (int i = 1; i < 32; i++) {
            const float v = x[32 * j + i];
            if (v < mn) mn = v;
            if (v > mx) mx = v;
        }
        if (mn > 0.0f) mn = 0.0f;
        scale[j] = (mx - mn) / 15.0f;
        mins[j] = -mn;
        if (scale[j] > max_scale) max_scale = scale[j];
        if (mins[j] > max_min) max_min = mins[j];
    }
    const uint16_t dh = qo_float_to_half(max_scale / 63.0f);
    const uint16_t mh = qo_float_to_half(max_min / 63.0f);
    const float dq = qo_half_to_float(dh), mq = qo_half_to_float(mh);
    uint8_t sc[8], mm[8];
    for (int j = 0; j < 8; j++) {
        sc[j] = (uint8_t)(dq > 0.0f ? clampi((int)roundf(scale[j] / dq), 0, 63) : 0);
        mm[j] = (uint8_t)(mq > 0.0f ? clampi((int)roundf(mins[j] / mq), 0, 63) : 0);
    }
    memcpy(blk, &dh, 2);
    memcpy(blk + 2, &mh, 2);
    uint8_t *s = blk + 4;
    for (int j = 0; j < 4; j++) {
        s[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
        s[j + 4] = (uint8_t)((mm[j] & 63) | ((mm[j + 4] >> 4) << 6));
        s[j + 8] = (uint8_t)((sc[j + 4] & 0xF) | ((mm[j + 4] & 0xF) << 4));
    }
    uint8_t *qs = blk + 16;
    for (int g = 0; g < 4; g++) {
        uint8_t nib[2][32];
        for (int h = 0; h < 2; h++) {
            const int j = 2 * g + h;
            const float ds = dq * (float)sc[j];
            const float dm = mq * (float)mm[j];
            const float ids = ds > 0.0f ? 1.0f / ds : 0.0f;
            for (int i = 0; i < 32; i++) {
                const float t = x[32 * j + i] + dm;
                nib[h][i] = (uint8_t)(ds > 0.0f ? clampi((int)roundf(t * ids), 0, 15) : 0);
            }
        }
        for (int l = 0; l < 32; l++) qs[32 * g + l] = (uint8_t)(nib[0][l] | (nib[1][l] << 4));
    }
}

void qo_quantize_q6k(const float *x, uint8_t *blk)
{
    float scale[16];
    float max_scale = 0.0f;
    for (int g = 0; g < 16; g++) {
        float amax = 0.0f;
        for (int i = 0; i < 16; i++) {
            const float a = fabsf(x[16 * g + i]);
            if (a > amax) amax = a;
        }
        scale[g] = amax / 31.0f;
        if (scale[g] > max_scale) max_scale = scale[g];
    }
    const uint16_t dh = qo_float_to_half(max_scale / 127.0f);
    const float dq = qo_half_to_float(dh);
    int8_t sc[16];
    uint8_t u[256];
    for (int g = 0; g < 16; g++) {
        sc[g] = (int8_t)(dq > 0.0f ? clampi((int)roundf(scale[g] / dq), -128, 127) : 0);
        const float ds = dq * (float)sc[g];
        const float ids = ds > 0.0f ? 1.0f / ds : 0.0f;
        for (int i = 0; i < 16; i++) {
            const int q = ds > 0.0f ? clampi((int)roundf(x[16 * g + i] * ids), -32, 31) : 0;
            u[16 * g + i] = (uint8_t)(q + 32);
        }
    }
    uint8_t *ql = blk, *qh = blk + 128;
    memset(blk, 0, 192);
    for (int half = 0; half < 2; half++) {
        for (int w = 0; w < 128; w++) {
            const int v = u[128 * half + w];
            const int L = w & 63, hi = w >> 6;
            const int shift = 2 * ((L >> 5) + 2 * hi);
            if (hi) ql[64 * half + L] |= (uint8_t)((v & 0xF) << 4);
            else    ql[64 * half + L] |= (uint8_t)(v & 0xF);
            qh[32 * half + (L & 31)] |= (uint8_t)(((v >> 4) & 3) << shift);
        }
    }
    memcpy(blk + 192, sc, 16);
    memcpy(blk + 208, &dh, 2);
}

void qo_quantize_q80(const float *x, uint8_t *blk)
{
    float amax = 0.0f;
    for (int i = 0; i < 32; i++) {
        const float a = fabsf(x[i]);
        if (a > amax) amax = a;
    }
    const uint16_t dh = qo_float_to_half(amax / 127.0f);
    const float dq = qo_half_to_float(dh);
    const float id = dq > 0.0f ? 1.0f / dq : 0.0f;
    memcpy(blk, &dh, 2);
    int8_t *q = (int8_t *)(blk + 2);
    for (int i = 0; i < 32; i++) q[i] = (int8_t)clampi((int)roundf(x[i] * id), -127, 127);
}

/* --------------------------------------------------------- synthetic model */
uint64_t qo_name_key(const char *name, uint64_t seed)
{
    uint64_t h = 0xcbf29ce484222325ull;             /* FNV-1a 64 */
    for (const char *p = name; *p; p++) {
        h ^= (uint8_t)*p;
        h *= 0x100000001b3ull;
    }
    return h ^ (seed * 0x9E3779B97F4A7C15ull);
}

static inline uint64_t splitmix64(uint64_t z)
{
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* Irwin-Hall(4) standard normal from one 64-bit hash: four 16-bit uniforms
   summed exactly in integers, centred, scaled by sqrt(3)/65536. */
static inline float synth_normal(uint64_t key, uint64_t idx)
{
    const uint64_t h = splitmix64(key + idx);
    const int s = (int)(h & 0xffff) + (int)((h >> 16) & 0xffff) +
                  (int)((h >> 32) & 0xffff) + (int)(h >> 48);
    return (float)(s - 131070) * 0x1.bb67aep-16f;
}

float qo_synth_value(uint64_t key, uint64_t idx, float mu, float sigma)
{
    const float t = sigma * synth_normal(key, idx);
    return mu + t;
}

/* tensor kinds: distribution of the pre-quantization values */
enum { KIND_W = 0, KIND_NORM, KIND_CONV, KIND_DT, KIND_A };

static int tensor_kind(const char *name)
{
    const size_t n = strlen(name);
    const char *sfx_norm = "norm.weight";
    const size_t ln = strlen(sfx_norm);
    if (n >= ln && strcmp(name + n - ln, sfx_norm) == 0) return KIND_NORM;
    if (strstr(name, "ssm_conv1d")) return KIND_CONV;
    if (strstr(name, "ssm_dt")) return KIND_DT;
    if (n >= 5 && strcmp(name + n - 5, "ssm_a") == 0) return KIND_A;
    return KIND_W;
}

static inline float kind_value(int kind, uint64_t key, uint64_t idx)
{
    switch (kind) {
    case KIND_NORM: return qo_synth_value(key, idx, 1.0f, 0.05f);
    case KIND_CONV: return qo_synth_value(key, idx, 0.0f, 0.25f);
    case KIND_DT:   return qo_synth_value(key, idx, 0.0f, 0.5f);
    case KIND_A: {
        const float t = 0.25f * fabsf(synth_normal(key, idx));
        return -0.5f - t;
    }
    default:        return qo_synth_value(key, idx, 0.0f, 0.02f);
    }
}

typedef struct {
    const qo_tensor *t;
    uint8_t *dst;
    uint64_t key;
    int kind;
    uint64_t blk0, blk1;
} synth_job;

static void *synth_worker(void *arg)
{
    synth_job *j = arg;
    const qo_tensor *t = j->t;
    float v[256];
    if (t->type == QO_F32) {
        float *o = (float *)j->dst;
        for (uint64_t i = j->blk0; i < j->blk1; i++) o[i] = kind_value(j->kind, j->key, i);
        return NULL;
    }
    const int per = t->type == QO_Q8_0 ? 32 : 256;
    const size_t bb = t->type == QO_Q4_K ? QO_Q4K_BYTES : t->type == QO_Q6_K ? QO_Q6K_BYTES : QO_Q80_BYTES;
    for (uint64_t b = j->blk0; b < j->blk1; b++) {
        const uint64_t base = b * (uint64_t)per;
        for (int i = 0; i < per; i++) v[i] = kind_value(j->kind, j->key, base + (uint64_t)i);
        uint8_t *o = j->dst + b * bb;
        if (t->type == QO_Q4_K) qo_quantize_q4k(v, o);
        else if (t->type == QO_Q6_K) qo_quantize_q6k(v, o);
        else qo_quantize_q80(v, o);
    }
    return NULL;
}

void qo_synth_tensor(const qo_tensor *t, uint8_t *blob, uint64_t seed, int n_threads)
{
    const uint64_t nel = (uint64_t)t->ne[0] * (uint64_t)t->ne[1] * (uint64_t)t->ne[2];
    const int per = t->type == QO_F32 ? 1 : (t->type == QO_Q8_0 ? 32 : 256);
    const uint64_t nunits = nel / (uint64_t)per;
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 64) n_threads = 64;
    if (nunits < 4096) n_threads = 1;
    pthread_t th[64];
    synth_job jobs[64];
    const uint64_t key = qo_name_key(t->name, seed);
    const int kind = tensor_kind(t->name);
    for (int k = 0; k < n_threads; k++) {
        jobs[k].t = t;
        jobs[k].dst = blob + t->off;
        jobs[k].key = key;
        jobs[k].kind = kind;
        jobs[k].blk0 = nunits * (uint64_t)k / (uint64_t)n_threads;
        jobs[k].blk1 = nunits * (uint64_t)(k + 1) / (uint64_t)n_threads;
    }
    if (n_threads == 1) {
        synth_worker(&jobs[0]);
        return;
    }
    for (int k = 0; k < n_threads; k++) pthread_create(&th[k], NULL, synth_worker, &jobs[k]);
    for (int k = 0; k < n_threads; k++) pthread_join(th[k], NULL);
}

/* GGUF-order tensor table of the synthetic model (names: gguf.c:308-345). */
static int add_tensor(qo_tensor *t, int cap, int *n, uint64_t *off, const char *name,
                      uint32_t type, int64_t ne0, int64_t ne1, int64_t ne2)
{
    if (*n >= cap) return -1;
    qo_tensor *x = &t[*n];
    memset(x, 0, sizeof(*x));
    strncpy(x->name, name, sizeof(x->name) - 1);
    x->type = type;
    x->ne[0] = ne0;
    x->ne[1] = ne1;
    x->ne[2] = ne2;
    x->off = *off;
    x->nbytes = qo_row_bytes((int)type, (int)ne0) * (uint64_t)ne1 * (uint64_t)ne2;
    *off += (x->nbytes + 255) & ~(uint64_t)255;
    (*n)++;
    return 0;
}

int qo_synth_layout(const qo_synth_cfg *cfg, qo_tensor *t, int cap, uint64_t *blob_bytes)
{
    int n = 0;
    uint64_t off = 0;
    char nm[96];
    const uint32_t P = (uint32_t)cfg->proj_type, D = (uint32_t)cfg->down_type;
    if (add_tensor(t, cap, &n, &off, "token_embd.weight", (uint32_t)cfg->embd_type, QO_EMBD, cfg->n_vocab, 1)) return -1;
    if (add_tensor(t, cap, &n, &off, "output_norm.weight", QO_F32, QO_EMBD, 1, 1)) return -1;
    if (add_tensor(t, cap, &n, &off, "output.weight", (uint32_t)cfg->out_type, QO_EMBD, cfg->n_vocab, 1)) return -1;
    for (int il = 0; il < QO_LAYER; il++) {
#define ADD(suffix, type, a, b, c)                                              \
        do {                                                                    \
            snprintf(nm, sizeof(nm), "blk.%d.%s", il, suffix);                  \
            if (add_tensor(t, cap, &n, &off, nm, type, a, b, c)) return -1;     \
        } while (0)
        ADD("attn_norm.weight", QO_F32, QO_EMBD, 1, 1);
        ADD("post_attention_norm.weight", QO_F32, QO_EMBD, 1, 1);
        if (QO_IS_ATTN(il)) {
            ADD("attn_q.weight", P, QO_EMBD, QO_WQ_DIM, 1);
            ADD("attn_k.weight", P, QO_EMBD, QO_WKV_DIM, 1);
            ADD("attn_v.weight", P, QO_EMBD, QO_WKV_DIM, 1);
            ADD("attn_output.weight", P, QO_WO_DIM, QO_EMBD, 1);
            ADD("attn_q_norm.weight", QO_F32, QO_HEAD_DIM, 1, 1);
            ADD("attn_k_norm.weight", QO_F32, QO_HEAD_DIM, 1, 1);
        } else {
            ADD("attn_qkv.weight", P, QO_EMBD, QO_CONV_DIM, 1);
            ADD("attn_gate.weight", P, QO_EMBD, QO_VAL_DIM, 1);
            ADD("ssm_conv1d.weight", QO_F32, QO_CONV, QO_CONV_DIM, 1);
            ADD("ssm_dt.bias", QO_F32, QO_VHEADS, 1, 1);
            ADD("ssm_a", QO_F32, QO_VHEADS, 1, 1);
            ADD("ssm_beta.weight", P, QO_EMBD, QO_VHEADS, 1);
            ADD("ssm_alpha.weight", P, QO_EMBD, QO_VHEADS, 1);
            ADD("ssm_norm.weight", QO_F32, QO_STATE, 1, 1);
            ADD("ssm_out.weight", P, QO_VAL_DIM, QO_EMBD, 1);
        }
        ADD("ffn_gate_inp.weight", QO_F32, QO_EMBD, QO_EXPERT, 1);
        ADD("ffn_gate_exps.weight", QO_Q4_K, QO_EMBD, QO_FF, QO_EXPERT);
        ADD("ffn_up_exps.weight", QO_Q4_K, QO_EMBD, QO_FF, QO_EXPERT);
        ADD("ffn_down_exps.weight", D, QO_FF, QO_EMBD, QO_EXPERT);
        ADD("ffn_gate_inp_shexp.weight", QO_F32, QO_EMBD, 1, 1);
        ADD("ffn_gate_shexp.weight", QO_Q4_K, QO_EMBD, QO_FF, 1);
        ADD("ffn_up_shexp.weight", QO_Q4_K, QO_EMBD, QO_FF, 1);
        ADD("ffn_down_shexp.weight", D, QO_FF, QO_EMBD, 1);
#undef ADD
    }
    *blob_bytes = off;
    return n;
}
