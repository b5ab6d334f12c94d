/*
 * synth.c -- seeded synthetic weights for GGUF test and benchmark models.
 *
 * The benchmark configurations describe random-init models (weights N(0, 0.02), norm
 * gains 1.0) quantised to GGUF Q4_K / Q6_K / Q8_0 or stored as F16.  This file draws
 * the values and encodes the blocks; tpt_spark_b200/synth.py writes the GGUF container.
 *
 * Random numbers: element i of a tensor is a Box-Muller normal from splitmix64 of
 * (tensor seed, i / 2), so any slice of a tensor can be generated independently and in
 * parallel with identical results.
 *
 * Block encoders (layouts as in gguf-py gguf/quants.py, GGUF block sizes from
 * gguf/constants.py):
 *   Q8_0: d = amax/127, q = round(x/d) half away from zero, d stored as f16 -- the
 *         same arithmetic as gguf-py Q8_0.quantize_blocks, which the tests pin.
 *   Q4_K: per 32-element sub-block an affine range [min(x,0), max(x)] in 15 steps; the
 *         eight scales and mins are quantised to 6 bits against f16 super-scales.
 *   Q6_K: per 16-element sub-block a symmetric scale mapping the largest magnitude to
 *         -32; the sixteen scales are quantised to int8 against an f16 super-scale.
 * The Q4_K / Q6_K encoders are this project's own (no search over scales as in
 * llama.cpp); they produce valid blocks, and the forward pass reads whatever bytes the
 * file holds, so the encoder does not affect parity.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

enum { SY_F32 = 0, SY_F16 = 1, SY_Q4_0 = 2, SY_Q4_1 = 3, SY_Q5_0 = 6, SY_Q5_1 = 7, SY_Q8_0 = 8, SY_Q2_K = 10, SY_Q3_K = 11, SY_Q4_K = 12, SY_Q5_K = 13, SY_Q6_K = 14 };

static inline uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

static inline float normal_at(uint64_t seed, int64_t i) {
    uint64_t r = splitmix64(seed ^ splitmix64((uint64_t)(i >> 1)));
    /* two 24-bit uniforms in (0, 1] and [0, 1) */
    double u1 = ((double)((r >> 40) & 0xffffff) + 1.0) / 16777216.0;
    double u2 = (double)((r >> 8) & 0xffffff) / 16777216.0;
    double rad = sqrt(-2.0 * log(u1));
    double a = 6.283185307179586 * u2;
    return (float)((i & 1) ? rad * sin(a) : rad * cos(a));
}

/* x[i] = mean + std * N(0,1) for i in [start, start+n). */
void sy_fill_normal(uint64_t seed, int64_t start, int64_t n, float mean, float std, float* x) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) x[i] = mean + std * normal_at(seed, start + i);
}

static inline uint16_t f2h(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u, ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);
    if (ax < 0x38800000u) {
        if (ax < 0x33000000u) return (uint16_t)sign;
        uint32_t e = ax >> 23, m = (ax & 0x7fffffu) | 0x800000u;
        uint32_t shift = 126u - e, r = m >> shift, rem = m & ((1u << shift) - 1u), half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (r & 1u))) r++;
        return (uint16_t)(sign | r);
    }
    uint32_t r = (ax >> 13) - (112u << 10), rem = ax & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) r++;
    return (uint16_t)(sign | r);
}

static inline float h2f(uint16_t h) {
    uint32_t s = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1fu, m = h & 0x3ffu, u;
    if (e == 0) {
        if (m == 0) {
            u = s;
        } else {
            int sh = 0;
            while (!(m & 0x400u)) { m <<= 1; sh++; }
            m &= 0x3ffu;
            u = s | ((uint32_t)(113 - sh) << 23) | (m << 13);
        }
    } else if (e == 31) {
        u = s | 0x7f800000u | (m << 13);
    } else {
        u = s | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static inline int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

static void enc_q80(const float* x, uint8_t* b) {
    float amax = 0.f;
    for (int j = 0; j < 32; j++) amax = fmaxf(amax, fabsf(x[j]));
    float d = amax / 127.f;
    float id = d != 0.f ? 1.f / d : 0.f;
    uint16_t h = f2h(d);
    b[0] = (uint8_t)(h & 0xff);
    b[1] = (uint8_t)(h >> 8);
    for (int j = 0; j < 32; j++) b[2 + j] = (uint8_t)(int8_t)roundf(x[j] * id);
}

static void enc_q4k(const float* x, uint8_t* b) {
    float scales[8], mins[8], max_scale = 0.f, max_min = 0.f;
    for (int j = 0; j < 8; j++) {
        float mn = x[32 * j], mx = x[32 * j];
        for (int l = 1; l < 32; l++) {
            mn = fminf(mn, x[32 * j + l]);
            mx = fmaxf(mx, x[32 * j + l]);
        }
        if (mn > 0.f) mn = 0.f;
        scales[j] = (mx - mn) / 15.f;
        mins[j] = -mn;
        max_scale = fmaxf(max_scale, scales[j]);
        max_min = fmaxf(max_min, mins[j]);
    }
    uint16_t dh = f2h(max_scale / 63.f), mh = f2h(max_min / 63.f);
    float d = h2f(dh), dm = h2f(mh);
    uint8_t sc[8], mq[8];
    for (int j = 0; j < 8; j++) {
        sc[j] = (uint8_t)(d > 0.f ? clampi((int)lroundf(scales[j] / d), 0, 63) : 0);
        mq[j] = (uint8_t)(dm > 0.f ? clampi((int)lroundf(mins[j] / dm), 0, 63) : 0);
    }
    b[0] = (uint8_t)(dh & 0xff);
    b[1] = (uint8_t)(dh >> 8);
    b[2] = (uint8_t)(mh & 0xff);
    b[3] = (uint8_t)(mh >> 8);
    uint8_t* s = b + 4;
    for (int j = 0; j < 4; j++) {
        s[j] = (uint8_t)(sc[j] | ((sc[j + 4] >> 4) << 6));
        s[j + 4] = (uint8_t)(mq[j] | ((mq[j + 4] >> 4) << 6));
        s[j + 8] = (uint8_t)((sc[j + 4] & 0x0f) | ((mq[j + 4] & 0x0f) << 4));
    }
    uint8_t q[256];
    for (int j = 0; j < 8; j++) {
        float es = d * (float)sc[j], em = dm * (float)mq[j];
        for (int l = 0; l < 32; l++) q[32 * j + l] = (uint8_t)(es > 0.f ? clampi((int)lroundf((x[32 * j + l] + em) / es), 0, 15) : 0);
    }
    uint8_t* qs = b + 16;
    for (int g = 0; g < 4; g++)
        for (int l = 0; l < 32; l++) qs[32 * g + l] = (uint8_t)(q[64 * g + l] | (q[64 * g + 32 + l] << 4));
}

/* Q4_0 / Q5_0 as gguf-py's quantize_blocks (gguf/quants.py :222-239, :293-312): d = signed
 * max / -8 (-16), q = trunc(x / d + 8.5 (16.5)) clipped to 0..15 (0..31); element l < 16 in the
 * low nibble of qs[l], l + 16 in the high nibble, Q5_0's 5th bits in the little-endian qh. */
static void enc_q40_q50(const float* x, uint8_t* b, int five) {
    float mx = 0.f, amx = 0.f;
    for (int j = 0; j < 32; j++)
        if (fabsf(x[j]) > amx) { amx = fabsf(x[j]); mx = x[j]; }
    const float d = mx / (five ? -16.f : -8.f), id = d != 0.f ? 1.f / d : 0.f;
    uint8_t q[32];
    for (int j = 0; j < 32; j++) q[j] = (uint8_t)clampi((int)truncf(x[j] * id + (five ? 16.5f : 8.5f)), 0, five ? 31 : 15);
    const uint16_t h = f2h(d);
    b[0] = (uint8_t)(h & 0xff);
    b[1] = (uint8_t)(h >> 8);
    uint8_t* qs = b + (five ? 6 : 2);
    for (int j = 0; j < 16; j++) qs[j] = (uint8_t)((q[j] & 0x0f) | ((q[j + 16] & 0x0f) << 4));
    if (five) {
        uint32_t qh = 0;
        for (int j = 0; j < 32; j++) qh |= (uint32_t)(q[j] >> 4) << j;
        memcpy(b + 2, &qh, 4);
    }
}

/* Q4_1 / Q5_1 as gguf-py's quantize_blocks (gguf/quants.py :256-274, :335-355): d = (max -
 * min) / 15 (31), m = min, q = trunc((x - min) / d + 0.5) clipped; layouts as Q4_0 / Q5_0 with
 * m after d. */
static void enc_q41_q51(const float* x, uint8_t* b, int five) {
    float mn = x[0], mx = x[0];
    for (int j = 1; j < 32; j++) {
        mn = fminf(mn, x[j]);
        mx = fmaxf(mx, x[j]);
    }
    const float d = (mx - mn) / (five ? 31.f : 15.f), id = d != 0.f ? 1.f / d : 0.f;
    uint8_t q[32];
    for (int j = 0; j < 32; j++) q[j] = (uint8_t)clampi((int)truncf((x[j] - mn) * id + 0.5f), 0, five ? 31 : 15);
    const uint16_t dh = f2h(d), mh = f2h(mn);
    b[0] = (uint8_t)(dh & 0xff);
    b[1] = (uint8_t)(dh >> 8);
    b[2] = (uint8_t)(mh & 0xff);
    b[3] = (uint8_t)(mh >> 8);
    uint8_t* qs = b + (five ? 8 : 4);
    for (int j = 0; j < 16; j++) qs[j] = (uint8_t)((q[j] & 0x0f) | ((q[j + 16] & 0x0f) << 4));
    if (five) {
        uint32_t qh = 0;
        for (int j = 0; j < 32; j++) qh |= (uint32_t)(q[j] >> 4) << j;
        memcpy(b + 4, &qh, 4);
    }
}

/* Q5_K: enc_q4k with 32 levels (scales (max - min) / 31) and the 5th bits in qh. */
static void enc_q5k(const float* x, uint8_t* b) {
    float scales[8], mins[8], max_scale = 0.f, max_min = 0.f;
    for (int j = 0; j < 8; j++) {
        float mn = x[32 * j], mx = x[32 * j];
        for (int l = 1; l < 32; l++) {
            mn = fminf(mn, x[32 * j + l]);
            mx = fmaxf(mx, x[32 * j + l]);
        }
        if (mn > 0.f) mn = 0.f;
        scales[j] = (mx - mn) / 31.f;
        mins[j] = -mn;
        max_scale = fmaxf(max_scale, scales[j]);
        max_min = fmaxf(max_min, mins[j]);
    }
    uint16_t dh = f2h(max_scale / 63.f), mh = f2h(max_min / 63.f);
    float d = h2f(dh), dm = h2f(mh);
    uint8_t sc[8], mq[8];
    for (int j = 0; j < 8; j++) {
        sc[j] = (uint8_t)(d > 0.f ? clampi((int)lroundf(scales[j] / d), 0, 63) : 0);
        mq[j] = (uint8_t)(dm > 0.f ? clampi((int)lroundf(mins[j] / dm), 0, 63) : 0);
    }
    b[0] = (uint8_t)(dh & 0xff);
    b[1] = (uint8_t)(dh >> 8);
    b[2] = (uint8_t)(mh & 0xff);
    b[3] = (uint8_t)(mh >> 8);
    uint8_t* s = b + 4;
    for (int j = 0; j < 4; j++) {
        s[j] = (uint8_t)(sc[j] | ((sc[j + 4] >> 4) << 6));
        s[j + 4] = (uint8_t)(mq[j] | ((mq[j + 4] >> 4) << 6));
        s[j + 8] = (uint8_t)((sc[j + 4] & 0x0f) | ((mq[j + 4] & 0x0f) << 4));
    }
    uint8_t q[256];
    for (int j = 0; j < 8; j++) {
        float es = d * (float)sc[j], em = dm * (float)mq[j];
        for (int l = 0; l < 32; l++) q[32 * j + l] = (uint8_t)(es > 0.f ? clampi((int)lroundf((x[32 * j + l] + em) / es), 0, 31) : 0);
    }
    uint8_t* qh = b + 16;
    uint8_t* qs = b + 48;
    memset(qh, 0, 32);
    for (int j = 0; j < 8; j++)
        for (int l = 0; l < 32; l++) qh[l] |= (uint8_t)((q[32 * j + l] >> 4) << j);
    for (int g = 0; g < 4; g++)
        for (int l = 0; l < 32; l++) qs[32 * g + l] = (uint8_t)((q[64 * g + l] & 0x0f) | ((q[64 * g + 32 + l] & 0x0f) << 4));
}

/* Q2_K (scales[16] qs[64] d dmin): per 16-element group an unsigned 4-bit scale and min over
 * 2-bit codes, value (d*sc)*q - (dmin*m). */
static void enc_q2k(const float* x, uint8_t* b) {
    float sc_f[16], mn_f[16], max_sc = 0.f, max_mn = 0.f;
    for (int g = 0; g < 16; g++) {
        float mn = x[16 * g], mx = x[16 * g];
        for (int l = 1; l < 16; l++) {
            mn = fminf(mn, x[16 * g + l]);
            mx = fmaxf(mx, x[16 * g + l]);
        }
        if (mn > 0.f) mn = 0.f;
        sc_f[g] = (mx - mn) / 3.f;
        mn_f[g] = -mn;
        max_sc = fmaxf(max_sc, sc_f[g]);
        max_mn = fmaxf(max_mn, mn_f[g]);
    }
    const uint16_t dh = f2h(max_sc / 15.f), mh = f2h(max_mn / 15.f);
    const float d = h2f(dh), dm = h2f(mh);
    memset(b, 0, 84);
    for (int g = 0; g < 16; g++) {
        const int sc = d > 0.f ? clampi((int)lroundf(sc_f[g] / d), 0, 15) : 0;
        const int m = dm > 0.f ? clampi((int)lroundf(mn_f[g] / dm), 0, 15) : 0;
        b[g] = (uint8_t)(sc | (m << 4));
        const float es = d * (float)sc, em = dm * (float)m;
        for (int l = 0; l < 16; l++) {
            const int e = 16 * g + l;
            const int q = es > 0.f ? clampi((int)lroundf((x[e] + em) / es), 0, 3) : 0;
            b[16 + 32 * (e >> 7) + (e & 31)] |= (uint8_t)(q << (2 * ((e >> 5) & 3)));
        }
    }
    b[80] = (uint8_t)(dh & 0xff);
    b[81] = (uint8_t)(dh >> 8);
    b[82] = (uint8_t)(mh & 0xff);
    b[83] = (uint8_t)(mh >> 8);
}

/* Q3_K (hmask[32] qs[64] scales[12] d): per 16-element group a signed 6-bit scale over codes
 * -4..3 stored as 2 low bits plus the hmask bit (set when the code is >= 0). */
static void enc_q3k(const float* x, uint8_t* b) {
    float sc_f[16], amax_sc = 0.f;
    for (int g = 0; g < 16; g++) {
        float mx = 0.f, amx = 0.f;
        for (int l = 0; l < 16; l++)
            if (fabsf(x[16 * g + l]) > amx) { amx = fabsf(x[16 * g + l]); mx = x[16 * g + l]; }
        sc_f[g] = mx / -4.f;
        amax_sc = fmaxf(amax_sc, fabsf(sc_f[g]));
    }
    const uint16_t dh = f2h(amax_sc / 31.f);
    const float d = h2f(dh);
    memset(b, 0, 110);
    for (int g = 0; g < 16; g++) {
        const int sc = d > 0.f ? clampi((int)lroundf(sc_f[g] / d), -32, 31) : 0;
        const int u = sc + 32;
        b[96 + (g & 7)] |= (uint8_t)((u & 0x0f) << (4 * (g >> 3)));
        b[96 + 8 + (g & 3)] |= (uint8_t)(((u >> 4) & 3) << (2 * (g >> 2)));
        const float es = d * (float)sc;
        for (int l = 0; l < 16; l++) {
            const int e = 16 * g + l;
            const int q = es != 0.f ? clampi((int)lroundf(x[e] / es), -4, 3) : 0;
            b[32 + 32 * (e >> 7) + (e & 31)] |= (uint8_t)(((q + 4) & 3) << (2 * ((e >> 5) & 3)));
            if (q >= 0) b[e & 31] |= (uint8_t)(1 << (e >> 5));
        }
    }
    b[108] = (uint8_t)(dh & 0xff);
    b[109] = (uint8_t)(dh >> 8);
}

static void enc_q6k(const float* x, uint8_t* b) {
    float scales[16], max_scale = 0.f, amax_scale = 0.f;
    for (int j = 0; j < 16; j++) {
        float mx = 0.f, amx = 0.f;
        for (int l = 0; l < 16; l++) {
            float v = x[16 * j + l];
            if (fabsf(v) > amx) { amx = fabsf(v); mx = v; }
        }
        scales[j] = amx > 0.f ? mx / -32.f : 0.f;
        if (fabsf(scales[j]) > amax_scale) { amax_scale = fabsf(scales[j]); max_scale = scales[j]; }
    }
    int8_t sc[16];
    float iscale = max_scale != 0.f ? -128.f / max_scale : 0.f;
    uint16_t dh = f2h(iscale != 0.f ? 1.f / iscale : 0.f);
    float d = h2f(dh);
    for (int j = 0; j < 16; j++) sc[j] = (int8_t)clampi((int)lroundf(iscale * scales[j]), -128, 127);
    uint8_t L[256];
    for (int j = 0; j < 16; j++) {
        float es = d * (float)sc[j];
        for (int l = 0; l < 16; l++) {
            int q = es != 0.f ? clampi((int)lroundf(x[16 * j + l] / es), -32, 31) : 0;
            L[16 * j + l] = (uint8_t)(q + 32);
        }
    }
    uint8_t* ql = b;
    uint8_t* qh = b + 128;
    for (int h = 0; h < 2; h++) {
        for (int l = 0; l < 32; l++) {
            int e = 128 * h + l;
            uint8_t q1 = L[e], q2 = L[e + 32], q3 = L[e + 64], q4 = L[e + 96];
            ql[64 * h + l] = (uint8_t)((q1 & 0x0f) | ((q3 & 0x0f) << 4));
            ql[64 * h + l + 32] = (uint8_t)((q2 & 0x0f) | ((q4 & 0x0f) << 4));
            qh[32 * h + l] = (uint8_t)((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
        }
    }
    memcpy(b + 192, sc, 16);
    b[208] = (uint8_t)(dh & 0xff);
    b[209] = (uint8_t)(dh >> 8);
}

int64_t sy_type_bytes(int type, int64_t n) {
    switch (type) {
    case SY_F32: return n * 4;
    case SY_F16: return n * 2;
    case SY_Q8_0: return n / 32 * 34;
    case SY_Q4_K: return n / 256 * 144;
    case SY_Q6_K: return n / 256 * 210;
    case SY_Q4_0: return n / 32 * 18;
    case SY_Q5_0: return n / 32 * 22;
    case SY_Q5_K: return n / 256 * 176;
    case SY_Q2_K: return n / 256 * 84;
    case SY_Q4_1: return n / 32 * 20;
    case SY_Q5_1: return n / 32 * 24;
    case SY_Q3_K: return n / 256 * 110;
    }
    return -1;
}

/* Encode n f32 values (n a multiple of the block size) into `out`. Returns bytes. */
int64_t sy_encode(int type, const float* x, int64_t n, uint8_t* out) {
    int64_t nb;
    switch (type) {
    case SY_F32:
        memcpy(out, x, (size_t)n * 4);
        return n * 4;
    case SY_F16:
#pragma omp parallel for schedule(static)
        for (int64_t i = 0; i < n; i++) {
            uint16_t h = f2h(x[i]);
            memcpy(out + 2 * i, &h, 2);
        }
        return n * 2;
    case SY_Q8_0:
        nb = n / 32;
#pragma omp parallel for schedule(static)
        for (int64_t i = 0; i < nb; i++) enc_q80(x + 32 * i, out + 34 * i);
        return nb * 34;
    case SY_Q4_K:
        nb = n / 256;
#pragma omp parallel for schedule(static)
        for (int64_t i = 0; i < nb; i++) enc_q4k(x + 256 * i, out + 144 * i);
        return nb * 144;
    case SY_Q6_K:
        nb = n / 256;
#pragma omp parallel for schedule(static)
        for (int64_t i = 0; i < nb; i++) enc_q6k(x + 256 * i, out + 210 * i);
        return nb * 210;
    case SY_Q4_0:
    case SY_Q5_0:
        nb = n / 32;
#pragma omp parallel for schedule(static)
        for (int64_t i = 0; i < nb; i++) enc_q40_q50(x + 32 * i, out + (type == SY_Q5_0 ? 22 : 18) * i, type == SY_Q5_0);
        return nb * (type == SY_Q5_0 ? 22 : 18);
    case SY_Q5_K:
        nb = n / 256;
#pragma omp parallel for schedule(static)
        for (int64_t i = 0; i < nb; i++) enc_q5k(x + 256 * i, out + 176 * i);
        return nb * 176;
    case SY_Q4_1:
    case SY_Q5_1:
        nb = n / 32;
#pragma omp parallel for schedule(static)
        for (int64_t i = 0; i < nb; i++) enc_q41_q51(x + 32 * i, out + (type == SY_Q5_1 ? 24 : 20) * i, type == SY_Q5_1);
        return nb * (type == SY_Q5_1 ? 24 : 20);
    case SY_Q2_K:
        nb = n / 256;
#pragma omp parallel for schedule(static)
        for (int64_t i = 0; i < nb; i++) enc_q2k(x + 256 * i, out + 84 * i);
        return nb * 84;
    case SY_Q3_K:
        nb = n / 256;
#pragma omp parallel for schedule(static)
        for (int64_t i = 0; i < nb; i++) enc_q3k(x + 256 * i, out + 110 * i);
        return nb * 110;
    }
    return -1;
}

/* Draw n = rows*cols values N(mean, std) for tensor `seed` and encode them. A scratch
 * f32 buffer of n floats must be supplied by the caller. Returns bytes written. */
int64_t sy_make_tensor(int type, uint64_t seed, int64_t n, float mean, float std, float* scratch, uint8_t* out) {
    if (std == 0.f) {
#pragma omp parallel for schedule(static)
        for (int64_t i = 0; i < n; i++) scratch[i] = mean;
    } else {
        sy_fill_normal(seed, 0, n, mean, std, scratch);
    }
    return sy_encode(type, scratch, n, out);
}
