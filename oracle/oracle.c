/*
 * oracle.c -- CPU restatement of tpt-spark's CPU inference path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (the tpt_spark_b200 package and
 * its libtptc.so) links, loads or calls this file.  Only tests/, the smoke() check in
 * __graft_entry__.py and the cpu_baseline / --impl reference legs of bench.py use it,
 * and only as the checker or as the timed CPU baseline.
 *
 * What it restates.  The reference runs its CPU path through candle 0.8.4
 * (src-tauri/src/engine/candle_engine.rs:217-324 -> candle-transformers
 * models::quantized_llama::ModelWeights::{from_gguf, forward}, candle-core k_quants
 * vec_dot / QMatMul).  candle is pinned in src-tauri/Cargo.lock:316-356 but is not
 * vendored, and no Rust toolchain exists here, so the reference cannot be built.  This
 * file restates candle 0.8.4's published algorithm:
 *   - GGUF block formats Q4_K (144 B / 256), Q6_K (210 B / 256), Q8_0 (34 B / 32), F16, and
 *     Q4_0 (18 B / 32), Q4_1 (20 B / 32), Q5_0 (22 B / 32), Q5_1 (24 B / 32), Q2_K (84 B / 256),
 *     Q3_K (110 B / 256), Q5_K (176 B / 256); dequantisation follows the formulas and the
 *     evaluation order of gguf-py 0.19 (gguf/quants.py Q4_0 :241-251, Q4_1 :276-288, Q5_0
 *     :314-330, Q5_1 :357-375, Q8_0 :378-401, Q2_K :406-428, Q3_K :433-472, Q4_K :475-522,
 *     Q5_K :527-549, Q6_K :552-572), which the golden tests pin bit-for-bit;
 *   - activation quantisation for the integer dot: Q8_K (BlockQ8K::from_float) for
 *     Q4_K / Q6_K weights, Q8_0 (BlockQ8_0::from_float) for Q8_0 weights; F16 weights
 *     are dequantised to f32 and multiplied in f32 (QMatMul::from_arc);
 *   - vec_dot_q2k / q3k / q4k / q5k / q6k x q8k and q4_0 / q5_0 / q8_0 x q8_0 in candle's
 *     scalar accumulation order (the k_quants vec_dot_unopt loops of BlockQ2K, BlockQ3K,
 *     BlockQ4K, BlockQ5K, BlockQ6K, BlockQ4_0, BlockQ5_0, BlockQ8_0);
 *   - the quantized_llama forward: RmsNorm, interleaved RoPE (rope_i) from an f32
 *     cos/sin table, f32 KV concatenation, causal softmax(QK^T/sqrt(d))V, SwiGLU MLP,
 *     residual adds, final norm and the output projection on the last position only;
 *   - its mixture-of-experts block (MlpOrMoe::MoE, the Mixtral GGUFs): softmax routing over
 *     every expert, the top n_used by a stable descending sort, weights renormalised over
 *     them, outputs accumulated in expert order (moe_ffn below); the reference's wgpu path adds
 *     stacked expert tensors and a shared expert (wgpu_loader.rs:151-173,
 *     wgpu_engine.rs:781-864), taken over here;
 *   - gemma's GEGLU (the reference's shaders/geglu.wgsl tanh form) and sqrt(dim) embedding
 *     scale.
 * The reference's own wgpu path (engine/wgpu_engine.rs) is not followed: its Q4_K
 * nibble layout is wrong (shaders/dequant_q4k.wgsl:9-21) and run_forward_pass has no
 * residual connections (wgpu_engine.rs:443,474).
 *
 * Parity pins: block dequantisation and Q8_0 quantisation are pinned against gguf-py
 * (tests/golden/).  Semantics inside candle (Q8_K rounding, accumulation order, rope
 * table) are restated from candle's published source and cannot be run here; that part
 * of the oracle is "parity unpinned" against candle itself.
 *
 * Build: gcc -O3 -march=native -fopenmp -ffp-contract=off (oracle/Makefile).  FMA
 * contraction is off so that every float expression rounds once per operation, as
 * candle's Rust code does.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif
#include <immintrin.h>

#define QK_K 256
#define QK8_0 32
#define Q4K_BYTES 144
#define Q6K_BYTES 210
#define Q80_BYTES 34
#define Q40_BYTES 18
#define Q41_BYTES 20
#define Q50_BYTES 22
#define Q51_BYTES 24
#define Q2K_BYTES 84
#define Q3K_BYTES 110
#define Q5K_BYTES 176

enum {
    OR_F32 = 0, OR_F16 = 1, OR_Q4_0 = 2, OR_Q4_1 = 3, OR_Q5_0 = 6, OR_Q5_1 = 7, OR_Q8_0 = 8,
    OR_Q2_K = 10, OR_Q3_K = 11, OR_Q4_K = 12, OR_Q5_K = 13, OR_Q6_K = 14
};

/* block_q8_K layout: f32 d, int8 qs[256], int16 bsums[16] = 292 bytes. */
typedef struct {
    float d;
    int8_t qs[QK_K];
    int16_t bsums[QK_K / 16];
} or_q8k;

static int g_threads = 1;
/* Optional per-layer trace of the last position (q after RoPE, attention output, residual
 * stream after the layer) in rows 3l, 3l+1, 3l+2 -- the layout tptc_debug_trace uses. */
static float* g_trace = NULL;

void or_set_trace(float* trace) { g_trace = trace; }

void or_set_threads(int n) { g_threads = n > 0 ? n : 1; }
int or_get_threads(void) { return g_threads; }

/* AVX2 versions of the quantised vec dots (on by default).  They keep candle's
 * vec_dot_unopt accumulation exactly: its eight int32 lanes aux32[l] collect the products of
 * elements l (mod 8), which is one 8-lane vector; the per-block float update
 * sums[l] += d * (float)aux32[l] is the same multiply and add per lane; the lanes are summed
 * in order at the end.  So both paths return the same bits (tests/test_oracle_golden.py
 * compares them); the scalar path stays for reference. */
static int g_simd = 1;
void or_set_simd(int on) { g_simd = on ? 1 : 0; }

/* ---------------------------------------------------------------- half floats */

float or_h2f(uint16_t h) {
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

/* f32 -> f16, round to nearest even (numpy astype(float16), Rust half::f16::from_f32). */
uint16_t or_f2h(float f) {
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

static inline uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* Q4_K 6-bit scale/min unpack (gguf/quants.py Q4_K.get_scale_min :479-503). */
static inline void q4k_scale_min(const uint8_t* s, uint8_t* sc, uint8_t* mn) {
    for (int j = 0; j < 4; j++) {
        sc[j] = s[j] & 63;
        mn[j] = s[j + 4] & 63;
        sc[j + 4] = (uint8_t)((s[j + 8] & 0x0f) | ((s[j] >> 6) << 4));
        mn[j + 4] = (uint8_t)((s[j + 8] >> 4) | ((s[j + 4] >> 6) << 4));
    }
}

/* ------------------------------------------------------------- dequantisation */

/* gguf/quants.py Q4_K.dequantize_blocks :505-522: (d*sc)*q - (dmin*m), one rounding each. */
void or_dequant_q4k(const uint8_t* blocks, int64_t nb, float* y) {
    for (int64_t b = 0; b < nb; b++) {
        const uint8_t* blk = blocks + b * Q4K_BYTES;
        float d = or_h2f(rd16(blk)), dmin = or_h2f(rd16(blk + 2));
        uint8_t sc[8], mn[8];
        q4k_scale_min(blk + 4, sc, mn);
        const uint8_t* qs = blk + 16;
        float* out = y + b * QK_K;
        for (int g = 0; g < 4; g++) {
            float d1 = d * (float)sc[2 * g], m1 = dmin * (float)mn[2 * g];
            float d2 = d * (float)sc[2 * g + 1], m2 = dmin * (float)mn[2 * g + 1];
            for (int l = 0; l < 32; l++) {
                out[64 * g + l] = d1 * (float)(qs[32 * g + l] & 0x0f) - m1;
                out[64 * g + 32 + l] = d2 * (float)(qs[32 * g + l] >> 4) - m2;
            }
        }
    }
}

/* Q6_K element value q-32 for element e of a block (layout: ql[128] qh[64] sc[16] d). */
static inline int q6k_val(const uint8_t* blk, int e) {
    int h = e >> 7, r = e & 127, i = r >> 5, l = r & 31;
    const uint8_t* ql = blk + 64 * h;
    const uint8_t* qh = blk + 128 + 32 * h;
    int lo = (i & 1) ? ql[l + 32] : ql[l];
    lo = (i & 2) ? (lo >> 4) : (lo & 0x0f);
    int hi = (qh[l] >> (2 * i)) & 3;
    return (lo | (hi << 4)) - 32;
}

/* gguf/quants.py Q6_K.dequantize_blocks :554-572: (d*scale)*q. */
void or_dequant_q6k(const uint8_t* blocks, int64_t nb, float* y) {
    for (int64_t b = 0; b < nb; b++) {
        const uint8_t* blk = blocks + b * Q6K_BYTES;
        const int8_t* sc = (const int8_t*)(blk + 192);
        float d = or_h2f(rd16(blk + 208));
        for (int e = 0; e < QK_K; e++) {
            float ds = d * (float)sc[e >> 4];
            y[b * QK_K + e] = ds * (float)q6k_val(blk, e);
        }
    }
}

/* gguf/quants.py Q8_0.dequantize_blocks :395-401: q*d. */
void or_dequant_q80(const uint8_t* blocks, int64_t nb, float* y) {
    for (int64_t b = 0; b < nb; b++) {
        const uint8_t* blk = blocks + b * Q80_BYTES;
        float d = or_h2f(rd16(blk));
        const int8_t* qs = (const int8_t*)(blk + 2);
        for (int l = 0; l < QK8_0; l++) y[b * QK8_0 + l] = (float)qs[l] * d;
    }
}

void or_dequant_f16(const uint16_t* x, int64_t n, float* y) {
    for (int64_t i = 0; i < n; i++) y[i] = or_h2f(x[i]);
}

/* Q5_0 / Q5_1 high bit of element l (0..31) of a block: bit l of the little-endian qh. */
static inline int q5_hbit(const uint8_t* qh, int l) { return (qh[l >> 3] >> (l & 7)) & 1; }

/* gguf/quants.py Q4_0.dequantize_blocks :241-251: d*(q-8); element l < 16 is the low
 * nibble of qs[l], element l + 16 its high nibble. */
void or_dequant_q40(const uint8_t* blocks, int64_t nb, float* y) {
    for (int64_t b = 0; b < nb; b++) {
        const uint8_t* blk = blocks + b * Q40_BYTES;
        float d = or_h2f(rd16(blk));
        for (int l = 0; l < 16; l++) {
            y[b * 32 + l] = d * (float)((blk[2 + l] & 0x0f) - 8);
            y[b * 32 + 16 + l] = d * (float)((blk[2 + l] >> 4) - 8);
        }
    }
}

/* gguf/quants.py Q4_1.dequantize_blocks :276-288: (d*q) + m. */
void or_dequant_q41(const uint8_t* blocks, int64_t nb, float* y) {
    for (int64_t b = 0; b < nb; b++) {
        const uint8_t* blk = blocks + b * Q41_BYTES;
        float d = or_h2f(rd16(blk)), m = or_h2f(rd16(blk + 2));
        for (int l = 0; l < 16; l++) {
            y[b * 32 + l] = d * (float)(blk[4 + l] & 0x0f) + m;
            y[b * 32 + 16 + l] = d * (float)(blk[4 + l] >> 4) + m;
        }
    }
}

/* gguf/quants.py Q5_0.dequantize_blocks :314-330: d*(q-16), q = nibble | hbit << 4. */
void or_dequant_q50(const uint8_t* blocks, int64_t nb, float* y) {
    for (int64_t b = 0; b < nb; b++) {
        const uint8_t* blk = blocks + b * Q50_BYTES;
        float d = or_h2f(rd16(blk));
        const uint8_t* qh = blk + 2;
        const uint8_t* qs = blk + 6;
        for (int l = 0; l < 16; l++) {
            y[b * 32 + l] = d * (float)(((qs[l] & 0x0f) | (q5_hbit(qh, l) << 4)) - 16);
            y[b * 32 + 16 + l] = d * (float)(((qs[l] >> 4) | (q5_hbit(qh, l + 16) << 4)) - 16);
        }
    }
}

/* gguf/quants.py Q5_1.dequantize_blocks :357-375: (d*q) + m. */
void or_dequant_q51(const uint8_t* blocks, int64_t nb, float* y) {
    for (int64_t b = 0; b < nb; b++) {
        const uint8_t* blk = blocks + b * Q51_BYTES;
        float d = or_h2f(rd16(blk)), m = or_h2f(rd16(blk + 2));
        const uint8_t* qh = blk + 4;
        const uint8_t* qs = blk + 8;
        for (int l = 0; l < 16; l++) {
            y[b * 32 + l] = d * (float)((qs[l] & 0x0f) | (q5_hbit(qh, l) << 4)) + m;
            y[b * 32 + 16 + l] = d * (float)((qs[l] >> 4) | (q5_hbit(qh, l + 16) << 4)) + m;
        }
    }
}

/* gguf/quants.py Q2_K.dequantize_blocks :406-428 (scales[16] qs[64] d dmin): element
 * 128h + 32s + l = (qs[32h + l] >> 2s) & 3, group e/16: (d*(sc & 15))*q - (dmin*(sc >> 4)). */
void or_dequant_q2k(const uint8_t* blocks, int64_t nb, float* y) {
    for (int64_t b = 0; b < nb; b++) {
        const uint8_t* blk = blocks + b * Q2K_BYTES;
        float d = or_h2f(rd16(blk + 80)), dmin = or_h2f(rd16(blk + 82));
        for (int e = 0; e < QK_K; e++) {
            const int h = e >> 7, sh = (e >> 5) & 3, l = e & 31, g = e >> 4;
            const int q = (blk[16 + 32 * h + l] >> (2 * sh)) & 3;
            const float dl = d * (float)(blk[g] & 0x0f), ml = dmin * (float)(blk[g] >> 4);
            y[b * QK_K + e] = dl * (float)q - ml;
        }
    }
}

/* Q3_K 6-bit scale k (0..15), minus 32: low 4 bits from scales[k % 8] (nibble k / 8), high
 * 2 bits from scales[8 + k % 4] (bits 2 (k / 4)). */
static inline int q3k_scale(const uint8_t* sc, int k) {
    const int lo = (sc[k & 7] >> (4 * (k >> 3))) & 0x0f;
    const int hi = (sc[8 + (k & 3)] >> (2 * (k >> 2))) & 0x03;
    return (lo | (hi << 4)) - 32;
}

/* gguf/quants.py Q3_K.dequantize_blocks :433-472 (hmask[32] qs[64] scales[12] d): element
 * e = 128h + 32s + l: q = ((qs[32h + l] >> 2s) & 3) - 4 * (1 - ((hmask[l] >> (e / 32)) & 1)),
 * value (d*scale(e / 16))*q. */
void or_dequant_q3k(const uint8_t* blocks, int64_t nb, float* y) {
    for (int64_t b = 0; b < nb; b++) {
        const uint8_t* blk = blocks + b * Q3K_BYTES;
        float d = or_h2f(rd16(blk + 108));
        for (int e = 0; e < QK_K; e++) {
            const int h = e >> 7, sh = (e >> 5) & 3, l = e & 31;
            const int ql = (blk[32 + 32 * h + l] >> (2 * sh)) & 3;
            const int hb = (blk[l] >> (e >> 5)) & 1;
            const int q = ql - ((hb ^ 1) << 2);
            const float dl = d * (float)q3k_scale(blk + 96, e >> 4);
            y[b * QK_K + e] = dl * (float)q;
        }
    }
}

/* Q5_K element value q (0..31) for element e of a block (d dmin scales[12] qh[32] qs[128]). */
static inline int q5k_val(const uint8_t* blk, int e) {
    const int g = e >> 6, j = e >> 5, l = e & 31;
    const uint8_t b = blk[48 + 32 * g + l];
    const int lo = (j & 1) ? (b >> 4) : (b & 0x0f);
    return lo | (((blk[16 + l] >> j) & 1) << 4);
}

/* gguf/quants.py Q5_K.dequantize_blocks :527-549: (d*sc)*q - (dmin*m). */
void or_dequant_q5k(const uint8_t* blocks, int64_t nb, float* y) {
    for (int64_t b = 0; b < nb; b++) {
        const uint8_t* blk = blocks + b * Q5K_BYTES;
        float d = or_h2f(rd16(blk)), dmin = or_h2f(rd16(blk + 2));
        uint8_t sc[8], mn[8];
        q4k_scale_min(blk + 4, sc, mn);
        for (int e = 0; e < QK_K; e++) {
            const int j = e >> 5;
            const float dl = d * (float)sc[j], ml = dmin * (float)mn[j];
            y[b * QK_K + e] = dl * (float)q5k_val(blk, e) - ml;
        }
    }
}

int64_t or_type_block_elems(int type) {
    switch (type) {
    case OR_F32: case OR_F16: return 1;
    case OR_Q4_0: case OR_Q4_1: case OR_Q5_0: case OR_Q5_1: case OR_Q8_0: return 32;
    }
    return 256;
}
int64_t or_type_block_bytes(int type) {
    switch (type) {
    case OR_F32: return 4;
    case OR_F16: return 2;
    case OR_Q8_0: return Q80_BYTES;
    case OR_Q4_K: return Q4K_BYTES;
    case OR_Q6_K: return Q6K_BYTES;
    case OR_Q4_0: return Q40_BYTES;
    case OR_Q4_1: return Q41_BYTES;
    case OR_Q5_0: return Q50_BYTES;
    case OR_Q5_1: return Q51_BYTES;
    case OR_Q2_K: return Q2K_BYTES;
    case OR_Q3_K: return Q3K_BYTES;
    case OR_Q5_K: return Q5K_BYTES;
    }
    return 0;
}

/* Dequantise n elements of any supported type into f32. Returns 0 or -1. */
int or_dequant(int type, const void* src, int64_t n, float* y) {
    switch (type) {
    case OR_F32: memcpy(y, src, (size_t)n * 4); return 0;
    case OR_F16: or_dequant_f16((const uint16_t*)src, n, y); return 0;
    case OR_Q8_0: or_dequant_q80((const uint8_t*)src, n / 32, y); return 0;
    case OR_Q4_K: or_dequant_q4k((const uint8_t*)src, n / 256, y); return 0;
    case OR_Q6_K: or_dequant_q6k((const uint8_t*)src, n / 256, y); return 0;
    case OR_Q4_0: or_dequant_q40((const uint8_t*)src, n / 32, y); return 0;
    case OR_Q4_1: or_dequant_q41((const uint8_t*)src, n / 32, y); return 0;
    case OR_Q5_0: or_dequant_q50((const uint8_t*)src, n / 32, y); return 0;
    case OR_Q5_1: or_dequant_q51((const uint8_t*)src, n / 32, y); return 0;
    case OR_Q2_K: or_dequant_q2k((const uint8_t*)src, n / 256, y); return 0;
    case OR_Q3_K: or_dequant_q3k((const uint8_t*)src, n / 256, y); return 0;
    case OR_Q5_K: or_dequant_q5k((const uint8_t*)src, n / 256, y); return 0;
    }
    return -1;
}

/* ---------------------------------------------------- activation quantisation */

/* candle k_quants BlockQ8K::from_float: signed max of largest magnitude, iscale=-128/max,
 * q=min(127, round(iscale*x)) with round half away from zero, d=1/iscale, 16-element bsums. */
void or_quant_q8k(const float* x, int64_t k, or_q8k* y) {
    for (int64_t i = 0; i < k / QK_K; i++) {
        const float* xs = x + i * QK_K;
        or_q8k* b = y + i;
        float max = 0.f, amax = 0.f;
        for (int j = 0; j < QK_K; j++) {
            float ax = fabsf(xs[j]);
            if (amax < ax) { amax = ax; max = xs[j]; }
        }
        if (amax == 0.f) {
            b->d = 0.f;
            memset(b->qs, 0, sizeof b->qs);
            memset(b->bsums, 0, sizeof b->bsums);
            continue;
        }
        float iscale = -128.f / max;
        for (int j = 0; j < QK_K; j++) {
            float v = roundf(iscale * xs[j]);
            b->qs[j] = (int8_t)(v < 127.f ? v : 127.f);
        }
        for (int j = 0; j < QK_K / 16; j++) {
            int s = 0;
            for (int l = 0; l < 16; l++) s += b->qs[16 * j + l];
            b->bsums[j] = (int16_t)s;
        }
        b->d = 1.f / iscale;
    }
}

/* candle k_quants BlockQ8_0::from_float (same as gguf-py Q8_0.quantize_blocks :381-393):
 * d=amax/127, id=1/d, q=round(x*id), d stored as f16. Output: 34-byte blocks. */
void or_quant_q80(const float* x, int64_t k, uint8_t* y) {
    for (int64_t i = 0; i < k / QK8_0; i++) {
        const float* xs = x + i * QK8_0;
        uint8_t* b = y + i * Q80_BYTES;
        float amax = 0.f;
        for (int j = 0; j < QK8_0; j++) amax = fmaxf(amax, fabsf(xs[j]));
        float d = amax / 127.f;
        float id = d != 0.f ? 1.f / d : 0.f;
        uint16_t h = or_f2h(d);
        b[0] = (uint8_t)(h & 0xff);
        b[1] = (uint8_t)(h >> 8);
        for (int j = 0; j < QK8_0; j++) b[2 + j] = (uint8_t)(int8_t)roundf(xs[j] * id);
    }
}

/* ------------------------------------------------------- integer block dots */

/* Per super-block integer sums of Q4_K x Q8_K:
 * isum = sum_j sc_j * (sum_{l in sub-block j} q4*q8),  msum = sum_j m_j*(bsum_2j+bsum_2j+1). */
static inline void q4k_block_ints(const uint8_t* blk, const or_q8k* y, int32_t* isum, int32_t* msum) {
    uint8_t sc[8], mn[8];
    q4k_scale_min(blk + 4, sc, mn);
    const uint8_t* qs = blk + 16;
    int32_t is = 0, ms = 0;
    for (int g = 0; g < 4; g++) {
        int32_t lo = 0, hi = 0;
        for (int l = 0; l < 32; l++) {
            lo += (int32_t)(qs[32 * g + l] & 0x0f) * y->qs[64 * g + l];
            hi += (int32_t)(qs[32 * g + l] >> 4) * y->qs[64 * g + 32 + l];
        }
        is += (int32_t)sc[2 * g] * lo + (int32_t)sc[2 * g + 1] * hi;
    }
    for (int j = 0; j < 16; j++) ms += (int32_t)y->bsums[j] * mn[j / 2];
    *isum = is;
    *msum = ms;
}

static inline int32_t q6k_block_int(const uint8_t* blk, const or_q8k* y) {
    const int8_t* sc = (const int8_t*)(blk + 192);
    int32_t is = 0;
    for (int h = 0; h < 2; h++) {
        const uint8_t* ql = blk + 64 * h;
        const uint8_t* qh = blk + 128 + 32 * h;
        const int8_t* q8 = y->qs + 128 * h;
        int32_t s[8] = {0};
        for (int l = 0; l < 32; l++) {
            int q1 = ((ql[l] & 0x0f) | (((qh[l] >> 0) & 3) << 4)) - 32;
            int q2 = ((ql[l + 32] & 0x0f) | (((qh[l] >> 2) & 3) << 4)) - 32;
            int q3 = ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
            int q4 = ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
            int sub = l >> 4;
            s[sub + 0] += q1 * q8[l];
            s[sub + 2] += q2 * q8[l + 32];
            s[sub + 4] += q3 * q8[l + 64];
            s[sub + 6] += q4 * q8[l + 96];
        }
        for (int j = 0; j < 8; j++) is += (int32_t)sc[8 * h + j] * s[j];
    }
    return is;
}

/* Per super-block integer sums of Q5_K x Q8_K (as Q4_K with 5-bit q). */
static inline void q5k_block_ints(const uint8_t* blk, const or_q8k* y, int32_t* isum, int32_t* msum) {
    uint8_t sc[8], mn[8];
    q4k_scale_min(blk + 4, sc, mn);
    int32_t is = 0, ms = 0;
    for (int j = 0; j < 8; j++) {
        int32_t s = 0;
        for (int l = 0; l < 32; l++) s += (int32_t)q5k_val(blk, 32 * j + l) * y->qs[32 * j + l];
        is += (int32_t)sc[j] * s;
    }
    for (int j = 0; j < 16; j++) ms += (int32_t)y->bsums[j] * mn[j / 2];
    *isum = is;
    *msum = ms;
}

/* Q2_K value q (0..3) of element e, and the 4-bit scale / min of its 16-element group. */
static inline int q2k_q(const uint8_t* blk, int e) { return (blk[16 + 32 * (e >> 7) + (e & 31)] >> (2 * ((e >> 5) & 3))) & 3; }

/* Per super-block integer sums of Q2_K x Q8_K (candle BlockQ2K::vec_dot_unopt):
 * isum = sum_g (sc_g & 15) * dot_g, msum = sum_g (sc_g >> 4) * bsum_g over 16-element groups. */
static inline void q2k_block_ints(const uint8_t* blk, const or_q8k* y, int32_t* isum, int32_t* msum) {
    int32_t is = 0, ms = 0;
    for (int g = 0; g < 16; g++) {
        int32_t s = 0;
        for (int l = 0; l < 16; l++) s += q2k_q(blk, 16 * g + l) * y->qs[16 * g + l];
        is += (int32_t)(blk[g] & 0x0f) * s;
        ms += (int32_t)(blk[g] >> 4) * y->bsums[g];
    }
    *isum = is;
    *msum = ms;
}

/* Q3_K value q (-4..3) of element e (or_dequant_q3k's q). */
static inline int q3k_q(const uint8_t* blk, int e) {
    const int ql = (blk[32 + 32 * (e >> 7) + (e & 31)] >> (2 * ((e >> 5) & 3))) & 3;
    return ql - ((((blk[e & 31] >> (e >> 5)) & 1) ^ 1) << 2);
}

/* Per super-block integer sum of Q3_K x Q8_K: sum_g scale_g * dot_g (6-bit scales - 32). */
static inline int32_t q3k_block_int(const uint8_t* blk, const or_q8k* y) {
    int32_t is = 0;
    for (int g = 0; g < 16; g++) {
        int32_t s = 0;
        for (int l = 0; l < 16; l++) s += q3k_q(blk, 16 * g + l) * y->qs[16 * g + l];
        is += q3k_scale(blk + 96, g) * s;
    }
    return is;
}

/* Q4_1 / Q5_1 unsigned code of element l (0..31) of a block (d m [qh] qs layout). */
static inline int q41_code(const uint8_t* blk, int l) {
    const uint8_t* qs = blk + 4;
    return l < 16 ? (qs[l] & 0x0f) : (qs[l - 16] >> 4);
}
static inline int q51_code(const uint8_t* blk, int l) {
    const uint8_t* qs = blk + 8;
    return (l < 16 ? (qs[l] & 0x0f) : (qs[l - 16] >> 4)) | (q5_hbit(blk + 4, l) << 4);
}

/* candle BlockQ4_1 / BlockQ5_1 ::vec_dot_unopt block sum against a Q8_1 block: sum_l q_l y_l.
 * candle's Q8_1 quants and d equal Q8_0's (d = amax/127, q = round(x/d)), so the Q8_0 block
 * stands in; its s = f16(f16(sum y) * d) is formed in q81_s. */
static inline int32_t q41_q51_block_int(int type, const uint8_t* blk, const uint8_t* xb) {
    const int8_t* y = (const int8_t*)(xb + 2);
    int32_t s = 0;
    for (int l = 0; l < 32; l++) s += (type == OR_Q4_1 ? q41_code(blk, l) : q51_code(blk, l)) * y[l];
    return s;
}
static inline float q81_s(const uint8_t* xb) {
    const int8_t* y = (const int8_t*)(xb + 2);
    int32_t sum = 0;
    for (int l = 0; l < 32; l++) sum += y[l];
    return or_h2f(or_f2h(or_h2f(or_f2h((float)sum)) * or_h2f(rd16(xb))));
}

/* candle BlockQ4_0::vec_dot_unopt block sum: sum_j (lo_j - 8) y_j + (hi_j - 8) y_{j+16}. */
static inline int32_t q40_block_int(const uint8_t* blk, const uint8_t* xb) {
    const int8_t* y = (const int8_t*)(xb + 2);
    int32_t s = 0;
    for (int j = 0; j < 16; j++) s += ((blk[2 + j] & 0x0f) - 8) * y[j] + ((blk[2 + j] >> 4) - 8) * y[j + 16];
    return s;
}

/* candle BlockQ5_0::vec_dot_unopt block sum, q = nibble | hbit << 4, minus 16. */
static inline int32_t q50_block_int(const uint8_t* blk, const uint8_t* xb) {
    const int8_t* y = (const int8_t*)(xb + 2);
    const uint8_t* qh = blk + 2;
    const uint8_t* qs = blk + 6;
    int32_t s = 0;
    for (int j = 0; j < 16; j++)
        s += (((qs[j] & 0x0f) | (q5_hbit(qh, j) << 4)) - 16) * y[j] +
             (((qs[j] >> 4) | (q5_hbit(qh, j + 16) << 4)) - 16) * y[j + 16];
    return s;
}

static inline int32_t q80_block_int(const uint8_t* blk, const uint8_t* xb) {
    const int8_t* a = (const int8_t*)(blk + 2);
    const int8_t* b = (const int8_t*)(xb + 2);
    int32_t s = 0;
    for (int l = 0; l < 32; l++) s += (int32_t)a[l] * b[l];
    return s;
}

/* Exported per-block integer sums for one weight row (test hook). msum may be NULL for
 * formats without mins.  xq: or_q8k[] for Q4_K/Q5_K/Q6_K, 34-byte Q8_0 blocks for
 * Q8_0/Q4_0/Q5_0. */
int or_block_dots(int type, const void* wrow, const void* xq, int nb, int32_t* isum, int32_t* msum) {
    const uint8_t* w = (const uint8_t*)wrow;
    for (int b = 0; b < nb; b++) {
        if (type == OR_Q4_K) {
            int32_t m;
            q4k_block_ints(w + (size_t)b * Q4K_BYTES, (const or_q8k*)xq + b, isum + b, &m);
            if (msum) msum[b] = m;
        } else if (type == OR_Q6_K) {
            isum[b] = q6k_block_int(w + (size_t)b * Q6K_BYTES, (const or_q8k*)xq + b);
            if (msum) msum[b] = 0;
        } else if (type == OR_Q8_0) {
            isum[b] = q80_block_int(w + (size_t)b * Q80_BYTES, (const uint8_t*)xq + (size_t)b * Q80_BYTES);
            if (msum) msum[b] = 0;
        } else if (type == OR_Q5_K) {
            int32_t m;
            q5k_block_ints(w + (size_t)b * Q5K_BYTES, (const or_q8k*)xq + b, isum + b, &m);
            if (msum) msum[b] = m;
        } else if (type == OR_Q2_K) {
            int32_t m;
            q2k_block_ints(w + (size_t)b * Q2K_BYTES, (const or_q8k*)xq + b, isum + b, &m);
            if (msum) msum[b] = m;
        } else if (type == OR_Q3_K) {
            isum[b] = q3k_block_int(w + (size_t)b * Q3K_BYTES, (const or_q8k*)xq + b);
            if (msum) msum[b] = 0;
        } else if (type == OR_Q4_0) {
            isum[b] = q40_block_int(w + (size_t)b * Q40_BYTES, (const uint8_t*)xq + (size_t)b * Q80_BYTES);
            if (msum) msum[b] = 0;
        } else if (type == OR_Q4_1 || type == OR_Q5_1) {
            const size_t bb = type == OR_Q4_1 ? Q41_BYTES : Q51_BYTES;
            isum[b] = q41_q51_block_int(type, w + (size_t)b * bb, (const uint8_t*)xq + (size_t)b * Q80_BYTES);
            if (msum) msum[b] = 0;
        } else if (type == OR_Q5_0) {
            isum[b] = q50_block_int(w + (size_t)b * Q50_BYTES, (const uint8_t*)xq + (size_t)b * Q80_BYTES);
            if (msum) msum[b] = 0;
        } else {
            return -1;
        }
    }
    return 0;
}

/* ------------------------------------------------------------------ vec dots */

/* Eight int8 values at p as eight int32 lanes. */
static inline __m256i ld8_epi32(const int8_t* p) {
    return _mm256_cvtepi8_epi32(_mm_loadl_epi64((const __m128i*)p));
}

/* Lanes summed in order 0..7, as the scalar loop does. */
static inline float sum8_in_order(__m256 v) {
    float t[8];
    _mm256_storeu_ps(t, v);
    float s = 0.f;
    for (int l = 0; l < 8; l++) s += t[l];
    return s;
}

static float vec_dot_q4k_avx2(int n, const uint8_t* w, const or_q8k* y) {
    __m256 sums = _mm256_setzero_ps();
    float sumf = 0.f;
    const __m256i m4 = _mm256_set1_epi8(0x0f);
    for (int b = 0; b < n / QK_K; b++) {
        const uint8_t* blk = w + (size_t)b * Q4K_BYTES;
        uint8_t sc[8], mn[8];
        q4k_scale_min(blk + 4, sc, mn);
        const uint8_t* qs = blk + 16;
        int8_t a[QK_K];
        for (int g = 0; g < 4; g++) {  /* low nibbles: elements 64g..64g+31, high: +32 */
            const __m256i q = _mm256_loadu_si256((const __m256i*)(qs + 32 * g));
            _mm256_storeu_si256((__m256i*)(a + 64 * g), _mm256_and_si256(q, m4));
            _mm256_storeu_si256((__m256i*)(a + 64 * g + 32), _mm256_and_si256(_mm256_srli_epi16(q, 4), m4));
        }
        int32_t sumi = 0;
        for (int j = 0; j < 16; j++) sumi += (int32_t)y[b].bsums[j] * mn[j / 2];
        __m256i aux = _mm256_setzero_si256();
        for (int s8 = 0; s8 < 8; s8++) {
            const __m256i scale = _mm256_set1_epi32(sc[s8]);
            for (int k4 = 0; k4 < 4; k4++) {
                const int idx = 32 * s8 + 8 * k4;
                const __m256i prod = _mm256_mullo_epi32(ld8_epi32(y[b].qs + idx), ld8_epi32(a + idx));
                aux = _mm256_add_epi32(aux, _mm256_mullo_epi32(scale, prod));
            }
        }
        const float d = or_h2f(rd16(blk)) * y[b].d;
        sums = _mm256_add_ps(sums, _mm256_mul_ps(_mm256_set1_ps(d), _mm256_cvtepi32_ps(aux)));
        const float dmin = or_h2f(rd16(blk + 2)) * y[b].d;
        sumf -= dmin * (float)sumi;
    }
    return sumf + sum8_in_order(sums);
}

static float vec_dot_q6k_avx2(int n, const uint8_t* w, const or_q8k* y) {
    __m256 sums = _mm256_setzero_ps();
    const __m256i m4 = _mm256_set1_epi8(0x0f), m2 = _mm256_set1_epi8(0x03), k32 = _mm256_set1_epi8(32);
    for (int b = 0; b < n / QK_K; b++) {
        const uint8_t* blk = w + (size_t)b * Q6K_BYTES;
        const int8_t* sc = (const int8_t*)(blk + 192);
        int8_t a[QK_K];
        for (int h = 0; h < 2; h++) {  /* elements 128h + l, +32, +64, +96 (q6k_val) */
            const __m256i ql0 = _mm256_loadu_si256((const __m256i*)(blk + 64 * h));
            const __m256i ql1 = _mm256_loadu_si256((const __m256i*)(blk + 64 * h + 32));
            const __m256i qh = _mm256_loadu_si256((const __m256i*)(blk + 128 + 32 * h));
            const __m256i h0 = _mm256_slli_epi16(_mm256_and_si256(qh, m2), 4);
            const __m256i h1 = _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(qh, 2), m2), 4);
            const __m256i h2 = _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(qh, 4), m2), 4);
            const __m256i h3 = _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(qh, 6), m2), 4);
            const __m256i q1 = _mm256_or_si256(_mm256_and_si256(ql0, m4), h0);
            const __m256i q2 = _mm256_or_si256(_mm256_and_si256(ql1, m4), h1);
            const __m256i q3 = _mm256_or_si256(_mm256_and_si256(_mm256_srli_epi16(ql0, 4), m4), h2);
            const __m256i q4 = _mm256_or_si256(_mm256_and_si256(_mm256_srli_epi16(ql1, 4), m4), h3);
            _mm256_storeu_si256((__m256i*)(a + 128 * h), _mm256_sub_epi8(q1, k32));
            _mm256_storeu_si256((__m256i*)(a + 128 * h + 32), _mm256_sub_epi8(q2, k32));
            _mm256_storeu_si256((__m256i*)(a + 128 * h + 64), _mm256_sub_epi8(q3, k32));
            _mm256_storeu_si256((__m256i*)(a + 128 * h + 96), _mm256_sub_epi8(q4, k32));
        }
        __m256i aux = _mm256_setzero_si256();
        for (int j = 0; j < QK_K / 16; j++) {
            const __m256i scale = _mm256_set1_epi32(sc[j]);
            for (int k2 = 0; k2 < 2; k2++) {
                const int idx = 16 * j + 8 * k2;
                const __m256i prod = _mm256_mullo_epi32(ld8_epi32(y[b].qs + idx), ld8_epi32(a + idx));
                aux = _mm256_add_epi32(aux, _mm256_mullo_epi32(scale, prod));
            }
        }
        const float d = or_h2f(rd16(blk + 208)) * y[b].d;
        sums = _mm256_add_ps(sums, _mm256_mul_ps(_mm256_set1_ps(d), _mm256_cvtepi32_ps(aux)));
    }
    return sum8_in_order(sums);
}

/* Integer sum of one Q8_0 x Q8_0 block (exact in any order). */
static inline int32_t q80_block_int_avx2(const uint8_t* blk, const uint8_t* xb) {
    const __m256i a = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i*)(blk + 2)));
    const __m256i b = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i*)(xb + 2)));
    const __m256i c = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i*)(blk + 18)));
    const __m256i e = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i*)(xb + 18)));
    __m256i s = _mm256_add_epi32(_mm256_madd_epi16(a, b), _mm256_madd_epi16(c, e));
    __m128i t = _mm_add_epi32(_mm256_castsi256_si128(s), _mm256_extracti128_si256(s, 1));
    t = _mm_add_epi32(t, _mm_shuffle_epi32(t, 0x4e));
    t = _mm_add_epi32(t, _mm_shuffle_epi32(t, 0xb1));
    return _mm_cvtsi128_si32(t);
}

/* candle Q4K::vec_dot_unopt order: eight lane sums of d*aux32, mins subtracted from sumf. */
static float vec_dot_q4k(int n, const uint8_t* w, const or_q8k* y) {
    if (g_simd) return vec_dot_q4k_avx2(n, w, y);
    float sums[8] = {0}, sumf = 0.f;
    for (int b = 0; b < n / QK_K; b++) {
        const uint8_t* blk = w + (size_t)b * Q4K_BYTES;
        uint8_t sc[8], mn[8];
        q4k_scale_min(blk + 4, sc, mn);
        const uint8_t* qs = blk + 16;
        int8_t a[QK_K];
        for (int g = 0; g < 4; g++)
            for (int l = 0; l < 32; l++) {
                a[64 * g + l] = (int8_t)(qs[32 * g + l] & 0x0f);
                a[64 * g + 32 + l] = (int8_t)(qs[32 * g + l] >> 4);
            }
        int32_t sumi = 0;
        for (int j = 0; j < 16; j++) sumi += (int32_t)y[b].bsums[j] * mn[j / 2];
        int32_t aux32[8] = {0};
        int idx = 0;
        for (int s = 0; s < 8; s++) {
            int32_t scale = sc[s];
            for (int k4 = 0; k4 < 4; k4++) {
                for (int l = 0; l < 8; l++) aux32[l] += scale * (int32_t)((int16_t)y[b].qs[idx + l] * (int16_t)a[idx + l]);
                idx += 8;
            }
        }
        float d = or_h2f(rd16(blk)) * y[b].d;
        for (int l = 0; l < 8; l++) sums[l] += d * (float)aux32[l];
        float dmin = or_h2f(rd16(blk + 2)) * y[b].d;
        sumf -= dmin * (float)sumi;
    }
    float s = 0.f;
    for (int l = 0; l < 8; l++) s += sums[l];
    return sumf + s;
}

/* candle Q6K::vec_dot_unopt order. */
static float vec_dot_q6k(int n, const uint8_t* w, const or_q8k* y) {
    if (g_simd) return vec_dot_q6k_avx2(n, w, y);
    float sums[8] = {0};
    for (int b = 0; b < n / QK_K; b++) {
        const uint8_t* blk = w + (size_t)b * Q6K_BYTES;
        const int8_t* sc = (const int8_t*)(blk + 192);
        int8_t a[QK_K];
        for (int e = 0; e < QK_K; e++) a[e] = (int8_t)q6k_val(blk, e);
        int32_t aux32[8] = {0};
        int idx = 0;
        for (int j = 0; j < QK_K / 16; j++) {
            int32_t scale = sc[j];
            for (int k2 = 0; k2 < 2; k2++) {
                for (int l = 0; l < 8; l++) aux32[l] += scale * (int32_t)((int16_t)y[b].qs[idx + l] * (int16_t)a[idx + l]);
                idx += 8;
            }
        }
        float d = or_h2f(rd16(blk + 208)) * y[b].d;
        for (int l = 0; l < 8; l++) sums[l] += d * (float)aux32[l];
    }
    float s = 0.f;
    for (int l = 0; l < 8; l++) s += sums[l];
    return s;
}

/* candle BlockQ8_0::vec_dot: sumf += (float)sumi * xd * yd, left to right. */
static float vec_dot_q80(int n, const uint8_t* w, const uint8_t* xq) {
    float sumf = 0.f;
    for (int b = 0; b < n / QK8_0; b++) {
        const uint8_t* blk = w + (size_t)b * Q80_BYTES;
        const uint8_t* xb = xq + (size_t)b * Q80_BYTES;
        int32_t si = g_simd ? q80_block_int_avx2(blk, xb) : q80_block_int(blk, xb);
        sumf += (float)si * or_h2f(rd16(blk)) * or_h2f(rd16(xb));
    }
    return sumf;
}

/* candle BlockQ5K::vec_dot_unopt: Q4_K's order with q = nibble + 16 * hbit. */
static float vec_dot_q5k(int n, const uint8_t* w, const or_q8k* y) {
    float sums[8] = {0}, sumf = 0.f;
    for (int b = 0; b < n / QK_K; b++) {
        const uint8_t* blk = w + (size_t)b * Q5K_BYTES;
        uint8_t sc[8], mn[8];
        q4k_scale_min(blk + 4, sc, mn);
        int8_t a[QK_K];
        for (int e = 0; e < QK_K; e++) a[e] = (int8_t)q5k_val(blk, e);
        int32_t sumi = 0;
        for (int j = 0; j < 16; j++) sumi += (int32_t)y[b].bsums[j] * mn[j / 2];
        int32_t aux32[8] = {0};
        int idx = 0;
        for (int s = 0; s < 8; s++) {
            int32_t scale = sc[s];
            for (int k4 = 0; k4 < 4; k4++) {
                for (int l = 0; l < 8; l++) aux32[l] += scale * (int32_t)((int16_t)y[b].qs[idx + l] * (int16_t)a[idx + l]);
                idx += 8;
            }
        }
        float d = or_h2f(rd16(blk)) * y[b].d;
        for (int l = 0; l < 8; l++) sums[l] += d * (float)aux32[l];
        float dmin = or_h2f(rd16(blk + 2)) * y[b].d;
        sumf -= dmin * (float)sumi;
    }
    float s = 0.f;
    for (int l = 0; l < 8; l++) s += sums[l];
    return sumf + s;
}

/* candle BlockQ2K::vec_dot_unopt: sumf += dall * isum - dmin * summs per super-block, with
 * dall = d_x * d_w and dmin = d_x * dmin_w. */
static float vec_dot_q2k(int n, const uint8_t* w, const or_q8k* y) {
    float sumf = 0.f;
    for (int b = 0; b < n / QK_K; b++) {
        const uint8_t* blk = w + (size_t)b * Q2K_BYTES;
        int32_t isum, summs;
        q2k_block_ints(blk, y + b, &isum, &summs);
        const float dall = y[b].d * or_h2f(rd16(blk + 80)), dmin = y[b].d * or_h2f(rd16(blk + 82));
        sumf += dall * (float)isum - dmin * (float)summs;
    }
    return sumf;
}

/* candle BlockQ3K::vec_dot_unopt: Q6_K's order (eight lane sums of d*aux32 over 8-element
 * groups, each group's products scaled by its 16-element scale). */
static float vec_dot_q3k(int n, const uint8_t* w, const or_q8k* y) {
    float sums[8] = {0};
    for (int b = 0; b < n / QK_K; b++) {
        const uint8_t* blk = w + (size_t)b * Q3K_BYTES;
        int8_t a[QK_K];
        for (int e = 0; e < QK_K; e++) a[e] = (int8_t)q3k_q(blk, e);
        int32_t aux32[8] = {0};
        int idx = 0;
        for (int j = 0; j < QK_K / 16; j++) {
            const int32_t scale = q3k_scale(blk + 96, j);
            for (int k2 = 0; k2 < 2; k2++) {
                for (int l = 0; l < 8; l++) aux32[l] += scale * (int32_t)((int16_t)y[b].qs[idx + l] * (int16_t)a[idx + l]);
                idx += 8;
            }
        }
        const float d = or_h2f(rd16(blk + 108)) * y[b].d;
        for (int l = 0; l < 8; l++) sums[l] += d * (float)aux32[l];
    }
    float s = 0.f;
    for (int l = 0; l < 8; l++) s += sums[l];
    return s;
}

/* candle BlockQ4_0 / BlockQ5_0 ::vec_dot_unopt: sumf += (float)sumi * d_w * d_x per block. */
static float vec_dot_q40_q50(int type, int n, const uint8_t* w, const uint8_t* xq) {
    const size_t bb = type == OR_Q4_0 ? Q40_BYTES : Q50_BYTES;
    float sumf = 0.f;
    for (int b = 0; b < n / QK8_0; b++) {
        const uint8_t* blk = w + (size_t)b * bb;
        const uint8_t* xb = xq + (size_t)b * Q80_BYTES;
        int32_t si = type == OR_Q4_0 ? q40_block_int(blk, xb) : q50_block_int(blk, xb);
        sumf += (float)si * or_h2f(rd16(blk)) * or_h2f(rd16(xb));
    }
    return sumf;
}

/* candle BlockQ4_1 / BlockQ5_1 ::vec_dot_unopt: sumf += sumi * d_w * d_x + m_w * s_x per block. */
static float vec_dot_q41_q51(int type, int n, const uint8_t* w, const uint8_t* xq) {
    const size_t bb = type == OR_Q4_1 ? Q41_BYTES : Q51_BYTES;
    float sumf = 0.f;
    for (int b = 0; b < n / QK8_0; b++) {
        const uint8_t* blk = w + (size_t)b * bb;
        const uint8_t* xb = xq + (size_t)b * Q80_BYTES;
        const int32_t si = q41_q51_block_int(type, blk, xb);
        sumf += (float)si * or_h2f(rd16(blk)) * or_h2f(rd16(xb)) + or_h2f(rd16(blk + 2)) * q81_s(xb);
    }
    return sumf;
}

static float vec_dot_f32(int n, const float* a, const float* b) {
    float s = 0.f;
    for (int i = 0; i < n; i++) s += a[i] * b[i];
    return s;
}

/* ------------------------------------------------------------------- matmul */

/* y[m, N] = x[m, K] . W[N, K]^T with candle QMatMul semantics: every activation row is
 * quantised to the weight's vec-dot type, then one vec_dot per output element.  F16
 * weights are dequantised to f32 first (QMatMul::from_arc dequantises F16/F32). */
int or_matmul(int type, const void* W, int N, int K, const float* x, int m, float* y) {
    if (type == OR_Q4_K || type == OR_Q5_K || type == OR_Q6_K || type == OR_Q2_K || type == OR_Q3_K) {
        if (K % QK_K) return -1;
        or_q8k* xq = (or_q8k*)malloc(sizeof(or_q8k) * (size_t)m * (K / QK_K));
        for (int r = 0; r < m; r++) or_quant_q8k(x + (size_t)r * K, K, xq + (size_t)r * (K / QK_K));
        size_t rowb = (size_t)(K / QK_K) * (size_t)or_type_block_bytes(type);
#pragma omp parallel for num_threads(g_threads) schedule(static)
        for (int n = 0; n < N; n++) {
            const uint8_t* wr = (const uint8_t*)W + rowb * n;
            for (int r = 0; r < m; r++) {
                const or_q8k* xr = xq + (size_t)r * (K / QK_K);
                y[(size_t)r * N + n] = type == OR_Q4_K   ? vec_dot_q4k(K, wr, xr)
                                       : type == OR_Q5_K ? vec_dot_q5k(K, wr, xr)
                                       : type == OR_Q2_K ? vec_dot_q2k(K, wr, xr)
                                       : type == OR_Q3_K ? vec_dot_q3k(K, wr, xr)
                                                         : vec_dot_q6k(K, wr, xr);
            }
        }
        free(xq);
        return 0;
    }
    if (type == OR_Q8_0 || type == OR_Q4_0 || type == OR_Q5_0 || type == OR_Q4_1 || type == OR_Q5_1) {
        if (K % QK8_0) return -1;
        size_t xrow = (size_t)(K / QK8_0) * Q80_BYTES;
        size_t wrow = (size_t)(K / QK8_0) * (size_t)or_type_block_bytes(type);
        uint8_t* xq = (uint8_t*)malloc(xrow * m);
        for (int r = 0; r < m; r++) or_quant_q80(x + (size_t)r * K, K, xq + xrow * r);
#pragma omp parallel for num_threads(g_threads) schedule(static)
        for (int n = 0; n < N; n++) {
            const uint8_t* wr = (const uint8_t*)W + wrow * n;
            for (int r = 0; r < m; r++)
                y[(size_t)r * N + n] = type == OR_Q8_0                      ? vec_dot_q80(K, wr, xq + xrow * r)
                                       : (type == OR_Q4_1 || type == OR_Q5_1) ? vec_dot_q41_q51(type, K, wr, xq + xrow * r)
                                                                              : vec_dot_q40_q50(type, K, wr, xq + xrow * r);
        }
        free(xq);
        return 0;
    }
    if (type == OR_F16 || type == OR_F32) {
#pragma omp parallel for num_threads(g_threads) schedule(static)
        for (int n = 0; n < N; n++) {
            float* wrow = (float*)malloc(sizeof(float) * K);
            if (type == OR_F16) or_dequant_f16((const uint16_t*)W + (size_t)n * K, K, wrow);
            else memcpy(wrow, (const float*)W + (size_t)n * K, sizeof(float) * K);
            for (int r = 0; r < m; r++) y[(size_t)r * N + n] = vec_dot_f32(K, x + (size_t)r * K, wrow);
            free(wrow);
        }
        return 0;
    }
    return -1;
}

/* -------------------------------------------------------------------- model */

/* Tensor order in or_model_desc.tensors (per layer, then globals):
 *   globals: [0] token_embd, [1] output_norm (f32), [2] output (may alias token_embd)
 *   layer l, base 3+9*l: attn_norm, attn_q, attn_k, attn_v, attn_output,
 *                        ffn_norm, ffn_gate, ffn_up, ffn_down */
typedef struct {
    int n_layers, dim, n_heads, n_kv_heads, head_dim, ffn, vocab, max_seq;
    float rope_base, rms_eps, rope_scale;
    const void** tensors;
    const int* types;
    /* qwen2 (candle quantized_qwen2): f32 q / k / v biases added after each projection
     * (biases[3l .. 3l+2], entries NULL when absent, the array NULL for none), and RoPE on
     * the two halves of each head (candle_nn::rotary_emb::rope) instead of interleaved pairs. */
    const float** biases;
    int rope_neox;
    /* gemma: GEGLU feed-forward (gelu in the tanh form of the reference's shaders/geglu.wgsl:24-25,
     * times up) and embedding rows times embd_scale (sqrt(dim)); 0 and 1.0 for the others. */
    int ffn_geglu;
    float embd_scale;
    /* Mixture of experts (candle quantized_llama MlpOrMoe::MoE), n_expert > 1: moe[l * S ...],
     * S = 4 + 3 * n_expert, holds layer l's router ([n_expert][dim], F32 or F16; NULL makes the
     * layer dense), then each expert's gate, up and down ([expert_ffn][dim], [expert_ffn][dim],
     * [dim][expert_ffn]), then a shared expert's gate, up and down ([shared_ffn] rows; NULL when
     * absent); moe_types the GGML types alike. */
    int n_expert, n_expert_used, expert_ffn, shared_ffn;
    const void** moe;
    const int* moe_types;
} or_model_desc;

typedef struct {
    or_model_desc d;
    const void** t;
    int* ty;
    float* embd;    /* token_embd dequantised to f32 [vocab, dim] (candle dequantises at load) */
    float* cos_t;   /* [max_seq, head_dim/2] */
    float* sin_t;
    float* kc;      /* [L, max_seq, n_kv, hd] f32 */
    float* vc;
    const float** b;  /* copy of desc->biases, or NULL */
    const void** moe; /* copies of desc->moe / moe_types, or NULL */
    int* moe_ty;
    int n_past;
} or_model;

/* candle quantized_llama precomput_freqs_cis: theta_i = 1/base^(i/hd) (f32 powf),
 * angle = pos * theta_i (f32), cos/sin in f32.  Linear rope scaling (reference
 * wgpu_loader.rs:337-353) divides pos by the factor; 1.0 leaves candle's table. */
void or_rope_table(int max_seq, int hd, float base, float scale, float* cos_t, float* sin_t) {
    int half = hd / 2;
    for (int p = 0; p < max_seq; p++) {
        float pos = (float)p;
        if (scale != 1.f) pos = pos / scale;
        for (int i = 0; i < half; i++) {
            float theta = 1.f / powf(base, (float)(2 * i) / (float)hd);
            float a = pos * theta;
            cos_t[(size_t)p * half + i] = cosf(a);
            sin_t[(size_t)p * half + i] = sinf(a);
        }
    }
}

void* or_model_create(const or_model_desc* desc) {
    or_model* m = (or_model*)calloc(1, sizeof(or_model));
    m->d = *desc;
    int nt = 3 + 9 * desc->n_layers;
    m->t = (const void**)malloc(sizeof(void*) * nt);
    m->ty = (int*)malloc(sizeof(int) * nt);
    memcpy(m->t, desc->tensors, sizeof(void*) * nt);
    memcpy(m->ty, desc->types, sizeof(int) * nt);
    m->d.tensors = m->t;
    m->d.types = m->ty;
    if (desc->biases) {
        m->b = (const float**)malloc(sizeof(float*) * 3 * desc->n_layers);
        memcpy(m->b, desc->biases, sizeof(float*) * 3 * desc->n_layers);
    }
    m->d.biases = m->b;
    if (desc->n_expert > 1 && desc->moe) {
        size_t nm = (size_t)desc->n_layers * (4 + 3 * (size_t)desc->n_expert);
        m->moe = (const void**)malloc(sizeof(void*) * nm);
        m->moe_ty = (int*)malloc(sizeof(int) * nm);
        memcpy(m->moe, desc->moe, sizeof(void*) * nm);
        memcpy(m->moe_ty, desc->moe_types, sizeof(int) * nm);
    }
    m->d.moe = m->moe;
    m->d.moe_types = m->moe_ty;
    size_t ne = (size_t)desc->vocab * desc->dim;
    m->embd = (float*)malloc(ne * sizeof(float));
    or_dequant(m->ty[0], m->t[0], (int64_t)ne, m->embd);
    int half = desc->head_dim / 2;
    m->cos_t = (float*)malloc(sizeof(float) * (size_t)desc->max_seq * half);
    m->sin_t = (float*)malloc(sizeof(float) * (size_t)desc->max_seq * half);
    or_rope_table(desc->max_seq, desc->head_dim, desc->rope_base, desc->rope_scale, m->cos_t, m->sin_t);
    size_t kvn = (size_t)desc->n_layers * desc->max_seq * desc->n_kv_heads * desc->head_dim;
    m->kc = (float*)calloc(kvn, sizeof(float));
    m->vc = (float*)calloc(kvn, sizeof(float));
    return m;
}

void or_model_destroy(void* p) {
    or_model* m = (or_model*)p;
    if (!m) return;
    free(m->t); free(m->ty); free(m->embd); free(m->cos_t); free(m->sin_t); free(m->kc); free(m->vc);
    free((void*)m->b);
    free((void*)m->moe); free(m->moe_ty);
    free(m);
}

/* Summation order of RMSNorm's sum of squares: 1 (default) is candle's sequential
 * Iterator::sum; n > 1 sums elements i (mod n) in n partial sums and then adds the partials
 * in order -- the order a build of the same source with n-wide SIMD reductions would take.
 * Both are valid f32 evaluations of the same formula; tests use the second to measure how
 * far a reordering of one reduction moves a model's logits (the floor any reimplementation
 * that sums in another order can reach). */
static int g_norm_lanes = 1;
void or_set_norm_lanes(int n) { g_norm_lanes = n > 1 ? (n > 64 ? 64 : n) : 1; }

/* candle_nn::ops::rms_norm (f32): m = sqrt(sum(x^2)/dim + eps); y = x / m * w. */
static void rms_norm(const float* x, const float* w, int dim, float eps, float* y) {
    float s = 0.f;
    if (g_norm_lanes <= 1) {
        for (int i = 0; i < dim; i++) s += x[i] * x[i];
    } else {
        float part[64] = {0.f};
        for (int i = 0; i < dim; i++) part[i % g_norm_lanes] += x[i] * x[i];
        for (int l = 0; l < g_norm_lanes; l++) s += part[l];
    }
    float m = sqrtf(s / (float)dim + eps);
    for (int i = 0; i < dim; i++) y[i] = x[i] / m * w[i];
}

/* candle_nn::rotary_emb::rope_i on one head vector. */
static void rope_i(float* v, int hd, const float* c, const float* s) {
    for (int i = 0; i < hd / 2; i++) {
        float x0 = v[2 * i], x1 = v[2 * i + 1];
        v[2 * i] = x0 * c[i] - x1 * s[i];
        v[2 * i + 1] = x0 * s[i] + x1 * c[i];
    }
}

/* candle_nn::rotary_emb::rope on one head vector: element i pairs with i + hd/2. */
static void rope_neox(float* v, int hd, const float* c, const float* s) {
    const int half = hd / 2;
    for (int i = 0; i < half; i++) {
        float x0 = v[i], x1 = v[i + half];
        v[i] = x0 * c[i] - x1 * s[i];
        v[i + half] = x0 * s[i] + x1 * c[i];
    }
}

/* y[r][i] += b[i] for n rows of width w (candle's broadcast_add of a projection bias). */
static void add_bias(float* y, const float* b, int n, int w) {
    if (!b) return;
    for (int r = 0; r < n; r++)
        for (int i = 0; i < w; i++) y[(size_t)r * w + i] += b[i];
}

/* GEGLU's gate activation times up, the reference's shaders/geglu.wgsl:24-25 operation order:
 * ((g * 0.5) * (1 + tanh(0.7978845608 * (g + ((0.044715 * g) * g) * g)))) * u. */
static float gelu_tanh_mul(float g, float u) {
    float g3 = 0.044715f * g * g * g;
    float t = tanhf(0.7978845608f * (g + g3));
    return g * 0.5f * (1.f + t) * u;
}

/* candle quantized_llama Mlp::forward for one row: down(act(gate(x)) * up(x)), the activation
 * silu (candle_nn::ops::silu: x / (1 + exp(-x))) or GEGLU's tanh gelu. */
static void mlp_row(int tg, const void* wg, int tu, const void* wu, int td, const void* wd, int rows, int dim,
                    const float* x, int geglu, float* g, float* u, float* y) {
    or_matmul(tg, wg, rows, dim, x, 1, g);
    or_matmul(tu, wu, rows, dim, x, 1, u);
    for (int i = 0; i < rows; i++) g[i] = geglu ? gelu_tanh_mul(g[i], u[i]) : g[i] / (1.f + expf(-g[i])) * u[i];
    or_matmul(td, wd, dim, rows, g, 1, y);
}

/* candle quantized_llama MlpOrMoe::MoE::forward over n rows, then the residual add:
 *   routing_weights = softmax_last_dim(router(x))          (max, exp(l - max), sum in order)
 *   experts sorted by weight, descending, stable (sort_by on total_cmp): the first n_used
 *   w_e = rw[e] / (sum of the chosen rw in that order)
 *   ys = 0; for e ascending among the chosen: ys = ys + mlp_e(x) * w_e   (index_add)
 * then a shared expert (the reference's wgpu_engine.rs:840-853, weight 1): ys = ys + mlp_s(x);
 * x = ys + x. */
/* Optional per-layer record of the last row's routing margin: the router-logit gap between
 * the n_used-th and the next expert (NaN for dense layers).  Tests use it to tell a routing
 * near-tie, where two correct evaluations may choose different experts, from an error. */
static float* g_route = NULL;
void or_set_route_trace(float* gaps) { g_route = gaps; }

static void moe_ffn(const or_model* m, int l, const float* xn, int n, float* x) {
    const or_model_desc* d = &m->d;
    const int E = d->n_expert, K = d->n_expert_used, eff = d->expert_ffn, sffn = d->shared_ffn, dim = d->dim;
    const size_t S = 4 + 3 * (size_t)E;
    const void** T = m->moe + (size_t)l * S;
    const int* Ty = m->moe_ty + (size_t)l * S;
    const int hmax = eff > sffn ? eff : sffn;
    float* lg = (float*)malloc(sizeof(float) * E);
    float* rw = (float*)malloc(sizeof(float) * E);
    int* order = (int*)malloc(sizeof(int) * (K > 0 ? K : 1));
    char* taken = (char*)malloc((size_t)E);
    float* g = (float*)malloc(sizeof(float) * hmax);
    float* u = (float*)malloc(sizeof(float) * hmax);
    float* y = (float*)malloc(sizeof(float) * dim);
    float* ys = (float*)malloc(sizeof(float) * dim);
    for (int i = 0; i < n; i++) {
        const float* xi = xn + (size_t)i * dim;
        or_matmul(Ty[0], T[0], E, dim, xi, 1, lg);
        float mx = -INFINITY, sum = 0.f;
        for (int e = 0; e < E; e++) if (lg[e] > mx) mx = lg[e];
        for (int e = 0; e < E; e++) rw[e] = expf(lg[e] - mx);
        for (int e = 0; e < E; e++) sum += rw[e];
        for (int e = 0; e < E; e++) rw[e] /= sum;
        memset(taken, 0, (size_t)E);
        for (int k = 0; k < K; k++) {
            int best = -1;
            for (int e = 0; e < E; e++)
                if (!taken[e] && (best < 0 || rw[e] > rw[best])) best = e;
            order[k] = best;
            taken[best] = 1;
        }
        float ssel = 0.f;
        for (int k = 0; k < K; k++) ssel += rw[order[k]];
        if (g_route && i == n - 1) {
            float next = -INFINITY;
            for (int e = 0; e < E; e++)
                if (!taken[e] && lg[e] > next) next = lg[e];
            float kth = INFINITY;
            for (int k = 0; k < K; k++)
                if (lg[order[k]] < kth) kth = lg[order[k]];
            g_route[l] = K < E ? kth - next : INFINITY;
        }
        for (int j = 0; j < dim; j++) ys[j] = 0.f;
        for (int e = 0; e < E; e++) {
            if (!taken[e]) continue;
            const float we = rw[e] / ssel;
            mlp_row(Ty[1 + 3 * e], T[1 + 3 * e], Ty[2 + 3 * e], T[2 + 3 * e], Ty[3 + 3 * e], T[3 + 3 * e], eff, dim, xi,
                    d->ffn_geglu, g, u, y);
            for (int j = 0; j < dim; j++) ys[j] = ys[j] + y[j] * we;
        }
        if (T[1 + 3 * E]) {
            mlp_row(Ty[1 + 3 * E], T[1 + 3 * E], Ty[2 + 3 * E], T[2 + 3 * E], Ty[3 + 3 * E], T[3 + 3 * E], sffn, dim, xi,
                    d->ffn_geglu, g, u, y);
            for (int j = 0; j < dim; j++) ys[j] = ys[j] + y[j];
        }
        for (int j = 0; j < dim; j++) x[(size_t)i * dim + j] = ys[j] + x[(size_t)i * dim + j];
    }
    free(lg); free(rw); free(order); free(taken); free(g); free(u); free(y); free(ys);
}

/* One forward call: tokens[0..n) at absolute positions pos..pos+n-1, attending the
 * cached positions [0, pos).  Writes the last position's logits [vocab] and, when
 * hidden_out is non-NULL, the final-normed hidden state of the last position [dim].
 * Mirrors ModelWeights::forward (mask only when n > 1). Returns 0, or -1 on overflow. */
int or_forward(void* p, const uint32_t* tokens, int n, int pos, float* logits, float* hidden_out) {
    or_model* m = (or_model*)p;
    const or_model_desc* d = &m->d;
    if (n <= 0 || pos < 0 || pos + n > d->max_seq) return -1;
    for (int i = 0; i < n; i++)
        if (tokens[i] >= (uint32_t)d->vocab) return -1;
    int dim = d->dim, hd = d->head_dim, nh = d->n_heads, nkv = d->n_kv_heads, ffn = d->ffn;
    int qd = nh * hd, kvd = nkv * hd, half = hd / 2, group = nh / nkv;
    float* x = (float*)malloc(sizeof(float) * (size_t)n * dim);
    float* xn = (float*)malloc(sizeof(float) * (size_t)n * dim);
    float* q = (float*)malloc(sizeof(float) * (size_t)n * qd);
    float* k = (float*)malloc(sizeof(float) * (size_t)n * kvd);
    float* v = (float*)malloc(sizeof(float) * (size_t)n * kvd);
    float* att = (float*)malloc(sizeof(float) * (size_t)n * qd);
    float* tmp = (float*)malloc(sizeof(float) * (size_t)n * dim);
    float* g = (float*)malloc(sizeof(float) * (size_t)n * ffn);
    float* u = (float*)malloc(sizeof(float) * (size_t)n * ffn);
    for (int i = 0; i < n; i++) memcpy(x + (size_t)i * dim, m->embd + (size_t)tokens[i] * dim, sizeof(float) * dim);
    if (d->embd_scale != 0.f && d->embd_scale != 1.f)
        for (size_t i = 0; i < (size_t)n * dim; i++) x[i] = x[i] * d->embd_scale;
    float scale = (float)(1.0 / sqrt((double)hd));
    int kv_len = pos + n;
    for (int l = 0; l < d->n_layers; l++) {
        const void** T = m->t + 3 + 9 * l;
        const int* Ty = m->ty + 3 + 9 * l;
        for (int i = 0; i < n; i++) rms_norm(x + (size_t)i * dim, (const float*)T[0], dim, d->rms_eps, xn + (size_t)i * dim);
        or_matmul(Ty[1], T[1], qd, dim, xn, n, q);
        or_matmul(Ty[2], T[2], kvd, dim, xn, n, k);
        or_matmul(Ty[3], T[3], kvd, dim, xn, n, v);
        if (m->b) {
            add_bias(q, m->b[3 * l], n, qd);
            add_bias(k, m->b[3 * l + 1], n, kvd);
            add_bias(v, m->b[3 * l + 2], n, kvd);
        }
        float* kc = m->kc + (size_t)l * d->max_seq * kvd;
        float* vc = m->vc + (size_t)l * d->max_seq * kvd;
        for (int i = 0; i < n; i++) {
            const float* c = m->cos_t + (size_t)(pos + i) * half;
            const float* s = m->sin_t + (size_t)(pos + i) * half;
            for (int h = 0; h < nh; h++) {
                if (d->rope_neox) rope_neox(q + (size_t)i * qd + h * hd, hd, c, s);
                else rope_i(q + (size_t)i * qd + h * hd, hd, c, s);
            }
            for (int h = 0; h < nkv; h++) {
                if (d->rope_neox) rope_neox(k + (size_t)i * kvd + h * hd, hd, c, s);
                else rope_i(k + (size_t)i * kvd + h * hd, hd, c, s);
            }
            memcpy(kc + (size_t)(pos + i) * kvd, k + (size_t)i * kvd, sizeof(float) * kvd);
            memcpy(vc + (size_t)(pos + i) * kvd, v + (size_t)i * kvd, sizeof(float) * kvd);
        }
        /* softmax(q k^T * scale [+ causal mask]) v per (row, head); repeat_kv maps head h
         * to kv head h / group. */
#pragma omp parallel for num_threads(g_threads) collapse(2) schedule(static)
        for (int i = 0; i < n; i++) {
            for (int h = 0; h < nh; h++) {
                float* sc = (float*)malloc(sizeof(float) * kv_len);
                const float* qv = q + (size_t)i * qd + h * hd;
                int kh = h / group;
                int lim = pos + i + 1; /* causal: keys 0..pos+i */
                float mx = -INFINITY;
                for (int t = 0; t < kv_len; t++) {
                    if (t >= lim) { sc[t] = -INFINITY; continue; }
                    float dot = vec_dot_f32(hd, qv, kc + (size_t)t * kvd + kh * hd);
                    sc[t] = dot * scale;
                    if (sc[t] > mx) mx = sc[t];
                }
                float sum = 0.f;
                for (int t = 0; t < kv_len; t++) { sc[t] = expf(sc[t] - mx); }
                for (int t = 0; t < kv_len; t++) sum += sc[t];
                for (int t = 0; t < kv_len; t++) sc[t] /= sum;
                float* o = att + (size_t)i * qd + h * hd;
                for (int e = 0; e < hd; e++) o[e] = 0.f;
                for (int t = 0; t < kv_len; t++) {
                    const float* vv = vc + (size_t)t * kvd + kh * hd;
                    for (int e = 0; e < hd; e++) o[e] += sc[t] * vv[e];
                }
                free(sc);
            }
        }
        if (g_trace) {
            memcpy(g_trace + (size_t)(3 * l) * dim, q + (size_t)(n - 1) * qd, sizeof(float) * qd);
            memcpy(g_trace + (size_t)(3 * l + 1) * dim, att + (size_t)(n - 1) * qd, sizeof(float) * qd);
        }
        or_matmul(Ty[4], T[4], dim, qd, att, n, tmp);
        for (size_t i = 0; i < (size_t)n * dim; i++) x[i] = tmp[i] + x[i];
        for (int i = 0; i < n; i++) rms_norm(x + (size_t)i * dim, (const float*)T[5], dim, d->rms_eps, xn + (size_t)i * dim);
        if (m->moe && m->moe[(size_t)l * (4 + 3 * (size_t)d->n_expert)]) {
            moe_ffn(m, l, xn, n, x);
        } else {
            or_matmul(Ty[6], T[6], ffn, dim, xn, n, g);
            or_matmul(Ty[7], T[7], ffn, dim, xn, n, u);
            for (size_t i = 0; i < (size_t)n * ffn; i++) {
                float a = g[i];
                g[i] = d->ffn_geglu ? gelu_tanh_mul(a, u[i]) : a / (1.f + expf(-a)) * u[i];
            }
            or_matmul(Ty[8], T[8], dim, ffn, g, n, tmp);
            for (size_t i = 0; i < (size_t)n * dim; i++) x[i] = tmp[i] + x[i];
        }
        if (g_trace) memcpy(g_trace + (size_t)(3 * l + 2) * dim, x + (size_t)(n - 1) * dim, sizeof(float) * dim);
    }
    float* last = x + (size_t)(n - 1) * dim;
    rms_norm(last, (const float*)m->t[1], dim, d->rms_eps, xn);
    if (hidden_out) memcpy(hidden_out, xn, sizeof(float) * dim);
    or_matmul(m->ty[2], m->t[2], d->vocab, dim, xn, 1, logits);
    m->n_past = kv_len;
    free(x); free(xn); free(q); free(k); free(v); free(att); free(tmp); free(g); free(u);
    return 0;
}

/* candle LogitsProcessor::sample_argmax: Iterator::max_by(total_cmp) keeps the LAST of
 * equal maxima, so ties resolve to the highest index. */
uint32_t or_argmax(const float* logits, int n) {
    int best = 0;
    for (int i = 1; i < n; i++)
        if (!(logits[i] < logits[best])) best = i;
    return (uint32_t)best;
}

/* candle_engine.rs:87-101 apply_repeat_penalty: every entry of `seen` (duplicates
 * included) divides a non-negative logit by the penalty or multiplies a negative one. */
void or_repeat_penalty(float* logits, int n, const uint32_t* seen, int n_seen, float penalty) {
    if (fabsf(penalty - 1.f) < 1.1920929e-7f) return;
    for (int i = 0; i < n_seen; i++) {
        uint32_t id = seen[i];
        if (id < (uint32_t)n) {
            if (logits[id] >= 0.f) logits[id] /= penalty;
            else logits[id] *= penalty;
        }
    }
}
