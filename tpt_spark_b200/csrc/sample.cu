// sample.cu -- the next token from the logits on the device: repeat penalty, temperature,
// top-p (nucleus) and one seeded draw, as a short chain of grid kernels.
//
// Replaces the per-token logits readback and host-side LogitsProcessor of the reference's
// decode loop (candle_engine.rs:87-101 apply_repeat_penalty, :257-267 LogitsProcessor::new(42,
// temperature, top_p) -> candle's softmax / sample_topp / sample_multinomial;
// wgpu_engine.rs:868-888): 4 bytes leave the GPU per token instead of 513 KB, and no host
// sort of the vocabulary.
//
// Semantics, in order:
//   1. repeat penalty: a logit is divided by `penalty` (multiplied when negative) once per
//      occurrence of its token in the context -- the reference's loop over `seen`, duplicates
//      included, skipped when |penalty - 1| < FLT_EPSILON; the same IEEE operations in the
//      same order per logit, so bit-identical to the host loop;
//   2. temperature below 1e-7 (candle's LogitsProcessor::new takes such a temperature as
//      none): argmax of the penalised logits, ties to the highest index (candle's
//      sample_argmax keeps the last maximum);
//   3. otherwise x / temperature, e = exp(x - max) (softmax numerators);
//   4. top-p in (0, 1): candle's sample_topp walks the tokens in descending order of
//      probability (a stable sort) and keeps each while the sum of those before it is below
//      top_p.  Here every token whose strictly larger tokens sum to less than top_p is kept:
//      the same set unless several tokens tie at the cut, where candle keeps only those of
//      them that come first in index order while its running sum stays below top_p and this
//      kernel keeps them all.  Here the masses are fixed
//      point (m = floor(e * 2^40), summed in 64-bit integers, so the result does not depend on
//      the order of atomics or on the grid) and the cut is found exactly by a three-level radix
//      select over the bit patterns of e (10 + 10 + 10 bits, 1024 buckets per level): the kept
//      set is every e at or above the cut value;
//   5. one draw r in [0, sum of kept masses) from SplitMix64 (Steele, Lea and Flood 2014) of
//      (seed, step), and the token whose inclusive prefix of kept masses in index order first
//      exceeds r.  The draw is reproducible for a seed but is not candle's StdRng stream.
// The sampled token's context count is incremented (the next step's penalty), the step
// counter advanced, and the token optionally chained as the next decode input (as argmax).
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "common.cuh"
#include "kernels.h"

namespace tptc {

namespace {

constexpr float kFix = 1099511627776.f;  // 2^40: fixed-point scale of the masses (e <= 1)

__device__ __forceinline__ unsigned long long mass(float e) { return __float2ull_rz(e * kFix); }

// SplitMix64 output function over the state seed + (step + 1) * golden gamma.
__device__ __forceinline__ unsigned long long splitmix64(unsigned long long seed, unsigned long long step) {
    unsigned long long z = seed + (step + 1ull) * 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

// ---------------------------------------------------------------- the grid
//
// Six short kernels over CTA-contiguous index ranges of kR tokens (one CTA of kGT threads
// each), chained on the stream (programmatic dependent launch in the decode graph): the
// one-CTA form walked the 128k-token vocabulary five times on one SM (156-196 us).  Every
// quantity that crosses CTAs is a maximum, an integer sum or a deterministic function of
// integer sums, so the token, the cut and the masses are the same bits whatever the grid.
//   K1 penalty, then per-CTA argmax (greedy) or x / T into scratch and its maximum
//   K2 greedy: the token.  Otherwise e = exp(x - max) into scratch, per-CTA fixed-point mass
//      sums and the first radix level's histogram (top 10 bits of e)
//   K3 second radix level (the 10 bits below the first level's bucket)
//   K4 third radix level
//   K5 the cut, and each CTA's kept mass
//   K6 the draw: the CTA whose kept-mass range holds it walks its range
// Work area (SampleParams::work, kSampleWorkBytes): three 1024-bucket histograms, then per
// CTA: maximum, argmax value and index, mass sum, kept mass.
constexpr int kGT = 256;               // threads per CTA
constexpr int kR = 1024;               // tokens per CTA (4 per thread)
constexpr int kMaxG = 256;             // CTAs at most (vocabularies up to 256k tokens)
struct SampleWork {
    unsigned long long hist[3][1024];
    float maxp[kMaxG];
    float argv[kMaxG];
    int argi[kMaxG];
    unsigned long long massp[kMaxG];
    unsigned long long keptp[kMaxG];
};
static_assert(sizeof(SampleWork) <= kSampleWorkBytes, "sample work area");

__device__ __forceinline__ bool arg_better(float v, int i, float bv, int bi) {
    return i >= 0 && (bi < 0 || v > bv || (v == bv && i > bi));
}

__device__ __forceinline__ unsigned long long block_sum_g(unsigned long long v, unsigned long long* red) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    unsigned long long t = 0;
    for (int w = 0; w < kGT / 32; w++) t += red[w];
    return t;
}

__device__ __forceinline__ bool is_greedy(const SampleParams& p) { return !(p.temperature >= 1e-7f); }
__device__ __forceinline__ bool is_nucleus(const SampleParams& p) { return p.top_p > 0.f && p.top_p < 1.f; }
__host__ __device__ __forceinline__ int grid_of(int V) { return (V + kR - 1) / kR; }

// Level of the radix select over a single-copy histogram (find_bucket's rule).  Warp 0 only.
__device__ __forceinline__ int find_bucket1(const unsigned long long* hist, unsigned long long above,
                                            unsigned long long target, unsigned long long* above_out) {
    const int lane = threadIdx.x & 31;
    unsigned long long s = 0;
    for (int j = 0; j < 32; j++) s += hist[1023 - 32 * lane - j];
    unsigned long long incl = s;
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
    }
    const unsigned long long excl = incl - s;
    const unsigned ball = __ballot_sync(0xffffffffu, above + incl >= target);
    if (ball == 0) return 1024;
    const int l = __ffs(ball) - 1;
    int found = 1024;
    unsigned long long fa = 0;
    if (lane == l) {
        unsigned long long run = above + excl;
        for (int j = 0; j < 32; j++) {
            const int b = 1023 - 32 * lane - j;
            const unsigned long long hb = hist[b];
            if (run + hb >= target) {
                found = b;
                fa = run;
                break;
            }
            run += hb;
        }
    }
    found = __shfl_sync(0xffffffffu, found, l);
    fa = __shfl_sync(0xffffffffu, fa, l);
    *above_out = fa;
    return found;
}

// The first `levels` radix levels from the histograms: *prefix, and whether the target lies
// beyond the prefix found so far (*whole; then *prefix is what was found before that level).
// Every thread of the CTA gets the result.
__device__ __forceinline__ void radix_levels(const SampleWork& w, unsigned long long target, int levels,
                                             unsigned int* prefix_out, bool* whole_out, int* done_out) {
    __shared__ unsigned int sp;
    __shared__ int sw, sd;
    if (threadIdx.x < 32) {
        unsigned long long above = 0;
        unsigned int prefix = 0;
        bool whole = false;
        int done = 0;
        for (int level = 0; level < levels; level++) {
            unsigned long long a2 = 0;
            const int b = find_bucket1(w.hist[level], above, target, &a2);
            if (b >= 1024) {
                whole = true;
                break;
            }
            above = a2;
            prefix = (prefix << 10) | (unsigned int)b;
            done++;
        }
        if (threadIdx.x == 0) {
            sp = prefix;
            sw = whole ? 1 : 0;
            sd = done;
        }
    }
    __syncthreads();
    *prefix_out = sp;
    *whole_out = sw != 0;
    *done_out = sd;
}

__device__ __forceinline__ unsigned long long total_mass(const SampleWork& w, int G, unsigned long long* red) {
    unsigned long long v = threadIdx.x < G ? w.massp[threadIdx.x] : 0ull;
    return block_sum_g(v, red);
}

__device__ __forceinline__ unsigned long long nucleus_target(const SampleParams& p, unsigned long long total) {
    // keep iff the strictly larger mass G < top_p * total; for integer G that is
    // G < ceil(top_p * total) (>= 1, so the largest token is always kept)
    return (unsigned long long)ceil((double)p.top_p * (double)total);
}

// The token's bookkeeping: output, context count, step, chaining, debug words.  One thread.
__device__ __forceinline__ void finish(const SampleParams& p, int tok, bool greedy, unsigned int cut,
                                       unsigned long long kept, unsigned long long total) {
    if (tok < 0) tok = 0;
    *p.out_tok = (uint32_t)tok;
    if (p.counts) p.counts[tok] += 1;
    if (p.step) *p.step += 1;
    if (p.next_tok) *p.next_tok = (uint32_t)tok;
    if (p.pos) {
        const int ps = *p.pos;
        if (p.history) p.history[ps] = (uint32_t)tok;
        *p.pos = ps + 1;
    }
    if (p.dbg) {
        p.dbg[0] = greedy ? 0ull : (unsigned long long)cut;
        p.dbg[1] = greedy ? 0ull : kept;
        p.dbg[2] = greedy ? 0ull : total;
    }
}

__global__ void __launch_bounds__(kGT) sample_k1(SampleParams p) {
    __shared__ float rv[kGT / 32];
    __shared__ int ri[kGT / 32];
    pdl_wait();
    pdl_launch_dependents();
    SampleWork& w = *reinterpret_cast<SampleWork*>(p.work);
    const int g = blockIdx.x, t = threadIdx.x, lane = t & 31, warp = t >> 5, V = p.vocab;
    if (g == 0)
        for (int b = t; b < 3 * 1024; b += kGT) (&w.hist[0][0])[b] = 0ull;
    const bool pen = fabsf(p.penalty - 1.f) >= 1.1920929e-7f && p.counts != nullptr;
    const bool greedy = is_greedy(p);
    float mx = -INFINITY;
    int mi = -1;
    float xv[kR / kGT];
    int kv[kR / kGT];
#pragma unroll
    for (int u = 0; u < kR / kGT; u++) {
        const int i = g * kR + u * kGT + t;
        xv[u] = i < V ? p.logits[i] : 0.f;
        kv[u] = (pen && i < V) ? p.counts[i] : 0;
    }
#pragma unroll
    for (int u = 0; u < kR / kGT; u++) {
        const int i = g * kR + u * kGT + t;
        if (i >= V) break;
        float x = xv[u];
        for (int j = 0; j < kv[u]; j++) x = x >= 0.f ? __fdiv_rn(x, p.penalty) : __fmul_rn(x, p.penalty);
        if (greedy) {
            if (arg_better(x, i, mx, mi)) {
                mx = x;
                mi = i;
            }
        } else {
            x = __fdiv_rn(x, p.temperature);
            p.scratch[i] = x;
            mx = fmaxf(mx, x);
        }
    }
    for (int o = 16; o > 0; o >>= 1) {
        const float v2 = __shfl_xor_sync(0xffffffffu, mx, o);
        const int i2 = __shfl_xor_sync(0xffffffffu, mi, o);
        if (greedy) {
            if (arg_better(v2, i2, mx, mi)) {
                mx = v2;
                mi = i2;
            }
        } else {
            mx = fmaxf(mx, v2);
        }
    }
    if (lane == 0) {
        rv[warp] = mx;
        ri[warp] = mi;
    }
    __syncthreads();
    if (t == 0) {
        for (int k = 1; k < kGT / 32; k++) {
            if (greedy) {
                if (arg_better(rv[k], ri[k], mx, mi)) {
                    mx = rv[k];
                    mi = ri[k];
                }
            } else {
                mx = fmaxf(mx, rv[k]);
            }
        }
        if (greedy) {
            w.argv[g] = mx;
            w.argi[g] = mi;
        } else {
            w.maxp[g] = mx;
        }
    }
}

__global__ void __launch_bounds__(kGT) sample_k2(SampleParams p) {
    __shared__ unsigned long long hist[1024];
    __shared__ unsigned long long red[kGT / 32];
    __shared__ float rf[kGT / 32];
    pdl_wait();
    pdl_launch_dependents();
    SampleWork& w = *reinterpret_cast<SampleWork*>(p.work);
    const int g = blockIdx.x, t = threadIdx.x, lane = t & 31, warp = t >> 5, V = p.vocab, G = grid_of(V);
    if (is_greedy(p)) {
        if (g == 0 && t == 0) {
            float bv = -INFINITY;
            int bi = -1;
            for (int k = 0; k < G; k++)
                if (arg_better(w.argv[k], w.argi[k], bv, bi)) {
                    bv = w.argv[k];
                    bi = w.argi[k];
                }
            finish(p, bi, true, 0u, 0ull, 0ull);
        }
        return;
    }
    float mx = t < G ? w.maxp[t] : -INFINITY;
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) rf[warp] = mx;
    for (int b = t; b < 1024; b += kGT) hist[b] = 0ull;
    __syncthreads();
    mx = rf[0];
    for (int k = 1; k < kGT / 32; k++) mx = fmaxf(mx, rf[k]);
    const bool nucleus = is_nucleus(p);
    unsigned long long s = 0;
#pragma unroll
    for (int u = 0; u < kR / kGT; u++) {
        const int i = g * kR + u * kGT + t;
        if (i >= V) break;
        const float e = expf(p.scratch[i] - mx);
        p.scratch[i] = e;
        const unsigned long long m = mass(e);
        s += m;
        if (m && nucleus) atomicAdd(&hist[__float_as_uint(e) >> 20], m);
    }
    const unsigned long long tot = block_sum_g(s, red);
    if (t == 0) w.massp[g] = tot;
    if (nucleus)
        for (int b = t; b < 1024; b += kGT)
            if (hist[b]) atomicAdd(&w.hist[0][b], hist[b]);
}

// Radix level LEVEL (1 or 2: the 10 bits below the first LEVEL levels' prefix).
template <int LEVEL>
__global__ void __launch_bounds__(kGT) sample_level(SampleParams p) {
    __shared__ unsigned long long hist[1024];
    __shared__ unsigned long long red[kGT / 32];
    pdl_wait();
    pdl_launch_dependents();
    if (is_greedy(p) || !is_nucleus(p)) return;
    SampleWork& w = *reinterpret_cast<SampleWork*>(p.work);
    const int g = blockIdx.x, t = threadIdx.x, V = p.vocab, G = grid_of(V);
    const unsigned long long target = nucleus_target(p, total_mass(w, G, red));
    unsigned int prefix;
    bool whole;
    int done;
    radix_levels(w, target, LEVEL, &prefix, &whole, &done);
    if (whole) return;  // the cut lies above this level: its histogram stays unused
    for (int b = t; b < 1024; b += kGT) hist[b] = 0ull;
    __syncthreads();
    const int shp = 30 - 10 * LEVEL, shb = 20 - 10 * LEVEL;
#pragma unroll
    for (int u = 0; u < kR / kGT; u++) {
        const int i = g * kR + u * kGT + t;
        if (i >= V) break;
        const float e = p.scratch[i];
        const unsigned int bits = __float_as_uint(e);
        const unsigned long long m = mass(e);
        if (m && (bits >> shp) == prefix) atomicAdd(&hist[(bits >> shb) & 1023u], m);
    }
    __syncthreads();
    for (int b = t; b < 1024; b += kGT)
        if (hist[b]) atomicAdd(&w.hist[LEVEL][b], hist[b]);
}

// The kept-set cut from the three levels (sample_kernel's rule before the grid form).
__device__ __forceinline__ unsigned int nucleus_cut(const SampleParams& p, const SampleWork& w, int G,
                                                    unsigned long long* red, unsigned long long* total_out) {
    const unsigned long long total = total_mass(w, G, red);
    *total_out = total;
    if (!is_nucleus(p)) return 0u;
    unsigned int prefix;
    bool whole;
    int done;
    radix_levels(w, nucleus_target(p, total), 3, &prefix, &whole, &done);
    if (!whole) return prefix;
    if (!prefix) return 0u;
    int lv = 0;  // prefix of `lv` 10-bit groups: its smallest pattern
    for (unsigned int q = prefix; q; q >>= 10) lv++;
    return prefix << (30 - 10 * lv);
}

__global__ void __launch_bounds__(kGT) sample_k5(SampleParams p) {
    __shared__ unsigned long long red[kGT / 32];
    pdl_wait();
    pdl_launch_dependents();
    if (is_greedy(p)) return;
    SampleWork& w = *reinterpret_cast<SampleWork*>(p.work);
    const int g = blockIdx.x, t = threadIdx.x, V = p.vocab, G = grid_of(V);
    unsigned long long total;
    const unsigned int cut = nucleus_cut(p, w, G, red, &total);
    unsigned long long s = 0;
#pragma unroll
    for (int u = 0; u < kR / kGT; u++) {
        const int i = g * kR + u * kGT + t;
        if (i >= V) break;
        const float e = p.scratch[i];
        if (__float_as_uint(e) >= cut) s += mass(e);
    }
    const unsigned long long kept = block_sum_g(s, red);
    if (t == 0) w.keptp[g] = kept;
}

// One CTA: the draw r in [0, kept), the CTA range whose kept-mass prefix holds it, then the
// token in that range (thread-contiguous sub-ranges of kR / kGT tokens, an exclusive scan in
// index order, and the one thread whose sub-range holds r walks it).
__global__ void __launch_bounds__(kGT) sample_k6(SampleParams p) {
    __shared__ unsigned long long red[kGT / 32];
    __shared__ unsigned long long sh_u[2];
    __shared__ int sh_i[2];
    pdl_wait();
    pdl_launch_dependents();
    if (is_greedy(p)) return;
    SampleWork& w = *reinterpret_cast<SampleWork*>(p.work);
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5, V = p.vocab, G = grid_of(V);
    unsigned long long total;
    const unsigned int cut = nucleus_cut(p, w, G, red, &total);
    if (t == 0) {
        unsigned long long kept = 0;
        for (int k = 0; k < G; k++) kept += w.keptp[k];
        const unsigned long long step = p.step ? (unsigned long long)*p.step : 0ull;
        const unsigned long long r = __umul64hi(splitmix64(p.seed, step), kept);
        unsigned long long run = 0;
        int gs = G - 1;
        for (int k = 0; k < G; k++) {
            if (r < run + w.keptp[k]) {
                gs = k;
                break;
            }
            run += w.keptp[k];
        }
        sh_u[0] = r - run;  // the draw within CTA range gs
        sh_u[1] = kept;
        sh_i[0] = gs;
        sh_i[1] = -1;
    }
    __syncthreads();
    const int gs = sh_i[0];
    const unsigned long long r = sh_u[0];
    constexpr int C = kR / kGT;
    const int c0 = min(V, gs * kR + t * C), c1 = min(V, c0 + C);
    unsigned long long ts = 0;
    for (int j = c0; j < c1; j++) {
        const float e = p.scratch[j];
        if (__float_as_uint(e) >= cut) ts += mass(e);
    }
    unsigned long long incl = ts;
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
    }
    if (lane == 31) red[warp] = incl;
    __syncthreads();
    unsigned long long before = 0;  // kept mass of the warps before this one
    for (int k = 0; k < warp; k++) before += red[k];
    const unsigned long long run0 = before + incl - ts;
    if (ts && r >= run0 && r < run0 + ts) {
        unsigned long long run = run0;
        for (int j = c0; j < c1; j++) {
            const float e = p.scratch[j];
            const unsigned long long m = __float_as_uint(e) >= cut ? mass(e) : 0ull;
            if (m && run + m > r) {
                sh_i[1] = j;
                break;
            }
            run += m;
        }
    }
    __syncthreads();
    if (t == 0) finish(p, sh_i[1], false, cut, sh_u[1], total);
}

}  // namespace

cudaError_t launch_sample(const SampleParams& p, cudaStream_t st, bool pdl) {
    if (!p.logits || p.vocab <= 0 || !p.out_tok || !p.scratch || !p.work) return cudaErrorInvalidValue;
    const int G = grid_of(p.vocab);
    if (G > kMaxG) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(G);
    cfg.blockDim = dim3(kGT);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, sample_k1, p);
    if (e == cudaSuccess) e = cudaLaunchKernelEx(&cfg, sample_k2, p);
    if (e == cudaSuccess) e = cudaLaunchKernelEx(&cfg, sample_level<1>, p);
    if (e == cudaSuccess) e = cudaLaunchKernelEx(&cfg, sample_level<2>, p);
    if (e == cudaSuccess) e = cudaLaunchKernelEx(&cfg, sample_k5, p);
    if (e != cudaSuccess) return e;
    cfg.gridDim = dim3(1);
    return cudaLaunchKernelEx(&cfg, sample_k6, p);
}

}  // namespace tptc
