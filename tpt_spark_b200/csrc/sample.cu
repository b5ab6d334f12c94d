// sample.cu -- the next token from the logits on the device: repeat penalty, temperature,
// top-p (nucleus) and one seeded draw, in one CTA.
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
//      the order of atomics) and the cut is found exactly by a three-level radix select over
//      the bit patterns of e (10 + 10 + 10 bits, 1024 shared buckets per level): the kept set
//      is every e at or above the cut value;
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

constexpr int kST = 1024;  // threads of the sampling CTA
constexpr int kWarps = kST / 32;
constexpr float kFix = 1099511627776.f;  // 2^40: fixed-point scale of the masses (e <= 1)
// One CTA walks the vocabulary several times, so each pass is bound by load latency: every
// strided pass keeps kU independent loads in flight per thread.
constexpr int kU = 8;
// The radix histograms are kept in kHC copies, warp w adding into copy w % kHC: most tokens'
// masses fall into a few buckets, and same-address shared atomics from all warps serialise.
constexpr int kHC = 4;

__device__ __forceinline__ unsigned long long hsum(const unsigned long long* hist, int b) {
    unsigned long long v = 0;
#pragma unroll
    for (int c = 0; c < kHC; c++) v += hist[c * 1024 + b];
    return v;
}

__device__ __forceinline__ unsigned long long mass(float e) { return __float2ull_rz(e * kFix); }

// SplitMix64 output function over the state seed + (step + 1) * golden gamma.
__device__ __forceinline__ unsigned long long splitmix64(unsigned long long seed, unsigned long long step) {
    unsigned long long z = seed + (step + 1ull) * 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ unsigned long long block_sum_u64(unsigned long long v, unsigned long long* red) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        v = red[lane];
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) red[0] = v;
    }
    __syncthreads();
    return red[0];
}

__device__ __forceinline__ float block_max(float v, float* red) {
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        v = red[lane];
        for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (lane == 0) red[0] = v;
    }
    __syncthreads();
    return red[0];
}

// Level of the radix select: given the buckets' masses hist (kHC copies of 1024; bucket b = the
// next 10 bits of the pattern) and the mass `above` of everything larger than this level's prefix, the
// bucket in which the running sum from the top reaches `target`, and the mass above it.
// Returns 1024 when the whole level stays below the target.  Warp 0 only.
__device__ __forceinline__ int find_bucket(const unsigned long long* hist, unsigned long long above,
                                           unsigned long long target, unsigned long long* above_out) {
    const int lane = threadIdx.x & 31;
    // lane l owns buckets 1023 - 32 l .. 992 - 32 l (from the top)
    unsigned long long s = 0;
    for (int j = 0; j < 32; j++) s += hsum(hist, 1023 - 32 * lane - j);
    unsigned long long incl = s;  // inclusive prefix from the top over lanes
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
            const unsigned long long hb = hsum(hist, b);
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

__global__ void __launch_bounds__(kST, 1) sample_kernel(SampleParams p) {
    __shared__ unsigned long long hist[kHC * 1024];
    __shared__ unsigned long long redu[kWarps];
    __shared__ float redf[kWarps];
    __shared__ int redi[kWarps];
    __shared__ unsigned long long sh_u[4];
    __shared__ int sh_i[4];
    pdl_wait();
    pdl_launch_dependents();
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5, V = p.vocab;
    const bool pen = fabsf(p.penalty - 1.f) >= 1.1920929e-7f && p.counts != nullptr;
    // candle LogitsProcessor::new: a temperature below 1e-7 means none, i.e. argmax
    const bool greedy = !(p.temperature >= 1e-7f);
    int tok = 0;

    // 1-3: penalty, then argmax or x / T and its maximum
    float mx = -INFINITY;
    int mi = -1;
    for (int base = 0; base < V; base += kST * kU) {
        float xv[kU];
        int kv[kU];
#pragma unroll
        for (int u = 0; u < kU; u++) {
            const int i = base + u * kST + t;
            xv[u] = i < V ? p.logits[i] : 0.f;
            kv[u] = (pen && i < V) ? p.counts[i] : 0;
        }
#pragma unroll
        for (int u = 0; u < kU; u++) {
            const int i = base + u * kST + t;
            if (i >= V) break;
            float x = xv[u];
            for (int j = 0; j < kv[u]; j++) x = x >= 0.f ? __fdiv_rn(x, p.penalty) : __fmul_rn(x, p.penalty);
            if (greedy) {
                if (mi < 0 || x > mx || (x == mx && i > mi)) {
                    mx = x;
                    mi = i;
                }
            } else {
                x = __fdiv_rn(x, p.temperature);
                p.scratch[i] = x;
                mx = fmaxf(mx, x);
            }
        }
    }
    if (greedy) {
        for (int o = 16; o > 0; o >>= 1) {
            const float v2 = __shfl_xor_sync(0xffffffffu, mx, o);
            const int i2 = __shfl_xor_sync(0xffffffffu, mi, o);
            if (i2 >= 0 && (mi < 0 || v2 > mx || (v2 == mx && i2 > mi))) {
                mx = v2;
                mi = i2;
            }
        }
        if (lane == 0) {
            redf[warp] = mx;
            redi[warp] = mi;
        }
        __syncthreads();
        if (warp == 0) {
            mx = redf[lane];
            mi = redi[lane];
            for (int o = 16; o > 0; o >>= 1) {
                const float v2 = __shfl_xor_sync(0xffffffffu, mx, o);
                const int i2 = __shfl_xor_sync(0xffffffffu, mi, o);
                if (i2 >= 0 && (mi < 0 || v2 > mx || (v2 == mx && i2 > mi))) {
                    mx = v2;
                    mi = i2;
                }
            }
            if (lane == 0) sh_i[0] = mi < 0 ? 0 : mi;
        }
        __syncthreads();
        tok = sh_i[0];
    } else {
        mx = block_max(mx, redf);
        // 3-4: numerators, their fixed-point total and, for a nucleus, the first radix level
        // (top 10 bits of e)
        const bool nucleus = p.top_p > 0.f && p.top_p < 1.f;
        unsigned long long* hw = hist + (warp % kHC) * 1024;
        for (int b = t; b < kHC * 1024; b += kST) hist[b] = 0;
        __syncthreads();
        unsigned long long s = 0;
        for (int base = 0; base < V; base += kST * kU) {
            float xv[kU];
#pragma unroll
            for (int u = 0; u < kU; u++) {
                const int i = base + u * kST + t;
                xv[u] = i < V ? p.scratch[i] : 0.f;
            }
#pragma unroll
            for (int u = 0; u < kU; u++) {
                const int i = base + u * kST + t;
                if (i >= V) break;
                const float e = expf(xv[u] - mx);
                p.scratch[i] = e;
                const unsigned long long m = mass(e);
                s += m;
                if (m && nucleus) atomicAdd(&hw[__float_as_uint(e) >> 20], m);
            }
        }
        const unsigned long long total = block_sum_u64(s, redu);
        unsigned int cut = 0;  // keep every e whose bit pattern is >= cut
        if (nucleus) {
            // keep iff the strictly larger mass G < top_p * total; for integer G that is
            // G < ceil(top_p * total) (>= 1, so the largest token is always kept)
            const unsigned long long target = (unsigned long long)ceil((double)p.top_p * (double)total);
            unsigned long long above = 0;
            unsigned int prefix = 0;
            bool whole = false;
            for (int level = 0; level < 3; level++) {
                if (level > 0) {
                    __syncthreads();
                    for (int b = t; b < kHC * 1024; b += kST) hist[b] = 0;
                    __syncthreads();
                    const int shp = 30 - 10 * level, shb = 20 - 10 * level;
                    for (int base = 0; base < V; base += kST * kU) {
                        float ev[kU];
#pragma unroll
                        for (int u = 0; u < kU; u++) {
                            const int i = base + u * kST + t;
                            ev[u] = i < V ? p.scratch[i] : 0.f;
                        }
#pragma unroll
                        for (int u = 0; u < kU; u++) {
                            const unsigned int bits = __float_as_uint(ev[u]);
                            const unsigned long long m = mass(ev[u]);
                            if (m && (bits >> shp) == prefix) atomicAdd(&hw[(bits >> shb) & 1023u], m);
                        }
                    }
                }
                __syncthreads();
                if (warp == 0) {
                    unsigned long long a2 = 0;
                    const int b = find_bucket(hist, above, target, &a2);
                    if (lane == 0) {
                        sh_i[0] = b;
                        sh_u[0] = a2;
                    }
                }
                __syncthreads();
                const int b = sh_i[0];
                if (b >= 1024) {  // the target is not reached inside the prefix: keep all of it
                    whole = true;
                    break;
                }
                above = sh_u[0];
                prefix = (prefix << 10) | (unsigned int)b;
            }
            // the exact value whose strictly larger masses sum below the target (or the lower
            // edge of the prefix when the target lies beyond it)
            cut = whole ? 0u : prefix;
            if (whole && prefix) {
                // prefix of `level` 10-bit groups: its smallest pattern
                int lv = 0;
                for (unsigned int q = prefix; q; q >>= 10) lv++;
                cut = prefix << (30 - 10 * lv);
            }
        }
        // 5: kept mass per thread over thread-contiguous index ranges (C indices each), an
        // exclusive scan of those in index order, then the one thread whose range holds the
        // draw walks it
        const int C = (V + kST - 1) / kST, c0 = min(V, t * C), c1 = min(V, c0 + C);
        unsigned long long ts = 0;
        for (int j0 = c0; j0 < c1; j0 += kU) {
            float ev[kU];
#pragma unroll
            for (int u = 0; u < kU; u++) ev[u] = j0 + u < c1 ? p.scratch[j0 + u] : 0.f;
#pragma unroll
            for (int u = 0; u < kU; u++)
                if (j0 + u < c1 && __float_as_uint(ev[u]) >= cut) ts += mass(ev[u]);
        }
        // block exclusive scan of ts (thread order = index order)
        unsigned long long incl = ts;
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned long long n = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += n;
        }
        __syncthreads();
        if (lane == 31) redu[warp] = incl;
        __syncthreads();
        if (warp == 0) {
            const unsigned long long wv = redu[lane];
            unsigned long long wi = wv;
            for (int o = 1; o < 32; o <<= 1) {
                const unsigned long long n = __shfl_up_sync(0xffffffffu, wi, o);
                if (lane >= o) wi += n;
            }
            redu[lane] = wi - wv;  // exclusive prefix of the warps
            if (lane == 31) {
                const unsigned long long kept = wi;
                const unsigned long long step = p.step ? (unsigned long long)*p.step : 0ull;
                sh_u[1] = __umul64hi(splitmix64(p.seed, step), kept);
                sh_u[2] = kept;
                sh_u[3] = total;
                sh_i[2] = (int)cut;
                sh_i[3] = -1;
            }
        }
        __syncthreads();
        {
            const unsigned long long r = sh_u[1];
            unsigned long long run = redu[warp] + incl - ts;  // kept mass before this thread's range
            if (ts && r >= run && r < run + ts) {
                for (int j = c0; j < c1; j++) {
                    const float e = p.scratch[j];
                    const unsigned long long m = __float_as_uint(e) >= cut ? mass(e) : 0ull;
                    if (m && run + m > r) {
                        sh_i[3] = j;
                        break;
                    }
                    run += m;
                }
            }
        }
        __syncthreads();
        tok = sh_i[3];
        if (tok < 0) tok = 0;
    }
    if (t == 0) {
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
            p.dbg[0] = greedy ? 0ull : (unsigned long long)(unsigned int)sh_i[2];
            p.dbg[1] = greedy ? 0ull : sh_u[2];
            p.dbg[2] = greedy ? 0ull : sh_u[3];
        }
    }
}

}  // namespace

cudaError_t launch_sample(const SampleParams& p, cudaStream_t st, bool pdl) {
    if (!p.logits || p.vocab <= 0 || !p.out_tok || !p.scratch) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(kST);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, sample_kernel, p);
}

}  // namespace tptc
