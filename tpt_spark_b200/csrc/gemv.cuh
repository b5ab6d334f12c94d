// gemv.cuh -- batch-1 dequant-fused GEMV (decode) for Q4_K / Q5_K / Q6_K / Q4_0 / Q5_0 / Q8_0 /
// F16 weights.
#pragma once

#include "common.cuh"

namespace tptc {

// Bytes per 256-element super-block in the device layout (all of it, GGUF size), the part
// before a tile's scale section, and its share of that section; super-blocks per chunk.
__host__ __device__ constexpr int sb_main_bytes(int type) {
    switch (type) {
    case TPTC_TYPE_Q2_K: return 80;
    case TPTC_TYPE_Q3_K: return 96;
    case TPTC_TYPE_Q4_K: return 144;
    case TPTC_TYPE_Q5_K: return 176;
    case TPTC_TYPE_Q6_K: return 208;
    case TPTC_TYPE_Q4_0: case TPTC_TYPE_Q4_1: return 128;
    case TPTC_TYPE_Q5_0: case TPTC_TYPE_Q5_1: return 160;
    case TPTC_TYPE_Q8_0: return 256;
    }
    return 512;
}
__host__ __device__ constexpr int sb_d_bytes(int type) {
    switch (type) {
    case TPTC_TYPE_Q6_K: return 2;
    case TPTC_TYPE_Q2_K: return 4;
    case TPTC_TYPE_Q3_K: return 14;
    case TPTC_TYPE_Q4_0: case TPTC_TYPE_Q5_0: case TPTC_TYPE_Q8_0: return 16;
    case TPTC_TYPE_Q4_1: case TPTC_TYPE_Q5_1: return 32;
    }
    return 0;
}
__host__ __device__ constexpr int sb_bytes(int type) { return sb_main_bytes(type) + sb_d_bytes(type); }
// The 32-element formats: eight blocks per super-block, activations quantised to Q8_0.
__host__ __device__ inline bool type_q80_family(int type) {
    return type == TPTC_TYPE_Q8_0 || type == TPTC_TYPE_Q4_0 || type == TPTC_TYPE_Q5_0 || type == TPTC_TYPE_Q4_1 ||
           type == TPTC_TYPE_Q5_1;
}
__host__ __device__ inline int chunk_sb(int type) { return type == TPTC_TYPE_F16 ? 8 : 16; }

constexpr int kTileRows = 8;

// Device layout of a weight matrix [N out x K in] (K a multiple of 256).
//
// Per-super-block encoding (256 elements):
//   Q2_K   80 B: qs[64] | scales[16], plus its f16 d and dmin in the scale section
//   Q3_K   96 B: hmask[32] | qs[64], plus its scales[12] and f16 d (14 B) in the scale section
//   Q4_K  144 B: the GGUF block unchanged (d | dmin | scales[12] | qs[128])
//   Q5_K  176 B: the GGUF block unchanged (d | dmin | scales[12] | qh[32] | qs[128])
//   Q6_K  208 B: ql | qh | scales, plus its f16 d in the tile's scale section
//   Q4_0  128 B: qs of eight 32-blocks (16 B each), plus their eight f16 d in the scale section
//   Q5_0  160 B: qs of eight 32-blocks, then their eight 4-byte qh words; d as Q4_0
//   Q4_1 / Q5_1: Q4_0's / Q5_0's main part, each block's f16 d and m in the scale section
//   Q8_0  256 B: qs of eight 32-blocks, plus their eight f16 d in the scale section
//   F16   512 B: 256 f16 values
// Tiling: rows are grouped by 8 (N padded to Npad, zero rows) and each row is cut into
// chunks of cbs super-blocks; tile (rg, c) = 8 rows x chunk c is one contiguous run of
// 8 * cb * sb_bytes (cb = cbs, or the remainder for the last chunk): the 8 rows' quant bytes
// in row order (cb * sb_main_bytes each), then the scale section (row-major [8][cb] entries
// of sb_d_bytes).  A decode GEMV stage is therefore a single 1-D bulk copy of 18-35 KB that
// carries everything its dot products read, the size the copy engine needs to reach full
// HBM bandwidth (small copies are bound by a fixed per-copy cost).  glu = 1 marks a fused
// gate/up matrix: tile rows 0-3 are gate rows 4t..4t+3 and tile rows 4-7 the same up rows,
// N counts gate + up rows.
struct DevMatrix {
    int type = 0;
    int N = 0, K = 0;  // logical rows (gate + up for glu) and columns
    int Npad = 0;      // N rounded up to a multiple of 8
    int cbs = 16;      // super-blocks per chunk
    int glu = 0;
    uint8_t* main = nullptr;
    int64_t main_row_bytes = 0;  // bytes per row (K / 256 * sb_bytes)
    int64_t bytes() const { return main_row_bytes * N; }
    int64_t main_bytes() const { return main_row_bytes * Npad; }
};

// Geometry of a matrix in the device layout (pointers left null).
inline DevMatrix dm_geometry(int type, int N, int K, int glu) {
    DevMatrix m;
    m.type = type;
    m.N = N;
    m.K = K;
    m.glu = glu;
    m.Npad = (N + kTileRows - 1) / kTileRows * kTileRows;
    m.cbs = chunk_sb(type);
    m.main_row_bytes = (int64_t)(K / 256) * sb_bytes(type);
    return m;
}

// Physical row (tile order) of logical row `row`; for a glu matrix rows [0, N/2) are gate
// rows and [N/2, N) up rows.
__host__ __device__ inline int dm_phys_row(const DevMatrix& m, int row) {
    if (!m.glu) return row;
    const int half = m.N / 2, up = row >= half ? 1 : 0, r = up ? row - half : row;
    return (r / 4) * 8 + (r % 4) + 4 * up;
}

// Start of the tile holding super-block `sb` of physical row `prow`, its chunk length, and
// the super-block's index inside the chunk.
__host__ __device__ inline const uint8_t* dm_tile(const DevMatrix& m, int prow, int sb, int& cb, int& j) {
    const int nsb = m.K / 256, c = sb / m.cbs;
    cb = (nsb - c * m.cbs) < m.cbs ? (nsb - c * m.cbs) : m.cbs;
    j = sb - c * m.cbs;
    return m.main + (int64_t)(prow / kTileRows) * kTileRows * m.main_row_bytes +
           (int64_t)c * kTileRows * m.cbs * sb_bytes(m.type);
}

// Quant bytes of super-block `sb` of physical row `prow`.
__host__ __device__ inline const uint8_t* dm_block(const DevMatrix& m, int prow, int sb) {
    int cb, j;
    const uint8_t* t = dm_tile(m, prow, sb, cb, j);
    const int sbm = sb_main_bytes(m.type);
    return t + (int64_t)((prow % kTileRows) * cb + j) * sbm;
}

// Scale-section entry of super-block `sb` of physical row `prow` (Q6_K: d; Q2_K: d, dmin;
// Q3_K: scales[12] then d; Q4_0 / Q5_0 / Q8_0: the eight blocks' d; Q4_1 / Q5_1: their (d, m)).
__host__ __device__ inline const uint16_t* dm_scales(const DevMatrix& m, int prow, int sb) {
    int cb, j;
    const uint8_t* t = dm_tile(m, prow, sb, cb, j);
    return reinterpret_cast<const uint16_t*>(t + (int64_t)kTileRows * cb * sb_main_bytes(m.type) +
                                             (int64_t)((prow % kTileRows) * cb + j) * sb_d_bytes(m.type));
}

enum GemvEpi : int {
    EPI_STORE = 0,  // out[row] = y
    EPI_RESID = 1,  // out[row] += y   (residual stream update)
    EPI_QKV = 2,    // q -> out, k -> kraw (RoPE applied by the attention kernel), v -> V cache at pos
    EPI_GLU = 3,    // fused gate|up matrix: out[logical row] (silu(gate)*up is formed by the consumer)
    EPI_DOTS = 4,   // integer block sums (test hook)
};

// Layout of a prepared GEMV activation (the GEMV's shared-memory region, and the global
// buffer it is bulk-copied from): byte offsets of each part, -1 when absent.
//   f32           [K] f32                    (F16 weights)
//   q8k           [K] int8 Q8_K quants       (Q4_K / Q5_K / Q6_K weights), lane-transposed per chunk
//                 (xt_offset) for the forward kernels, natural order for the DOTS test hook
//   q8k_d / _bs / _ps  per 256-block scale, 16-element sums [K/16], 32-element sums [K/32]
//   q80 / q80_d   [K] int8 Q8_0 quants, per 32-block scale (f16-rounded, f32) (Q4_0 / Q5_0 /
//                 Q8_0 weights)
struct ActLayout {
    int f32, q8k, q8k_d, q8k_bs, q8k_ps, q80, q80_d;
    int bytes;  // total, a multiple of 128
    int cbs;    // super-blocks per weight chunk (the transposition period)
};

// Byte offset of the 8 Q8_K quants of lane `lane` (elements 8*lane .. +7) of 256-block b in
// the lane-transposed layout: per chunk of cbs blocks, 16-byte vector v of half block h
// (= 2 * block-in-chunk + half) sits at (v * nh + h) * 16, nh = 2 * blocks in the chunk.
__host__ __device__ __forceinline__ int xt_offset(int b, int lane, int nsb, int cbs) {
    const int c = b / cbs, j = b - c * cbs, cbc = (nsb - c * cbs) < cbs ? (nsb - c * cbs) : cbs, nh = 2 * cbc;
    const int h = lane >> 4, v = (lane & 15) >> 1;
    return c * cbs * 256 + (v * nh + 2 * j + h) * 16 + (lane & 1) * 8;
}

constexpr int kGemvMaxSeg = 3;
constexpr int kGemvMaxStages = 16;

// Tensor-parallel reduction of the row-parallel projections over NVLink peer memory (tp.cpp).
// Every rank owns an inbox [2 slots][size][dim] of 64-bit words (f32 value | 32-bit epoch);
// inbox[r] is rank r's, mapped into this process.  A row-parallel GEMV (EPI_RESID with tp
// set) stores each partial row, tagged with the epoch of this use of the slot, into row
// block `rank` of slot `tp_slot` of every rank's inbox -- one 64-bit store, so a reader sees
// a value and its epoch together and needs no separate flag or fence.  The next activation
// kernel (tp_gather) reads every rank's block, waiting (bounded) on words whose epoch is not
// yet the current one, and forms x_out = x + sum over ranks in rank order (the same bits on
// every rank).  Epoch of use u of a step: step * uses_per_step + u + 1, with the step
// counter advanced by the embedding kernel that opens every step.  After the [2][size][dim]
// reduction slots each inbox holds [size][2] words for the vocab-parallel argmax (each
// rank's best logit and its index, both tagged with the epoch of use 2 * n_layers).  A wait
// gives up after wait_polls reads (TPTC_ERR_TIMEOUT): a rank that stops taking steps leaves
// the others with an error, not a hung GPU.
constexpr int kTpMaxRanks = 8;
struct TpLink {
    int rank, size, dim;
    int uses_per_step;  // 2 per layer + 1 (the argmax exchange)
    unsigned long long* inbox[kTpMaxRanks];
    const int* step;    // this rank's decode step counter
    uint32_t wait_polls;
};
__host__ __device__ inline size_t tp_inbox_words(int size, int dim) { return (size_t)2 * size * dim + (size_t)2 * size; }
__host__ __device__ inline size_t tp_argmax_offset(int size, int dim) { return (size_t)2 * size * dim; }

struct GemvSeg {
    DevMatrix m;
    int unit_begin;    // filled by gemv_prepare
    int out_off = 0;   // EPI_GLU / EPI_RESID: added to the output row (several gate|up segments into one buffer)
    int sel = -1;      // >= 0: mixture-of-experts weights, expert moe_sel[sel] of the stack m.main points at
};

struct GemvParams {
    GemvSeg seg[kGemvMaxSeg];
    int nseg;
    int K;
    const float* x;       // input activation [K] (f32)
    const float* norm_w;  // RMSNorm gain [K] or nullptr (no norm)
    int glu_in;           // 1: x holds [gate | up] (2K floats); the input is silu(gate) * up
    int glu_act;          // EPI_GLU: 0 silu(gate) * up, 1 GEGLU's tanh-form gelu(gate) * up
    float eps;
    float* out;
    // EPI_QKV
    void* vcache;  // this layer's V cache, layout [n_kv][max_seq][hd], fp16 or f32
    int kv_f32;    // 1: the cache holds f32 (candle's precision), 0: fp16
    float* kraw;   // key rows before RoPE (the attention kernel rotates and caches them)
    const int* pos;  // device scalar: position being written
    int hd;
    int max_seq;
    const float* bias[kGemvMaxSeg];  // optional per-segment row biases (qwen2 q / k / v), added in f32
    // mixture of experts.  Segments with sel >= 0 read expert moe_sel[sel] (device, written by
    // the routing kernel; clamped to [0, moe_nexp)) at m.main + expert * moe_stride; the
    // producer waits for the previous kernel before it reads the index.  EPI_RESID with moe_acc
    // set accumulates candle's weighted sum instead of adding to out: a = y * moe_w[moe_slot]
    // (weight 1 for moe_slot < 0, a shared expert), acc = moe_first ? a : acc + a, and with
    // moe_last out[row] = acc + out[row] (the residual add) instead of storing acc.
    const int* moe_sel;
    int64_t moe_stride;
    int moe_nexp;
    const float* moe_w;
    int moe_slot;
    int moe_first, moe_last;
    float* moe_acc;
    // EPI_DOTS
    int32_t* isum;
    int32_t* msum;
    // filled by gemv_prepare
    int units;        // total work units (8-row tile groups)
    int cbs;          // super-blocks per chunk (same for every segment)
    int nchunks;      // chunks per row
    int stages;       // ring depth
    int stage_bytes;  // bytes per stage (one full tile)
    int grid;         // CTAs (persistent: units are strided over them)
    ActLayout act;  // the activation region at the start of shared memory
    // Device buffer of act.bytes (16-byte aligned) receiving the prepared activation in the
    // shared-memory layout, bulk-copied by every CTA.  act_prepared = 0: gemv_launch first
    // runs the activation kernel on x; 1: the previous kernel already wrote it (for example
    // the attention kernel for the o projection) and x is not read.
    uint8_t* act_global;
    int act_prepared;
    int* err;
    // tensor parallelism over peer memory (TpLink): EPI_RESID scatters instead of adding;
    // the activation kernel gathers (tp_gather) into x_out; tp_use = 2 * layer + slot
    const TpLink* tp;
    int tp_slot;
    int tp_use;
    int tp_gather;
    float* x_out;
};

// A chain of GEMVs in one persistent launch (gemv.cu gemv_chain_kernel): phases separated
// by grid-wide arrival counters; each phase's activation is built by every CTA from its x
// (RMSNorm with norm_w when set, then quantisation), or bulk-copied from act_global when
// act_prepared.  After the last phase the last CTA to arrive optionally reduces the argmax of
// the last phase's rows (EPI_STORE, candle sample_argmax ties to the higher index) and
// resets the counters for the next launch.  Every CTA of the grid must be resident together:
// the grid is two CTAs per SM, which the shared-memory budget allows.
constexpr int kChainMaxPhases = 4;
struct ChainParams {
    GemvParams ph[kChainMaxPhases];
    int epi[kChainMaxPhases];  // EPI_STORE / RESID / QKV / GLU
    int nph;
    int* bar;  // [kChainMaxPhases] arrival counters, zero at launch (left zero on success)
    // argmax after the last phase when out_tok != nullptr (same outputs as launch_argmax)
    float* best_val;  // [grid] per-CTA partials
    int* best_idx;
    uint32_t* out_tok;
    uint32_t* next_tok;
    int* pos;
    uint32_t* history;
    int* err;
    // filled by chain_prepare
    int act_bytes, stages, stage_bytes, grid;
};

// Host helpers (gemv.cu).
void gemv_prepare(GemvParams& p, int sm_count = 148);  // work split, ring, activation layout
size_t gemv_smem(const GemvParams& p);
// Two launches: the activation kernel (norm + quantisation into p.act_global), then the GEMV.
cudaError_t gemv_launch(const GemvParams& p, int epi, cudaStream_t st, bool pdl);
// Upper bound of act_bytes for inputs of K elements (buffer sizing).
inline size_t gemv_act_bytes_max(int K) { return (size_t)K * 7 + 1024; }
cudaError_t gemv_init_device();  // per-device kernel attributes (call once per device)
// Phases already gemv_prepare'd: common ring geometry and grid (2 CTAs per SM).
void chain_prepare(ChainParams& c, int sm_count = 148);
size_t chain_smem(const ChainParams& c);
// Whether every CTA of the chain's grid can be resident at once (its barriers need that).
bool chain_fits(const ChainParams& c, int sm_count);
cudaError_t chain_launch(const ChainParams& c, cudaStream_t st, bool pdl);

}  // namespace tptc
