// Paired sparse prefill: one CTA serves two adjacent 128-query blocks of a head
// (rows A = 2p and B = 2p + 1 of the plan) from ONE stream of gathered K/V
// granules, the union of the two rows' samples (the math is that of
// prefill.cu: FlashInfer's fa3 batch prefill with the ABSipAttention logit
// shift, ab_attention/flashinfer_backend.py:30-58,164-242).
//
// Adjacent query blocks share most of their sampled granules (the certain,
// top-scored granules above all: the union of two blocks is ~1.26x one block's
// samples at the Wan shape), so fetching the union once per pair moves about two
// thirds of the bytes two separate CTAs would gather, and each shared tile feeds
// both blocks' products.
//
// Pair plan (pair_plan_kernel, one CTA per pair): the union as a list of
// entries (16-bit slot of A | 16-bit slot of B << 16; 0xFFFF = not sampled by
// that row; slots >= samples are text granules), laid out in tiles of 32
// granules (128 keys):
//   [shared granules | text granules | padding]  tiles both rows attend to,
//   then tiles holding only A's or only B's granules, alternating A, B, A, B
//   until one side runs out, then the rest of the other side.
// Beside each entry the plan stores the granule it names (a video granule id,
// kTextCode + text granule, kPadCode, or kBadCode for an out-of-range id), so
// the gather resolves a source row with one load.
// A row's weight for an entry is its own SIP weight, 0 for text and -inf for a
// granule it did not sample (and for padding), so each row's softmax is
// exactly its own sparse attention. A plan row with a repeated or
// out-of-range id is never merged: the pair then gets exclusive tiles only,
// which keeps the unpaired semantics (repeats count twice; a bad id reads
// zeros and records ABX_ERR_INVALID_ARGUMENT).
//
// Prefill (prefill_pair_kernel, one CTA per pair, 16 warps), 128-key tiles:
//   warps 0-3, 4-7  softmax groups A and B (thread = query row = TMEM lane of
//              that row's block); group g walks its own tiles of the stream.
//   warp  8    MMA issue (the converged warp, one elected lane issues):
//              S_g = Q_g K^T into the group's S/P columns, O_g += P_g V with P
//              read from TMEM; per group PV(k) then S(k + 1), groups interleaved,
//              so one group's PV and S run while the other group's softmax runs.
//              V(k) and K(k + 1) are waited for before P(k), so both products
//              follow the softmax's hand-over back to back.
//   warps 9-11 K gathers (and Q), warps 12-15 V gathers: one TMA box of 4 rows
//              x 64 columns per lane, 128-byte swizzled into the UMMA tile.
// A softmax thread takes its tile's 32 granule weights (warp shuffles) while S is
// being computed, reads its whole 128-column S row from TMEM in one go (four
// loads, one wait), takes the row max and the exponentials in registers and
// writes P back with four stores: two TMEM round trips per tile.
// TMEM: O_A [0,128), O_B [128,256), S/P of A [256,384), of B [384,512).
// Shared memory: Q_A, Q_B (64 KB), three K and two V stages of 32 KB.
// Every wait is bounded as in prefill.cu, and lets the hardware suspend the
// waiting warp (mbarrier try_wait without a time hint): each sub-partition holds
// one warp of each softmax group beside the MMA or gather warps, and a polling
// warp would take issue slots from the one that is computing.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "f32x2.cuh"
#include "ibcs.cuh"
#include "tcgen05.cuh"
#include "tma_host.cuh"

namespace abx {
namespace {

// ---- pair plan -----------------------------------------------------------------------------

constexpr int kPairGranules = 32;  // granules per tile (128 keys)
constexpr uint32_t kNoSlot = 0xFFFFu;
constexpr uint32_t kPadEntry = 0xFFFFFFFFu;
// Granule codes: [0, fine) video granule; kTextCode + t text granule t.
constexpr int32_t kTextCode = 0x40000000;
constexpr int32_t kBadCode = 0x7FFFFFFE;  // out-of-range plan id: reads zeros, reports
constexpr int32_t kPadCode = 0x7FFFFFFF;  // padding: reads zeros
constexpr int kPlanThreads = 512;
constexpr int kPlanWarps = kPlanThreads / 32;

struct PairPlanArgs {
    const int32_t* ids;   // [rows, samples]
    uint32_t* entries;    // [pairs, stride]
    int32_t* codes;       // [pairs, stride] granule of each entry
    int4* info;           // [pairs]: shared tiles, A tiles, B tiles, tail entry (-1: none)
    int64_t qb;           // query blocks per head
    int64_t stride;       // entries per pair
    int pairs_per_head;
    int samples;
    int fine_blocks;
    int text_granules;
    int text_tail;
};

// Exclusive prefix sum over the block; `total` receives the block's sum.
__device__ int block_exclusive_scan(int v, int* warp_sums, int& total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int w = lane < kPlanWarps ? warp_sums[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += y;
        }
        if (lane < kPlanWarps) warp_sums[lane] = w;
    }
    __syncthreads();
    const int before = warp ? warp_sums[warp - 1] : 0;
    total = warp_sums[kPlanWarps - 1];
    __syncthreads();
    return before + x - v;
}

// Stream position of the i-th exclusive entry of group g (A = 0, B = 1).
__device__ __forceinline__ int64_t exclusive_pos(int shared_tiles, int a_tiles, int b_tiles, int g, int i) {
    const int e = i / kPairGranules;
    const int m = min(a_tiles, b_tiles);
    const int tile = shared_tiles + (e < m ? 2 * e + g : m + e);
    return static_cast<int64_t>(tile) * kPairGranules + i % kPairGranules;
}

__global__ void __launch_bounds__(kPlanThreads) pair_plan_kernel(const PairPlanArgs a) {
    extern __shared__ __align__(16) uint8_t plan_smem[];
    const int64_t p = blockIdx.x;
    const int64_t head = p / a.pairs_per_head;
    const int64_t block_a = 2 * (p - head * a.pairs_per_head);
    const bool has_b = block_a + 1 < a.qb;
    const int64_t row_a = head * a.qb + block_a;
    const int32_t* ids_a = a.ids + row_a * a.samples;
    const int32_t* ids_b = ids_a + a.samples;
    const int n = a.samples;
    const int fine = a.fine_blocks;

    // B's slot of each granule (16-bit, kNoSlot = not sampled by B), bitmaps of the
    // granules seen in A and in B (repeated ids), and B's slots matched by A.
    const int seen_words = (fine + 31) / 32;
    const int map_words = (fine + 1) / 2;
    uint16_t* slot_of_b = reinterpret_cast<uint16_t*>(plan_smem);                  // [2 * map_words]
    uint32_t* seen_a = reinterpret_cast<uint32_t*>(plan_smem) + map_words;         // [seen_words]
    uint32_t* seen_b = seen_a + seen_words;                                         // [seen_words]
    uint8_t* used_b = reinterpret_cast<uint8_t*>(seen_b + seen_words);              // [samples]
    __shared__ int warp_sums[kPlanWarps];

    for (int i = threadIdx.x; i < map_words; i += kPlanThreads) reinterpret_cast<uint32_t*>(plan_smem)[i] = ~0u;
    for (int i = threadIdx.x; i < 2 * seen_words; i += kPlanThreads) seen_a[i] = 0;
    for (int i = threadIdx.x; i < n; i += kPlanThreads) used_b[i] = 0;
    __syncthreads();
    bool bad = false;
    if (has_b) {
        for (int s = threadIdx.x; s < n; s += kPlanThreads) {
            const int id = __ldg(ids_b + s);
            if (id < 0 || id >= fine) {
                bad = true;
                continue;
            }
            const uint32_t bit = 1u << (id & 31);
            if (atomicOr(seen_b + (id >> 5), bit) & bit) bad = true;  // repeated id in B
            slot_of_b[id] = static_cast<uint16_t>(s);
        }
    }
    __syncthreads();
    for (int s = threadIdx.x; s < n; s += kPlanThreads) {
        const int id = __ldg(ids_a + s);
        if (id < 0 || id >= fine) {
            bad = true;
            continue;
        }
        const uint32_t bit = 1u << (id & 31);
        if (atomicOr(seen_a + (id >> 5), bit) & bit) bad = true;  // repeated id in A
        const uint32_t sb = slot_of_b[id];
        if (sb != kNoSlot) used_b[sb] = 1;
    }
    bad = __syncthreads_or(bad);

    // Shared entries of A (in A's slot order) and B-only entries (in B's order).
    const int chunk = (n + kPlanThreads - 1) / kPlanThreads;
    const int s0 = min(n, static_cast<int>(threadIdx.x) * chunk);
    const int s1 = min(n, s0 + chunk);
    int my_shared = 0, my_b_only = 0;
    for (int s = s0; s < s1; ++s) {
        if (!bad && has_b && slot_of_b[__ldg(ids_a + s)] != kNoSlot) ++my_shared;
        if (has_b && (bad || !used_b[s])) ++my_b_only;
    }
    int n_shared, n_b_only;
    const int shared_before = block_exclusive_scan(my_shared, warp_sums, n_shared);
    const int b_only_before = block_exclusive_scan(my_b_only, warp_sums, n_b_only);

    const int nt = a.text_granules;
    const int shared_len = has_b ? n_shared + nt : 0;
    const int n_a_only = n - n_shared + (has_b ? 0 : nt);
    const int shared_tiles = (shared_len + kPairGranules - 1) / kPairGranules;
    const int a_tiles = (n_a_only + kPairGranules - 1) / kPairGranules;
    const int b_tiles = (n_b_only + kPairGranules - 1) / kPairGranules;
    uint32_t* out = a.entries + p * a.stride;
    int32_t* code = a.codes + p * a.stride;
    auto video_code = [&](int id) { return (id >= 0 && id < fine) ? id : kBadCode; };

    int shared_idx = shared_before;
    int b_idx = b_only_before;
    for (int s = s0; s < s1; ++s) {
        const uint32_t sb_raw = (!bad && has_b) ? slot_of_b[__ldg(ids_a + s)] : kNoSlot;
        const int sb = sb_raw == kNoSlot ? -1 : static_cast<int>(sb_raw);
        const int id_a = video_code(__ldg(ids_a + s));
        if (sb >= 0) {
            code[shared_idx] = id_a;
            out[shared_idx++] = static_cast<uint32_t>(s) | (static_cast<uint32_t>(sb) << 16);
        } else {
            const int i = s - shared_idx;  // A-only entries before slot s
            const int64_t e = exclusive_pos(shared_tiles, a_tiles, b_tiles, 0, i);
            code[e] = id_a;
            out[e] = static_cast<uint32_t>(s) | (kNoSlot << 16);
        }
        if (has_b && (bad || !used_b[s])) {
            const int64_t e = exclusive_pos(shared_tiles, a_tiles, b_tiles, 1, b_idx++);
            code[e] = video_code(__ldg(ids_b + s));
            out[e] = kNoSlot | (static_cast<uint32_t>(s) << 16);
        }
    }
    // Text granules: shared by both rows (or A-only when the pair has no B), then padding.
    for (int t = threadIdx.x; t < nt; t += kPlanThreads) {
        const uint32_t slot = static_cast<uint32_t>(n + t);
        const int64_t e = has_b ? n_shared + t : exclusive_pos(shared_tiles, a_tiles, b_tiles, 0, n + t);
        out[e] = has_b ? slot | (slot << 16) : slot | (kNoSlot << 16);
        code[e] = kTextCode + t;
    }
    for (int i = shared_len + threadIdx.x; i < shared_tiles * kPairGranules; i += kPlanThreads) {
        out[i] = kPadEntry;
        code[i] = kPadCode;
    }
    for (int i = n_a_only + threadIdx.x; i < a_tiles * kPairGranules; i += kPlanThreads) {
        const int64_t e = exclusive_pos(shared_tiles, a_tiles, b_tiles, 0, i);
        out[e] = kPadEntry;
        code[e] = kPadCode;
    }
    for (int i = n_b_only + threadIdx.x; i < b_tiles * kPairGranules; i += kPlanThreads) {
        const int64_t e = exclusive_pos(shared_tiles, a_tiles, b_tiles, 1, i);
        out[e] = kPadEntry;
        code[e] = kPadCode;
    }
    if (threadIdx.x == 0) {
        int tail = -1;
        if (a.text_tail != 0 && nt > 0)
            tail = has_b ? n_shared + nt - 1
                         : static_cast<int>(exclusive_pos(shared_tiles, a_tiles, b_tiles, 0, n + nt - 1));
        a.info[p] = make_int4(shared_tiles, a_tiles, b_tiles, tail);
    }
}

// ---- paired prefill ------------------------------------------------------------------------

constexpr int kTileKeys = 128;
constexpr int kTileGranules = kTileKeys / kKv4;
static_assert(kTileGranules == kPairGranules, "pair plan tiles and prefill tiles must match");
constexpr int kKStages = 3;
constexpr int kVStages = 2;
constexpr uint32_t kSlabBytes = kTileKeys * 128;   // 128 rows x 64 bf16
constexpr uint32_t kTileBytes = 2 * kSlabBytes;    // one 128 x 128 bf16 operand tile
constexpr uint32_t kQSlabBytes = 128 * 128;        // 128 rows x 64 bf16
constexpr uint32_t kQBytes = 2 * kQSlabBytes;
constexpr int kGroups = 2;
constexpr int kMmaWarp = 8;
constexpr int kKGatherWarps = 3;
constexpr int kVGatherWarps = 4;
constexpr int kBoxesPerTile = 2 * kTileGranules;
constexpr uint32_t kBoxBytes = kKv4 * 128;
constexpr int kKLoadWarp = kMmaWarp + 1;
constexpr int kVLoadWarp = kKLoadWarp + kKGatherWarps;
constexpr int kThreads = (kVLoadWarp + kVGatherWarps) * 32;
constexpr int kChunk = 16;
constexpr int kChunks = kTileKeys / kChunk;
constexpr int kLaunchRegs = 128;
constexpr int kSoftmaxRegs = 200;  // a whole 128-column S row in registers
constexpr int kProducerRegs = 56;
static_assert(kThreads == 512, "register split below assumes 16 warps");
static_assert(kThreads * kLaunchRegs <= 65536, "launch register allocation exceeds the SM");
static_assert(8 * 32 * kSoftmaxRegs + (kThreads - 8 * 32) * kProducerRegs <= kThreads * kLaunchRegs,
              "setmaxnreg split exceeds the launch allocation (the increase would never complete)");

constexpr uint32_t kTmemColumns = 512;
__device__ __forceinline__ constexpr uint32_t col_o(int g) { return 128u * static_cast<uint32_t>(g); }
__device__ __forceinline__ constexpr uint32_t col_s(int g) { return 256u + 128u * static_cast<uint32_t>(g); }

constexpr uint32_t kOffQ = 0;  // Q_A, Q_B
constexpr uint32_t kOffK = kOffQ + 2 * kQBytes;
constexpr uint32_t kOffV = kOffK + kKStages * kTileBytes;
constexpr uint32_t kOffBar = kOffV + kVStages * kTileBytes;
constexpr int kBarQFull = 0;
constexpr int kBarKFull = 1;
constexpr int kBarKEmpty = kBarKFull + kKStages;
constexpr int kBarVFull = kBarKEmpty + kKStages;
constexpr int kBarVEmpty = kBarVFull + kVStages;
constexpr int kBarSFull = kBarVEmpty + kVStages;  // [group]
constexpr int kBarPFull = kBarSFull + 2;          // [group]
constexpr int kBarOFinal = kBarPFull + 2;         // [group]: the group's last PV done
constexpr int kBarDrain = kBarOFinal + 2;
constexpr int kNumBars = kBarDrain + 1;
constexpr uint32_t kOffTmemSlot = kOffBar + kNumBars * 8;
constexpr uint32_t kOffAbort = kOffTmemSlot + 4;
constexpr uint32_t kSmemUsed = kOffAbort + 4;
constexpr uint32_t kSmemBytes = kSmemUsed + 1024;
static_assert(kSmemBytes <= 227 * 1024, "shared memory exceeds the per-block limit");

constexpr uint64_t kWaitLimit = 400ull * 1000 * 1000;
constexpr float kRescaleThreshold = 32.0f;  // log2 units, as in prefill.cu

constexpr uint32_t kIdescS = tc::idesc_bf16_f32(128, kTileKeys, 0, 0);  // Q, K both K-major
constexpr uint32_t kIdescPV = tc::idesc_bf16_f32(128, 128, 0, 1);       // P K-major (TMEM), V MN-major

struct PairArgs {
    const int32_t* ids;
    const float* logw;
    const uint32_t* entries;
    const int32_t* codes;
    const int4* info;
    bf16* o;
    float* lse;
    int64_t seq;          // tokens per head (q, k, v, o, lse)
    int64_t qb;
    int64_t stride;       // entries per pair
    int64_t text_tokens;
    int64_t kv_rows;      // bh * seq: an index >= this reads zeros
    int pairs_per_head;
    int samples;
    int fine_blocks;
    int text_tail;
    float kappa;
    int* error;
    // Scatter form (num_outs > 0): every output row goes to each of `outs`, buffers
    // of the whole layer's [heads, seq, 128] output (on this GPU or on peers,
    // through their mapped addresses), at head out_head_base + head; `o` is unused.
    bf16* outs[kMaxScatterOutputs];
    int num_outs;
    int64_t out_head_base;
};

struct PairMaps {
    CUtensorMap q;        // box 64 x 128 rows
    CUtensorMap kv[2][2];  // [K, V][head tokens, text tokens], box 64 x 4 rows
};

// Stream tile of the k-th tile of group g.
__device__ __forceinline__ int stream_tile(const int4& inf, int g, int k) {
    if (k < inf.x) return k;
    const int e = k - inf.x;
    const int m = min(inf.y, inf.z);
    return inf.x + (e < m ? 2 * e + g : m + e);
}

// Source row of a granule code in the K/V tensor maps (text = the text maps).
// Row indices fit 32 bits: the maps' row coordinates are 32-bit.
struct RowBases {
    int32_t video;  // head * seq
    int32_t text;   // head * text_tokens
    int32_t none;   // bh * seq: reads zeros
};

__device__ __forceinline__ int32_t code_row(const PairArgs& a, const RowBases& rb, int32_t code, bool& text) {
    text = false;
    if (code < kTextCode) {
        if (code < 0 || code >= a.fine_blocks) {  // never read outside the head
            raise_device_error(a.error, ABX_ERR_INVALID_ARGUMENT);
            return rb.none;
        }
        return rb.video + code * kKv4;
    }
    if (code == kPadCode) return rb.none;
    if (code == kBadCode) {
        raise_device_error(a.error, ABX_ERR_INVALID_ARGUMENT);
        return rb.none;
    }
    text = true;
    return rb.text + (code - kTextCode) * kKv4;
}

// The largest of three floats in one instruction (sm_100 `max.f32` with three inputs).
__device__ __forceinline__ float max3f(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// Logit shift of an entry for group g: its SIP weight, 0 for text, -inf when
// the group's row did not sample it.
__device__ __forceinline__ float entry_weight(const PairArgs& a, int64_t row_g, int g, uint32_t entry) {
    const uint32_t slot = g ? entry >> 16 : entry & kNoSlot;
    if (slot == kNoSlot) return -INFINITY;
    if (slot >= static_cast<uint32_t>(a.samples)) return 0.f;
    return a.logw ? __ldg(a.logw + row_g * a.samples + slot) : 0.f;
}

// Scores of the keys of granule `local` of the tile past the last text token
// (its first `tail` keys are valid) -> -inf in TMEM. Warp-collective.
__device__ __forceinline__ void mask_tail(uint32_t s_col, int local, int tail) {
    const uint32_t col = s_col + kChunk * (local / (kChunk / kKv4));
    const int first = (local % (kChunk / kKv4)) * kKv4 + tail;
    uint32_t chunk[kChunk];
    tc::tmem_ld16(col, chunk);
    tc::tmem_wait_ld();
    tc::tmem_reg_fence(chunk);
#pragma unroll
    for (int e = 0; e < kChunk; ++e)
        if (e >= first) chunk[e] = 0xff800000u;
    tc::tmem_st16(col, chunk);
    tc::tmem_wait_st();
}

__global__ void __launch_bounds__(kThreads, 1) prefill_pair_kernel(const PairArgs args,
                                                                   const __grid_constant__ PairMaps maps) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_base = smem_addr(smem_raw);
    const uint32_t base = (raw_base + 1023u) & ~1023u;
    uint8_t* gbase = smem_raw + (base - raw_base);
    auto bar = [&](int i) { return base + kOffBar + 8u * i; };
    volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + kOffAbort);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + kOffTmemSlot);

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int64_t p = blockIdx.x;
    const int64_t head = p / args.pairs_per_head;
    const int64_t block_a = 2 * (p - head * args.pairs_per_head);
    const bool has_b = block_a + 1 < args.qb;
    const int64_t row_a = head * args.qb + block_a;
    int4 inf = __ldg(args.info + p);
    if (inf.x < 0 || inf.y < 0 || inf.z < 0 ||
        static_cast<int64_t>(inf.x + inf.y + inf.z) * kTileGranules > args.stride || (!has_b && (inf.x | inf.z))) {
        // never read past the pair's entries
        if (threadIdx.x == 0) raise_device_error(args.error, ABX_ERR_INVALID_ARGUMENT);
        inf = make_int4(0, 0, 0, -1);
    }
    auto tiles_of = [&](int g) { return inf.x + (g ? inf.z : inf.y); };
    const int stream_tiles = inf.x + inf.y + inf.z;
    const uint32_t* entries = args.entries + p * args.stride;

    if (tid == 0) {
        *abort_flag = 0;
        tc::mbar_init(bar(kBarQFull), 1);
        for (int st = 0; st < kKStages; ++st) {
            tc::mbar_init(bar(kBarKFull + st), kKGatherWarps);
            tc::mbar_init(bar(kBarKEmpty + st), 1);
        }
        for (int st = 0; st < kVStages; ++st) {
            tc::mbar_init(bar(kBarVFull + st), kVGatherWarps);
            tc::mbar_init(bar(kBarVEmpty + st), 1);
        }
        for (int g = 0; g < kGroups; ++g) {
            tc::mbar_init(bar(kBarSFull + g), 1);
            tc::mbar_init(bar(kBarPFull + g), 128);
            tc::mbar_init(bar(kBarOFinal + g), 1);
        }
        tc::mbar_init(bar(kBarDrain), 1);
        tc::mbar_init_fence();
    }
    if (warp == kMmaWarp) {
        tc::tmem_alloc(smem_addr(tmem_slot), kTmemColumns);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    // Register split by warpgroup: each warpgroup executes one setmaxnreg, and each
    // role's code sits under its own (no merge in between, so the compiler gives
    // the softmax code the raised count).
    if (warp >= kMmaWarp) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(kProducerRegs));
    if (warp >= kKLoadWarp) {
        // ---- producers: one TMA box per lane per operand tile, stream order -----------------
        const bool is_k = warp < kVLoadWarp;
        const int part = warp - (is_k ? kKLoadWarp : kVLoadWarp);
        const int nwarps = is_k ? kKGatherWarps : kVGatherWarps;
        const int box = part + nwarps * lane;
        const bool has_box = box < kBoxesPerTile;
        const int my_granule = has_box ? box >> 1 : 0;
        const int my_slab = box & 1;
        const int warp_boxes = (kBoxesPerTile - part + nwarps - 1) / nwarps;
        if (warp == kKLoadWarp && lane == 0) {
            // Q of both blocks: four 128-row x 64-column boxes (rows past a block are never stored).
            tc::mbar_arrive_expect_tx(bar(kBarQFull), 2 * kQBytes);
            const int32_t qy = static_cast<int32_t>(head * args.seq + block_a * kQueryBlock);
            for (int g = 0; g < kGroups; ++g) {
                tc::tma_load_2d(base + kOffQ + g * kQBytes, &maps.q, 0, qy + g * kQueryBlock, bar(kBarQFull));
                tc::tma_load_2d(base + kOffQ + g * kQBytes + kQSlabBytes, &maps.q, 64, qy + g * kQueryBlock,
                                bar(kBarQFull));
            }
        }
        const int op = is_k ? 0 : 1;
        const int stages = is_k ? kKStages : kVStages;
        const uint32_t ring = base + (is_k ? kOffK : kOffV);
        const int bar_full = is_k ? kBarKFull : kBarVFull;
        const int bar_empty = is_k ? kBarKEmpty : kBarVEmpty;
        int issued = 0;
        // Granule codes are loaded two tiles ahead.
        const RowBases rb{static_cast<int32_t>(head * args.seq), static_cast<int32_t>(head * args.text_tokens),
                          static_cast<int32_t>(args.kv_rows)};
        const int32_t* codes = args.codes + p * args.stride + my_granule;
        int32_t code_cur = stream_tiles > 0 ? __ldg(codes) : kPadCode;
        int32_t code_next = stream_tiles > 1 ? __ldg(codes + kTileGranules) : kPadCode;
        for (int j = 0; j < stream_tiles; ++j) {
            const int st = j % stages;
            const int use = j / stages;
            bool text;
            const int32_t y = code_row(args, rb, code_cur, text);
            code_cur = code_next;
            if (j + 2 < stream_tiles) code_next = __ldg(codes + (j + 2) * kTileGranules);
            const bool free_ok =
                use == 0 || tc::mbar_wait_suspend(bar(bar_empty + st), (use - 1) & 1, abort_flag, kWaitLimit);
            if (!__all_sync(0xffffffffu, free_ok)) break;
            issued = j + 1;
            if (lane == 0) tc::mbar_arrive_expect_tx(bar(bar_full + st), warp_boxes * kBoxBytes);
            __syncwarp();
            const uint32_t dst = ring + st * kTileBytes + my_slab * kSlabBytes + my_granule * kBoxBytes;
            if (has_box)
                tc::tma_load_2d(dst, &maps.kv[op][text], 64 * my_slab, y, bar(bar_full + st));
        }
        if (lane == 0) {
            for (int st = 0; st < stages && st < issued; ++st) {
                const int last_use = (issued - 1 - st) / stages;
                tc::mbar_wait_suspend(bar(bar_full + st), last_use & 1, abort_flag, kWaitLimit,
                                      /*honor_abort=*/false);
            }
            if (warp == kKLoadWarp)
                tc::mbar_wait_suspend(bar(kBarQFull), 0, abort_flag, kWaitLimit, /*honor_abort=*/false);
        }
        __syncwarp();
    } else if (warp == kMmaWarp) {
        // ---- MMA issue: per group PV(k) then S(k + 1); A's, then B's; stream order -------------
        // The whole warp runs this loop (warp-uniform operands); one elected lane issues.
        {
            bool ok = tc::mbar_wait_warp_suspend(bar(kBarQFull), 0, abort_flag, kWaitLimit);
            // A shared tile is read by A, then B; its stages are released after B's MMA.
            auto last_reader = [&](int j, int g) { return j >= inf.x || g == 1 || !has_b; };
            auto k_ready = [&](int j) {
                return tc::mbar_wait_warp_suspend(bar(kBarKFull + j % kKStages), (j / kKStages) & 1, abort_flag,
                                                  kWaitLimit);
            };
            // S_g = Q_g K^T of stream tile j into the group's S/P columns (its K stage resident).
            auto issue_s = [&](int g, int j) {
                const int st = j % kKStages;
                const uint64_t adesc0 = tc::smem_desc(base + kOffQ + g * kQBytes, 16, 1024, tc::kSwizzle128B);
                const uint64_t bdesc0 = tc::smem_desc(base + kOffK + st * kTileBytes, 16, 1024, tc::kSwizzle128B);
#pragma unroll
                for (int s = 0; s < 8; ++s) {
                    // 16 dims per step inside a 64-dim slab: advance the start by 32 bytes
                    // (the descriptor's start field counts 16-byte units).
                    const uint32_t off = ((s >> 2) * kSlabBytes + (s & 3) * 32) >> 4;
                    tc::mma_ss_elect(tmem + col_s(g), adesc0 + off, bdesc0 + off, kIdescS, s > 0 ? 1u : 0u);
                }
                tc::mma_commit_elect(bar(kBarSFull + g));
                if (last_reader(j, g)) tc::mma_commit_elect(bar(kBarKEmpty + st));
            };
            // Step k of group g: PV(k), then S(k + 1). V(k) and K(k + 1) are waited for
            // before P(k), so once the softmax hands over P both go out back to back.
            auto step = [&](int g, int k) -> bool {
                const int j = stream_tile(inf, g, k);
                const int st = j % kVStages;
                const bool next = k + 1 < tiles_of(g);
                const int jn = next ? stream_tile(inf, g, k + 1) : 0;
                if (!tc::mbar_wait_warp_suspend(bar(kBarVFull + st), (j / kVStages) & 1, abort_flag, kWaitLimit))
                    return false;
                if (next && !k_ready(jn)) return false;
                if (!tc::mbar_wait_warp_suspend(bar(kBarPFull + g), k & 1, abort_flag, kWaitLimit)) return false;
                tc::fence_after_sync();
                const uint64_t bdesc0 =
                    tc::smem_desc(base + kOffV + st * kTileBytes, kSlabBytes, 1024, tc::kSwizzle128B);
#pragma unroll
                for (int s = 0; s < kTileKeys / 16; ++s) {
                    // 16 keys per step: P columns [8s, 8s+8); V rows [16s, 16s+16) (MN-major,
                    // leading offset = the second 64-dim slab, stride offset = 8-row atom).
                    tc::mma_ts_elect(tmem + col_o(g), tmem + col_s(g) + 8 * s, bdesc0 + ((s * 16 * 128) >> 4),
                                     kIdescPV, (k > 0 || s > 0) ? 1u : 0u);
                }
                if (last_reader(j, g)) tc::mma_commit_elect(bar(kBarVEmpty + st));
                if (k + 1 == tiles_of(g)) tc::mma_commit_elect(bar(kBarOFinal + g));
                // S(k + 1) overwrites the group's S/P columns: it follows PV(k) in the pipe.
                if (next) issue_s(g, jn);
                return true;
            };
            for (int g = 0; ok && g < kGroups; ++g) {
                if (tiles_of(g) == 0) continue;
                const int j0 = stream_tile(inf, g, 0);
                if (!k_ready(j0)) {
                    ok = false;
                    break;
                }
                tc::fence_after_sync();
                issue_s(g, j0);
            }
            const int steps = max(tiles_of(0), tiles_of(1));
            for (int k = 0; ok && k < steps; ++k) {
                for (int g = 0; ok && g < kGroups; ++g) {
                    if (k >= tiles_of(g)) continue;
                    if (!step(g, k)) ok = false;
                }
            }
            tc::mma_commit_elect(bar(kBarDrain));
            if (lane == 0) tc::mbar_wait_suspend(bar(kBarDrain), 0, abort_flag, kWaitLimit, /*honor_abort=*/false);
        }
        __syncwarp();
    }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;\n" ::"n"(kSoftmaxRegs));
        // ---- softmax group g over its own tiles (thread = query row = TMEM lane) ----------------
        const int g = warp >> 2;
        const int r = tid & 127;
        const int64_t row_g = row_a + g;
        const bool exists = g == 0 || has_b;
        const int tiles = exists ? tiles_of(g) : 0;
        const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
        const uint32_t o_col = lane_base + col_o(g);
        float m_used = -INFINITY;
        float l_sum = 0.f;
        bool ok = true;
        // Lane j holds the weight of granule j of the current tile; the entry two
        // tiles ahead and the weight one tile ahead are in flight.
        const int wl = lane & (kTileGranules - 1);
        uint32_t entry_next = kPadEntry;
        float w_next = -INFINITY;
        if (tiles > 0) w_next = entry_weight(args, row_g, g, __ldg(entries + stream_tile(inf, g, 0) * kTileGranules + wl));
        if (tiles > 1) entry_next = __ldg(entries + stream_tile(inf, g, 1) * kTileGranules + wl);
        for (int k = 0; k < tiles; ++k) {
            const float w_lane = w_next;
            if (k + 1 < tiles) w_next = entry_weight(args, row_g, g, entry_next);
            if (k + 2 < tiles) entry_next = __ldg(entries + stream_tile(inf, g, k + 2) * kTileGranules + wl);
            // The tile's 32 granule weights in every lane, taken while S is still being computed.
            float wv[kTileGranules];
#pragma unroll
            for (int gi = 0; gi < kTileGranules; ++gi) {
                wv[gi] = __shfl_sync(0xffffffffu, w_lane, gi);
                asm volatile("" : "+f"(wv[gi]));
            }
            if (!tc::mbar_wait_warp_suspend(bar(kBarSFull + g), k & 1, abort_flag, kWaitLimit)) {
                ok = false;
                break;
            }
            tc::fence_after_sync();
            const uint32_t s_col = lane_base + col_s(g);
            const int j = stream_tile(inf, g, k);
            if (inf.w >= j * kTileGranules && inf.w < (j + 1) * kTileGranules)
                mask_tail(s_col, inf.w - j * kTileGranules, args.text_tail);
            // The whole S row: four 32-column loads, one wait.
            uint32_t r0[32], r1[32], r2[32], r3[32];
            // column i of the row (i is a compile-time constant in the unrolled loops)
            auto col = [&](int i) -> uint32_t {
                return i < 32 ? r0[i & 31] : i < 64 ? r1[i & 31] : i < 96 ? r2[i & 31] : r3[i & 31];
            };
            {
                tc::tmem_ld32(s_col, r0);
                tc::tmem_ld32(s_col + 32, r1);
                tc::tmem_ld32(s_col + 64, r2);
                tc::tmem_ld32(s_col + 96, r3);
                tc::tmem_wait_ld();
                tc::tmem_reg_fence(r0);
                tc::tmem_reg_fence(r1);
                tc::tmem_reg_fence(r2);
                tc::tmem_reg_fence(r3);
            }
            // Row max of x = s * kappa + w (per granule: fma(max s, kappa, w)); the
            // granule weights stay in registers for the exponentials.
            float part_max[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
            for (int gi = 0; gi < kTileGranules; ++gi) {
                const float w = wv[gi];
                const float smax = max3f(__uint_as_float(col(4 * gi)), __uint_as_float(col(4 * gi + 1)),
                                         fmaxf(__uint_as_float(col(4 * gi + 2)), __uint_as_float(col(4 * gi + 3))));
                part_max[gi & 3] = fmaxf(part_max[gi & 3], fmaf(smax, args.kappa, w));
            }
            const float tile_max = fmaxf(fmaxf(part_max[0], part_max[1]), fmaxf(part_max[2], part_max[3]));
            // Lazy rescale, decided per warp. O_g holds the PV of the group's earlier
            // tiles, all complete: S(k) was issued after PV(k - 1).
            const bool grow = tile_max > m_used + kRescaleThreshold;
            if (__any_sync(0xffffffffu, grow)) {
                const float m_new = grow ? tile_max : m_used;
                const float scale = grow ? exp2f(m_used - m_new) : 1.0f;
                l_sum *= scale;
                if (k > 0) {
#pragma unroll 1
                    for (int c = 0; c < 128 / kChunk; ++c) {
                        uint32_t o[kChunk];
                        tc::tmem_ld16(o_col + kChunk * c, o);
                        tc::tmem_wait_ld();
                        tc::tmem_reg_fence(o);
#pragma unroll
                        for (int e = 0; e < kChunk; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * scale);
                        tc::tmem_st16(o_col + kChunk * c, o);
                    }
                }
                m_used = m_new;
            }
            // P = 2^(s * kappa + (w - m)) as bf16 pairs into S columns [0, 64): four 16-column stores.
            uint64_t part_sum[2] = {kZeros2, kZeros2};
            {
                const uint64_t kappa2 = pack2(args.kappa, args.kappa);
#pragma unroll
                for (int quarter = 0; quarter < 4; ++quarter) {
                    uint32_t packed[16];
#pragma unroll
                    for (int gi = 0; gi < kTileGranules / 4; ++gi) {
                        const int gg = quarter * (kTileGranules / 4) + gi;
                        const float wm = wv[gg] - m_used;
                        const uint64_t wm2 = pack2(wm, wm);
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const int e = 2 * gg + h;  // pair index in the row
                            const uint64_t s2 = (static_cast<uint64_t>(col(2 * e + 1)) << 32) | col(2 * e);
                            const float2 x = unpack2(fma2(s2, kappa2, wm2));
                            const float p0 = exp2f(x.x);
                            const float p1 = exp2f(x.y);
                            part_sum[h] = add2(part_sum[h], pack2(p0, p1));
                            __nv_bfloat162 pair = __floats2bfloat162_rn(p0, p1);
                            packed[2 * gi + h] = *reinterpret_cast<uint32_t*>(&pair);
                        }
                    }
                    tc::tmem_st16(s_col + 16 * quarter, packed);
                }
            }
            const float2 ps0 = unpack2(part_sum[0]);
            const float2 ps1 = unpack2(part_sum[1]);
            l_sum += (ps0.x + ps0.y) + (ps1.x + ps1.y);
            tc::tmem_wait_st();
            tc::fence_before_sync();
            tc::mbar_arrive(bar(kBarPFull + g));
        }
        if (ok && tiles > 0 && tc::mbar_wait_warp_suspend(bar(kBarOFinal + g), 0, abort_flag, kWaitLimit)) {
            // o = O / l, lse = m + log2(l) for this block's rows.
            tc::fence_after_sync();
            const int64_t token0 = (block_a + g) * kQueryBlock;
            const int n = static_cast<int>(min(static_cast<int64_t>(kQueryBlock), args.seq - token0));
            const float inv = 1.f / l_sum;
            bf16* out_row = args.o + (head * args.seq + token0 + r) * kHeadDim;
#pragma unroll 1
            for (int c = 0; c < 128 / kChunk; ++c) {
                uint32_t o[kChunk];
                tc::tmem_ld16(o_col + kChunk * c, o);
                tc::tmem_wait_ld();
                tc::tmem_reg_fence(o);
                uint4 packed[2];
                uint32_t* pw = reinterpret_cast<uint32_t*>(packed);
#pragma unroll
                for (int e = 0; e < kChunk / 2; ++e) {
                    __nv_bfloat162 pair =
                        __floats2bfloat162_rn(__uint_as_float(o[2 * e]) * inv, __uint_as_float(o[2 * e + 1]) * inv);
                    pw[e] = *reinterpret_cast<uint32_t*>(&pair);
                }
                if (r < n) {
                    if (args.num_outs == 0) {
                        reinterpret_cast<uint4*>(out_row + kChunk * c)[0] = packed[0];
                        reinterpret_cast<uint4*>(out_row + kChunk * c)[1] = packed[1];
                    } else {
                        const int64_t row_off = ((args.out_head_base + head) * args.seq + token0 + r) * kHeadDim;
                        for (int d = 0; d < args.num_outs; ++d) {
                            uint4* dst = reinterpret_cast<uint4*>(args.outs[d] + row_off + kChunk * c);
                            dst[0] = packed[0];
                            dst[1] = packed[1];
                        }
                    }
                }
            }
            // Peers read the scattered rows once they learn (through a later
            // collective) that this kernel finished: make them visible system-wide.
            if (args.num_outs > 0) __threadfence_system();
            if (args.lse != nullptr && r < n) args.lse[head * args.seq + token0 + r] = m_used + log2f(l_sum);
        }
    }

    tc::fence_before_sync();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, kTmemColumns);
    }
    if (tid == 0 && *abort_flag) raise_device_error(args.error, ABX_ERR_DEVICE_TIMEOUT);
}

int64_t pair_stride(int64_t samples, int64_t text_granules) {
    return ceil_div(2 * samples + text_granules + 3 * kPairGranules, kPairGranules) * kPairGranules;
}

size_t plan_smem_bytes(int64_t fine_blocks, int64_t samples) {
    // 16-bit slot map (rounded to words), two bitmaps, one byte per sample
    return static_cast<size_t>(ceil_div(fine_blocks, 2)) * 4 + static_cast<size_t>(ceil_div(fine_blocks, 32)) * 8 +
           static_cast<size_t>(samples);
}

}  // namespace

size_t pair_workspace_bytes(int64_t bh, int64_t seq, int64_t samples, int64_t text_tokens) {
    const int64_t pairs = bh * ceil_div(ceil_div(seq, kQueryBlock), 2);
    const int64_t stride = pair_stride(samples, ceil_div(text_tokens, kKv4));
    return static_cast<size_t>(pairs) * static_cast<size_t>(stride) * 8 + static_cast<size_t>(pairs) * 16 + 256;
}

bool pair_supported(int64_t seq, int64_t samples, int64_t text_tokens) {
    const int64_t text_granules = ceil_div(text_tokens, kKv4);
    if (samples < 1 || samples + text_granules >= static_cast<int64_t>(kNoSlot)) return false;
    return plan_smem_bytes(seq / kKv4, samples) <= 200 * 1024;
}

namespace {

struct PairLayout {
    int64_t qb, pairs_per_head, pairs, text_granules, stride;
    int4* info;
    uint32_t* entries;
    int32_t* codes;
};

PairLayout pair_layout(int64_t bh, int64_t seq, int64_t samples, int64_t text_tokens, void* workspace) {
    PairLayout l{};
    l.qb = ceil_div(seq, kQueryBlock);
    l.pairs_per_head = ceil_div(l.qb, 2);
    l.pairs = bh * l.pairs_per_head;
    l.text_granules = ceil_div(text_tokens, kKv4);
    l.stride = pair_stride(samples, l.text_granules);
    const uintptr_t ws = (reinterpret_cast<uintptr_t>(workspace) + 255) & ~static_cast<uintptr_t>(255);
    l.info = reinterpret_cast<int4*>(ws);
    l.entries = reinterpret_cast<uint32_t*>(ws + static_cast<uintptr_t>(l.pairs) * 16);
    l.codes = reinterpret_cast<int32_t*>(l.entries + l.pairs * l.stride);
    return l;
}

}  // namespace

cudaError_t launch_pair_plan(const int32_t* ids, int64_t bh, int64_t seq, int64_t samples, int64_t text_tokens,
                             void* workspace, size_t workspace_bytes, cudaStream_t stream) {
    if (workspace_bytes < pair_workspace_bytes(bh, seq, samples, text_tokens)) return cudaErrorInvalidValue;
    const PairLayout l = pair_layout(bh, seq, samples, text_tokens, workspace);
    PairPlanArgs plan{};
    plan.ids = ids;
    plan.entries = l.entries;
    plan.codes = l.codes;
    plan.info = l.info;
    plan.qb = l.qb;
    plan.stride = l.stride;
    plan.pairs_per_head = static_cast<int>(l.pairs_per_head);
    plan.samples = static_cast<int>(samples);
    plan.fine_blocks = static_cast<int>(seq / kKv4);
    plan.text_granules = static_cast<int>(l.text_granules);
    plan.text_tail = static_cast<int>(text_tokens % kKv4);
    const size_t plan_smem = plan_smem_bytes(seq / kKv4, samples);
    cudaError_t err = cudaFuncSetAttribute(pair_plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(plan_smem));
    if (err != cudaSuccess) return err;
    pair_plan_kernel<<<static_cast<unsigned>(l.pairs), kPlanThreads, plan_smem, stream>>>(plan);
    return cudaGetLastError();
}

cudaError_t launch_pair_prefill(const bf16* q, const bf16* k, const bf16* v, int64_t bh, int64_t seq,
                                const int32_t* ids, const float* log_weights, int64_t samples, const bf16* text_k,
                                const bf16* text_v, int64_t text_tokens, bf16* o, float* lse, void* workspace,
                                size_t workspace_bytes, cudaStream_t stream, bf16* const* outs, int num_outs,
                                int64_t out_head_base) {
    if (workspace_bytes < pair_workspace_bytes(bh, seq, samples, text_tokens)) return cudaErrorInvalidValue;
    if (num_outs < 0 || num_outs > kMaxScatterOutputs || (num_outs > 0 && outs == nullptr)) return cudaErrorInvalidValue;
    const PairLayout l = pair_layout(bh, seq, samples, text_tokens, workspace);
    PairArgs args{};
    args.ids = ids;
    args.logw = log_weights;
    args.entries = l.entries;
    args.codes = l.codes;
    args.info = l.info;
    args.o = o;
    args.lse = lse;
    args.seq = seq;
    args.qb = l.qb;
    args.stride = l.stride;
    args.text_tokens = text_tokens;
    args.kv_rows = bh * seq;
    args.pairs_per_head = static_cast<int>(l.pairs_per_head);
    args.samples = static_cast<int>(samples);
    args.fine_blocks = static_cast<int>(seq / kKv4);
    args.text_tail = static_cast<int>(text_tokens % kKv4);
    args.kappa = qk_scale_log2();
    args.error = device_error_word();
    args.num_outs = num_outs;
    args.out_head_base = out_head_base;
    for (int d = 0; d < num_outs; ++d) args.outs[d] = outs[d];
    PairMaps maps;
    cudaError_t err;
    if ((err = encode_rows(&maps.q, q, bh * seq, 128)) != cudaSuccess) return err;
    const bool has_text = text_tokens > 0 && text_k != nullptr && text_v != nullptr;
    const void* sources[2][2] = {{k, has_text ? text_k : k}, {v, has_text ? text_v : v}};
    const int64_t rows[2] = {bh * seq, has_text ? bh * text_tokens : bh * seq};
    for (int op = 0; op < 2; ++op)
        for (int src = 0; src < 2; ++src)
            if ((err = encode_rows(&maps.kv[op][src], sources[op][src], rows[src], kKv4)) != cudaSuccess) return err;
    err = cudaFuncSetAttribute(prefill_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(kSmemBytes));
    if (err != cudaSuccess) return err;
    cudaFuncAttributes attr{};
    if ((err = cudaFuncGetAttributes(&attr, prefill_pair_kernel)) != cudaSuccess) return err;
    if (static_cast<int64_t>(attr.numRegs) * kThreads <
        static_cast<int64_t>(8 * 32 * kSoftmaxRegs + (kThreads - 8 * 32) * kProducerRegs))
        return cudaErrorInvalidConfiguration;
    prefill_pair_kernel<<<static_cast<unsigned>(l.pairs), kThreads, kSmemBytes, stream>>>(args, maps);
    return cudaGetLastError();
}

cudaError_t launch_prefill_pair(const bf16* q, const bf16* k, const bf16* v, int64_t bh, int64_t seq,
                                const int32_t* ids, const float* log_weights, int64_t samples, const bf16* text_k,
                                const bf16* text_v, int64_t text_tokens, bf16* o, float* lse, void* workspace,
                                size_t workspace_bytes, cudaStream_t stream) {
    cudaError_t err = launch_pair_plan(ids, bh, seq, samples, text_tokens, workspace, workspace_bytes, stream);
    if (err != cudaSuccess) return err;
    return launch_pair_prefill(q, k, v, bh, seq, ids, log_weights, samples, text_k, text_v, text_tokens, o, lse,
                               workspace, workspace_bytes, stream);
}

}  // namespace abx
