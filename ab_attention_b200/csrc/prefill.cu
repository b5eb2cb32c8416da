// Paged sparse prefill with Horvitz-Thompson weights on the sm_100a tensor
// cores (replaces FlashInfer's fa3 batch prefill + the ABSipAttention variant,
// ab_attention/flashinfer_backend.py:30-58,164-242).
//
// For row = (head, 128-query block), the keys are the KV4 granules named by
// ids[row, :] (4 consecutive tokens each) followed by the always-included text
// granules. Logits are in log2 units: l = (q.k) * 128^-0.5 * log2(e) + w_slot,
// where w_slot = log2(1/pi) is the SIP weight of the granule's slot (0 for
// text). o = sum 2^(l-m) v / sum 2^(l-m) and lse = m + log2(sum): the HT ratio
// estimator of softmax attention.
//
// One CTA per row, 128-key tiles, warp-specialised (20 warps):
//   warps 0-3, 4-7  two softmax warpgroups; group g takes the tiles t with
//              t % 2 == g, so two independent streams of dependent math share
//              each SM sub-partition. Thread i of a group owns query row i =
//              TMEM lane i (row max / sum need no shuffles); it streams S out of
//              TMEM in 16-column chunks, writes P (bf16) back over S for the PV
//              product and rescales its O lazily (only when its running max
//              grows by more than 2^32). Group 1 hands (m, l) to group 0, which
//              merges the two partial softmaxes into the output.
//   warp  8    TMEM allocation + MMA issue (one thread): S(t) = Q K(t)^T with
//              both operands in shared memory, O(t%2) += P(t) V(t) with P read
//              from TMEM.
//   warps 9-13 gather Q and the K tiles, warps 14-19 the V tiles, with TMA: an
//              operand tile is 64 boxes of 4 rows x 64 columns (32 granules x
//              two 64-dim slabs), one box per lane, landing 128-byte swizzled at
//              the granule's rows of the UMMA operand tile; the stage mbarrier
//              counts the bytes. Granules past the end load from an out-of-range
//              row (zero fill).
// TMEM: S/P double buffer in columns [0,128) and [128,256), O of group 0 in
// [256,384), O of group 1 in [384,512).
// Stages: three for K and three for V (231.6 KB of shared memory with Q, just
// under the 227 KB per-block limit); the gathers are issued as soon as a stage
// frees, so deeper rings keep more of each operand in flight.
// Registers: the launch gives every thread kLaunchRegs; the softmax warpgroups
// then raise theirs to kSoftmaxRegs and the MMA/gather warpgroups lower theirs
// to kProducerRegs (setmaxnreg). The split fits the launch's allocation
// (checked at compile time and against the kernel's attributes on the host).
// Every mbarrier wait is bounded; on expiry the CTA drains its copies and MMAs,
// frees TMEM, records ABX_ERR_DEVICE_TIMEOUT in the device error word and exits.
// The waits let the hardware suspend the waiting warp (try_wait without a time
// hint), so it takes no issue slots from the warps computing beside it.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "f32x2.cuh"
#include "ibcs.cuh"
#include "tcgen05.cuh"
#include "tma_host.cuh"

#include <cfloat>
#include <mutex>

namespace abx {
namespace {

constexpr int kTileKeys = 128;
constexpr int kTileGranules = kTileKeys / kKv4;
constexpr int kKStages = 3;
constexpr int kVStages = 3;
constexpr uint32_t kSlabBytes = 128 * 128;       // 128 rows x 64 bf16
constexpr uint32_t kTileBytes = 2 * kSlabBytes;  // one 128 x 128 bf16 operand tile
constexpr int kSoftmaxGroups = 2;
constexpr int kMmaWarp = 8;
// Gather warps per operand. An operand tile is 64 TMA boxes (32 granules x two
// 64-dim slabs, box b = granule b/2, slab b%2); gather warp p of P issues boxes
// p, p+P, p+2P, ... one per lane. (A TMA request costs the issuing warp tens of
// cycles per active lane, so the requests are spread over several warps.)
constexpr int kKGatherWarps = 5;
constexpr int kVGatherWarps = 6;
constexpr int kBoxesPerTile = 2 * kTileGranules;
constexpr uint32_t kBoxBytes = kKv4 * 128;
constexpr int kKLoadWarp = kMmaWarp + 1;                // first K warp (also loads Q)
constexpr int kVLoadWarp = kKLoadWarp + kKGatherWarps;  // first V warp
constexpr int kThreads = (kVLoadWarp + kVGatherWarps) * 32;
constexpr int kChunk = 16;                              // TMEM columns per softmax step
constexpr int kLaunchRegs = 96;                         // 640 threads x 96 = 61,440 of 65,536
constexpr int kSoftmaxRegs = 168;                       // warpgroups 0-1
constexpr int kProducerRegs = 48;                       // warpgroups 2-4 (MMA + gather warps)
static_assert(kThreads == 640, "register split below assumes 20 warps");
static_assert(kThreads * kLaunchRegs <= 65536, "launch register allocation exceeds the SM");
static_assert(8 * 32 * kSoftmaxRegs + (kThreads - 8 * 32) * kProducerRegs <= kThreads * kLaunchRegs,
              "setmaxnreg split exceeds the launch allocation (the increase would never complete)");

constexpr uint32_t kTmemColumns = 512;
__device__ __forceinline__ constexpr uint32_t col_s(int b) { return 128u * static_cast<uint32_t>(b); }
__device__ __forceinline__ constexpr uint32_t col_o(int g) { return 256u + 128u * static_cast<uint32_t>(g); }

// shared memory map (offsets from a 1024-byte aligned base)
constexpr uint32_t kOffQ = 0;
constexpr uint32_t kOffK = kOffQ + kTileBytes;
constexpr uint32_t kOffV = kOffK + kKStages * kTileBytes;
constexpr uint32_t kOffMerge = kOffV + kVStages * kTileBytes;  // group 1's (m, l) per row
constexpr uint32_t kOffBar = kOffMerge + 2 * 128 * 4;
// barrier slots (8 bytes each)
constexpr int kBarQFull = 0;
constexpr int kBarKFull = 1;                      // kKStages
constexpr int kBarKEmpty = kBarKFull + kKStages;  // kKStages
constexpr int kBarVFull = kBarKEmpty + kKStages;  // kVStages
constexpr int kBarVEmpty = kBarVFull + kVStages;  // kVStages
constexpr int kBarSFull = kBarVEmpty + kVStages;  // 2
constexpr int kBarPFull = kBarSFull + 2;          // 2
constexpr int kBarPv = kBarPFull + 2;             // 2 (one per O accumulator)
constexpr int kBarOFinal = kBarPv + 2;
constexpr int kBarMerge = kBarOFinal + 1;
constexpr int kBarDrain = kBarMerge + 1;
constexpr int kNumBars = kBarDrain + 1;
constexpr uint32_t kOffTmemSlot = kOffBar + kNumBars * 8;
constexpr uint32_t kOffAbort = kOffTmemSlot + 4;
constexpr uint32_t kSmemUsed = kOffAbort + 4;
constexpr uint32_t kSmemBytes = kSmemUsed + 1024;  // slack for aligning the base
static_assert(kSmemBytes <= 227 * 1024, "shared memory exceeds the per-block limit");

constexpr uint64_t kWaitLimit = 400ull * 1000 * 1000;  // SM cycles per wait (~0.2 s)
// log2 units: rescale O when the row max grows by more than 2^32. P is bf16 and
// O, l are f32 (both with f32's exponent range), so P <= 2^32 and O, l stay
// far from overflow; a large threshold makes rescales rare after the first tile.
constexpr float kRescaleThreshold = 32.0f;

constexpr uint32_t kIdescS = tc::idesc_bf16_f32(128, kTileKeys, 0, 0);  // Q, K both K-major
constexpr uint32_t kIdescPV = tc::idesc_bf16_f32(128, 128, 0, 1);       // P K-major (TMEM), V MN-major

struct PrefillArgs {
    const bf16* q;
    const bf16* k;
    const bf16* v;
    const int32_t* ids;   // null: dense (granule id = slot)
    const float* logw;    // null: all weights 0
    const bf16* text_k;
    const bf16* text_v;
    bf16* o;
    float* lse;
    int64_t seq;          // key tokens per head (k, v)
    int64_t seq_q;        // query tokens per head (q, o, lse)
    int64_t qb;           // ceil(seq_q / 128)
    int64_t text_tokens;
    int samples;
    int granules;         // samples + ceil(text_tokens / 4)
    int text_tail;        // text_tokens % 4: keys of the last text granule past it are masked
    int fine_blocks;      // seq / 4: valid ids are [0, fine_blocks)
    int64_t kv_rows;      // bh * seq: rows of the K/V tensor maps (an index >= this reads zeros)
    int64_t text_rows;    // bh * text_tokens
    float kappa;          // 128^-0.5 * log2(e)
    int* error;           // device error word
};

// Tensor maps over [rows, 128] bf16 with 64-column boxes and 128-byte swizzle.
// Gather boxes are one granule (4 rows x 64 columns): index [operand][source]
// with operand 0 = K, 1 = V; source 0 = the head's tokens, 1 = text tokens.
struct PrefillMaps {
    CUtensorMap q;  // box 64 x 128 rows
    CUtensorMap kv[2][2];
    CUtensorMap kv_dense[2];  // K, V of the head's tokens, box 64 x 128 rows (dense tiles)
};

// KV4 id of granule `slot` of this row (dense: the slot itself); -1 when the
// slot is not a sampled granule (padding or text).
__device__ __forceinline__ int granule_id(const PrefillArgs& a, const int32_t* row_ids, int slot) {
    if (slot >= a.samples) return -1;
    return row_ids ? __ldg(row_ids + slot) : slot;
}

// First tensor-map row of granule `slot` (whose id was read by granule_id), and
// whether it comes from the text maps. Padding slots and out-of-range ids map
// to an out-of-range row (the TMA reads zeros there).
__device__ __forceinline__ int64_t granule_row(const PrefillArgs& a, int64_t head, int slot, int id, bool& text) {
    text = false;
    if (slot >= a.granules) return a.kv_rows;
    if (slot < a.samples) {
        if (id < 0 || id >= a.fine_blocks) {  // never read outside the head
            raise_device_error(a.error, ABX_ERR_INVALID_ARGUMENT);
            return a.kv_rows;
        }
        return head * a.seq + static_cast<int64_t>(id) * kKv4;
    }
    text = true;
    return head * a.text_tokens + static_cast<int64_t>(slot - a.samples) * kKv4;
}

// In chunk c of the tile holding the last slot, scores of that granule's keys
// past the last text token (its first `tail` keys are valid) -> -inf; the
// chunk's later columns belong to padding slots and are -inf already by weight.
// Before the softmax of the tile holding the last slot: the scores of that
// granule's keys past the last text token (its first `tail` keys are valid) are
// set to -inf in TMEM, so both softmax passes exclude them. Warp-collective.
__device__ __forceinline__ void mask_tail(uint32_t s_col, int last_slot, int tail) {
    const int local = last_slot % kTileGranules;
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

// Logit shift of granule `slot`: its SIP weight, 0 for text, -inf past the end.
__device__ __forceinline__ float slot_weight(const PrefillArgs& a, const float* row_w, int slot) {
    if (slot >= a.granules) return -INFINITY;
    return (slot < a.samples && row_w) ? __ldg(row_w + slot) : 0.f;
}

__global__ void __launch_bounds__(kThreads, 1) prefill_kernel(const PrefillArgs args,
                                                              const __grid_constant__ PrefillMaps maps) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_base = smem_addr(smem_raw);
    const uint32_t base = (raw_base + 1023u) & ~1023u;
    uint8_t* gbase = smem_raw + (base - raw_base);
    auto bar = [&](int i) { return base + kOffBar + 8u * i; };
    volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + kOffAbort);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + kOffTmemSlot);
    float* merge_m = reinterpret_cast<float*>(gbase + kOffMerge);
    float* merge_l = merge_m + 128;

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int64_t row = blockIdx.x;
    const int64_t head = row / args.qb;
    const int64_t token0 = (row - head * args.qb) * kQueryBlock;
    const int n = static_cast<int>(min(static_cast<int64_t>(kQueryBlock), args.seq_q - token0));
    const int tiles = (args.granules + kTileGranules - 1) / kTileGranules;
    const int32_t* row_ids = args.ids ? args.ids + row * args.samples : nullptr;
    const float* row_w = args.logw ? args.logw + row * args.samples : nullptr;

    // ---- set-up: barriers, TMEM ------------------------------------------------------
    if (tid == 0) {
        *abort_flag = 0;
        tc::mbar_init(bar(kBarQFull), 1);
        for (int s = 0; s < kKStages; ++s) {
            tc::mbar_init(bar(kBarKFull + s), kKGatherWarps);
            tc::mbar_init(bar(kBarKEmpty + s), 1);
        }
        for (int s = 0; s < kVStages; ++s) {
            tc::mbar_init(bar(kBarVFull + s), kVGatherWarps);
            tc::mbar_init(bar(kBarVEmpty + s), 1);
        }
        for (int b = 0; b < 2; ++b) {
            tc::mbar_init(bar(kBarSFull + b), 1);
            tc::mbar_init(bar(kBarPFull + b), 128);
            tc::mbar_init(bar(kBarPv + b), 1);
        }
        tc::mbar_init(bar(kBarOFinal), 1);
        tc::mbar_init(bar(kBarMerge), 128);
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
        // ---- producers: one TMA box per lane per operand tile --------------------------------
        const bool is_k = warp < kVLoadWarp;
        const int part = warp - (is_k ? kKLoadWarp : kVLoadWarp);
        const int nwarps = is_k ? kKGatherWarps : kVGatherWarps;
        const int box = part + nwarps * lane;
        const bool has_box = box < kBoxesPerTile;
        const int my_granule = has_box ? box >> 1 : 0;
        const int my_slab = box & 1;
        const int warp_boxes = (kBoxesPerTile - part + nwarps - 1) / nwarps;
        if (warp == kKLoadWarp && lane == 0) {
            // Q tile: two 128-row x 64-column boxes (rows past the block are never stored).
            tc::mbar_arrive_expect_tx(bar(kBarQFull), kTileBytes);
            const int32_t qy = static_cast<int32_t>(head * args.seq_q + token0);
            tc::tma_load_2d(base + kOffQ, &maps.q, 0, qy, bar(kBarQFull));
            tc::tma_load_2d(base + kOffQ + kSlabBytes, &maps.q, 64, qy, bar(kBarQFull));
        }
        const int op = is_k ? 0 : 1;
        const int stages = is_k ? kKStages : kVStages;
        const uint32_t ring = base + (is_k ? kOffK : kOffV);
        const int bar_full = is_k ? kBarKFull : kBarVFull;
        const int bar_empty = is_k ? kBarKEmpty : kBarVEmpty;
        int issued = 0;
        int next_id = granule_id(args, row_ids, my_granule);  // ids are read one tile ahead
        for (int t = 0; t < tiles; ++t) {
            const int st = t % stages;
            const int use = t / stages;
            const int slot = t * kTileGranules + my_granule;
            const int id = next_id;
            if (t + 1 < tiles) next_id = granule_id(args, row_ids, slot + kTileGranules);
            const bool free_ok =
                use == 0 || tc::mbar_wait_suspend(bar(bar_empty + st), (use - 1) & 1, abort_flag, kWaitLimit);
            if (!__all_sync(0xffffffffu, free_ok)) break;
            issued = t + 1;
            if (row_ids == nullptr && (t + 1) * kTileGranules <= args.samples) {
                // Dense tile (granule id = slot): 128 consecutive rows, two 128-row
                // boxes issued by the operand's first warp.
                if (lane == 0) {
                    const uint32_t bytes = part == 0 ? kTileBytes : 0u;
                    tc::mbar_arrive_expect_tx(bar(bar_full + st), bytes);
                    if (part == 0) {
                        const int32_t y = static_cast<int32_t>(head * args.seq + t * kTileKeys);
                        tc::tma_load_2d(ring + st * kTileBytes, &maps.kv_dense[op], 0, y, bar(bar_full + st));
                        tc::tma_load_2d(ring + st * kTileBytes + kSlabBytes, &maps.kv_dense[op], 64, y,
                                        bar(bar_full + st));
                    }
                }
                __syncwarp();
                continue;
            }
            if (lane == 0) tc::mbar_arrive_expect_tx(bar(bar_full + st), warp_boxes * kBoxBytes);
            __syncwarp();
            bool text;
            const int64_t y = granule_row(args, head, slot, id, text);
            const uint32_t dst = ring + st * kTileBytes + my_slab * kSlabBytes + my_granule * kBoxBytes;
            if (has_box)
                tc::tma_load_2d(dst, &maps.kv[op][text], 64 * my_slab, static_cast<int32_t>(y), bar(bar_full + st));
        }
        // Drain: every box issued above has landed before the CTA may exit (on the
        // normal path the MMA warp consumed them all and these waits return at once).
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
        // ---- MMA issue ------------------------------------------------------------------------
        // The whole warp runs this loop (warp-uniform operands); one elected lane issues.
        {
            bool ok = tc::mbar_wait_warp_suspend(bar(kBarQFull), 0, abort_flag, kWaitLimit);
            const uint64_t qdesc0 = tc::smem_desc(base + kOffQ, 16, 1024, tc::kSwizzle128B);
            auto issue_pv = [&](int u) -> bool {
                const int b = u & 1;
                const int vst = u % kVStages;
                if (!tc::mbar_wait_warp_suspend(bar(kBarVFull + vst), (u / kVStages) & 1, abort_flag, kWaitLimit))
                    return false;
                if (!tc::mbar_wait_warp_suspend(bar(kBarPFull + b), (u >> 1) & 1, abort_flag, kWaitLimit)) return false;
                tc::fence_after_sync();
                const uint64_t vdesc0 =
                    tc::smem_desc(base + kOffV + vst * kTileBytes, kSlabBytes, 1024, tc::kSwizzle128B);
#pragma unroll
                for (int j = 0; j < kTileKeys / 16; ++j) {
                    // 16 keys per step: P columns [8j, 8j+8); V rows [16j, 16j+16) (MN-major,
                    // leading offset = the second 64-dim slab, stride offset = 8-row atom; the
                    // descriptor's start field counts 16-byte units).
                    tc::mma_ts_elect(tmem + col_o(b), tmem + col_s(b) + 8 * j, vdesc0 + ((j * 16 * 128) >> 4),
                                     kIdescPV, (u >= 2 || j > 0) ? 1u : 0u);
                }
                tc::mma_commit_elect(bar(kBarVEmpty + vst));
                tc::mma_commit_elect(bar(kBarPv + b));
                return true;
            };
            for (int t = 0; ok && t < tiles; ++t) {
                const int b = t & 1;
                const int kst = t % kKStages;
                if (!tc::mbar_wait_warp_suspend(bar(kBarKFull + kst), (t / kKStages) & 1, abort_flag, kWaitLimit)) {
                    ok = false;
                    break;
                }
                const uint64_t kdesc0 = tc::smem_desc(base + kOffK + kst * kTileBytes, 16, 1024, tc::kSwizzle128B);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    // 16 dims per step inside a 64-dim slab: advance the start by 32 bytes.
                    const uint32_t off = ((j >> 2) * kSlabBytes + (j & 3) * 32) >> 4;
                    tc::mma_ss_elect(tmem + col_s(b), qdesc0 + off, kdesc0 + off, kIdescS, j > 0 ? 1u : 0u);
                }
                tc::mma_commit_elect(bar(kBarKEmpty + kst));
                tc::mma_commit_elect(bar(kBarSFull + b));
                if (t > 0 && !issue_pv(t - 1)) ok = false;
            }
            if (ok && !issue_pv(tiles - 1)) ok = false;
            if (ok) tc::mma_commit_elect(bar(kBarOFinal));
            // Drain: every MMA issued above has completed before TMEM is freed.
            tc::mma_commit_elect(bar(kBarDrain));
            if (lane == 0) tc::mbar_wait_suspend(bar(kBarDrain), 0, abort_flag, kWaitLimit, /*honor_abort=*/false);
        }
        __syncwarp();
    }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;\n" ::"n"(kSoftmaxRegs));
        // ---- softmax group g (thread = query row = TMEM lane) ---------------------------------------
        const int g = warp >> 2;
        const int r = tid & 127;  // query row
        const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
        const uint32_t o_col = lane_base + col_o(g);
        float m_used = -INFINITY;
        float l_sum = 0.f;
        bool ok = true;
        // The last text granule (the last slot) may hold fewer than 4 keys; in
        // its tile the chunk holding it masks its columns past the last key.
        const int tail_tile = args.text_tail ? (args.granules - 1) / kTileGranules : -1;
        // Lane j holds the weight of granule j of the current tile; the group's
        // next tile (t + 2) is read one step ahead.
        float w_next = slot_weight(args, row_w, g * kTileGranules + lane);
        for (int t = g; t < tiles; t += kSoftmaxGroups) {
            const float w_lane = w_next;
            if (t + kSoftmaxGroups < tiles)
                w_next = slot_weight(args, row_w, (t + kSoftmaxGroups) * kTileGranules + lane);
            if (!tc::mbar_wait_warp_suspend(bar(kBarSFull + g), (t >> 1) & 1, abort_flag, kWaitLimit)) {
                ok = false;
                break;
            }
            tc::fence_after_sync();
            const uint32_t s_col = lane_base + col_s(g);
            if (t == tail_tile) mask_tail(s_col, args.granules - 1, args.text_tail);
            // Pass 1: row max of x = s * kappa + w over the tile, streaming S out of
            // TMEM 16 columns at a time (double-buffered), 4 independent chains.
            // x is monotone in s within a granule (one w, kappa > 0), so the max
            // of a granule is fma(max s, kappa, w): one FFMA per four columns.
            float part_max[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
            {
                uint32_t buf[2][kChunk];
                tc::tmem_ld16(s_col, buf[0]);
                tc::tmem_wait_ld();
                tc::tmem_reg_fence(buf[0]);
#pragma unroll
                for (int c = 0; c < kTileKeys / kChunk; ++c) {
                    if (c + 1 < kTileKeys / kChunk) tc::tmem_ld16(s_col + kChunk * (c + 1), buf[(c + 1) & 1]);
#pragma unroll
                    for (int q4 = 0; q4 < kChunk / 4; ++q4) {
                        const float w = __shfl_sync(0xffffffffu, w_lane, c * (kChunk / 4) + q4);
                        const uint32_t* g4 = buf[c & 1] + 4 * q4;
                        const float smax = fmaxf(fmaxf(__uint_as_float(g4[0]), __uint_as_float(g4[1])),
                                                 fmaxf(__uint_as_float(g4[2]), __uint_as_float(g4[3])));
                        part_max[q4] = fmaxf(part_max[q4], fmaf(smax, args.kappa, w));
                    }
                    if (c + 1 < kTileKeys / kChunk) {
                        tc::tmem_wait_ld();
                        tc::tmem_reg_fence(buf[(c + 1) & 1]);
                    }
                }
            }
            const float tile_max = fmaxf(fmaxf(part_max[0], part_max[1]), fmaxf(part_max[2], part_max[3]));
            // Lazy rescale, decided per warp (tcgen05.ld/st are warp-collective):
            // a row whose max grew by more than 2^32 moves its reference max and
            // scales its O row and sum; the other rows of the warp scale by 1.
            // O(g) holds PV of the group's earlier tiles, all complete: S(t) was
            // committed after them.
            const bool grow = tile_max > m_used + kRescaleThreshold;
            if (__any_sync(0xffffffffu, grow)) {
                const float m_new = grow ? tile_max : m_used;
                const float scale = grow ? exp2f(m_used - m_new) : 1.0f;
                l_sum *= scale;
                if (t >= kSoftmaxGroups) {
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
            // Pass 2: P = 2^(s * kappa + (w - m)) as bf16 pairs, re-reading S; chunk c's
            // 8 packed words overwrite S columns [8c, 8c + 8), which no later chunk reads.
            // Column pairs go through packed f32x2 FMAs and sums.
            uint64_t part_sum[2] = {kZeros2, kZeros2};
            {
                const uint64_t kappa2 = pack2(args.kappa, args.kappa);
                uint32_t buf[2][kChunk];
                tc::tmem_ld16(s_col, buf[0]);
                tc::tmem_wait_ld();
                tc::tmem_reg_fence(buf[0]);
#pragma unroll
                for (int c = 0; c < kTileKeys / kChunk; ++c) {
                    if (c + 1 < kTileKeys / kChunk) tc::tmem_ld16(s_col + kChunk * (c + 1), buf[(c + 1) & 1]);
                    uint32_t packed[kChunk / 2];
#pragma unroll
                    for (int q4 = 0; q4 < kChunk / 4; ++q4) {
                        const float wm = __shfl_sync(0xffffffffu, w_lane, c * (kChunk / 4) + q4) - m_used;
                        const uint64_t wm2 = pack2(wm, wm);
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const int e = 2 * q4 + h;
                            const uint64_t s2 = (static_cast<uint64_t>(buf[c & 1][2 * e + 1]) << 32) | buf[c & 1][2 * e];
                            const float2 x = unpack2(fma2(s2, kappa2, wm2));
                            const float p0 = exp2f(x.x);
                            const float p1 = exp2f(x.y);
                            part_sum[h] = add2(part_sum[h], pack2(p0, p1));
                            __nv_bfloat162 pair = __floats2bfloat162_rn(p0, p1);
                            packed[e] = *reinterpret_cast<uint32_t*>(&pair);
                        }
                    }
                    tc::tmem_st8(s_col + (kChunk / 2) * c, packed);
                    if (c + 1 < kTileKeys / kChunk) {
                        tc::tmem_wait_ld();
                        tc::tmem_reg_fence(buf[(c + 1) & 1]);
                    }
                }
            }
            const float2 ps0 = unpack2(part_sum[0]);
            const float2 ps1 = unpack2(part_sum[1]);
            l_sum += (ps0.x + ps0.y) + (ps1.x + ps1.y);
            tc::tmem_wait_st();
            tc::fence_before_sync();
            tc::mbar_arrive(bar(kBarPFull + g));
        }
        if (g == 1) {
            // Hand this group's running max and sum to group 0 (also on abort).
            merge_m[r] = m_used;
            merge_l[r] = l_sum;
            tc::mbar_arrive(bar(kBarMerge));
        } else if (ok && tc::mbar_wait_warp_suspend(bar(kBarOFinal), 0, abort_flag, kWaitLimit) &&
                   tc::mbar_wait_warp_suspend(bar(kBarMerge), 0, abort_flag, kWaitLimit)) {
            // Merge the two partial softmaxes: o = (O0 2^(m0-m) + O1 2^(m1-m)) / (l0 2^(m0-m) + l1 2^(m1-m)).
            tc::fence_after_sync();
            const float m1 = merge_m[r];
            const float l1 = merge_l[r];
            const bool has1 = tiles > 1;  // group 1 saw at least one tile
            const float m = has1 ? fmaxf(m_used, m1) : m_used;
            const float s0 = exp2f(m_used - m);
            const float s1 = has1 ? exp2f(m1 - m) : 0.f;
            const float l = l_sum * s0 + (has1 ? l1 * s1 : 0.f);
            const float inv = 1.f / l;
            const float a0 = s0 * inv;
            const float a1 = s1 * inv;
            const uint32_t o1_col = lane_base + col_o(1);
            bf16* out_row = args.o + (head * args.seq_q + token0 + r) * kHeadDim;
#pragma unroll 1
            for (int c = 0; c < 128 / kChunk; ++c) {
                uint32_t o0[kChunk], o1[kChunk];
                tc::tmem_ld16(o_col + kChunk * c, o0);
                if (has1) tc::tmem_ld16(o1_col + kChunk * c, o1);
                tc::tmem_wait_ld();
                tc::tmem_reg_fence(o0);
                tc::tmem_reg_fence(o1);
                uint4 packed[2];
                uint32_t* pw = reinterpret_cast<uint32_t*>(packed);
#pragma unroll
                for (int e = 0; e < kChunk / 2; ++e) {
                    float v0 = __uint_as_float(o0[2 * e]) * a0;
                    float v1 = __uint_as_float(o0[2 * e + 1]) * a0;
                    if (has1) {
                        v0 = fmaf(__uint_as_float(o1[2 * e]), a1, v0);
                        v1 = fmaf(__uint_as_float(o1[2 * e + 1]), a1, v1);
                    }
                    __nv_bfloat162 pair = __floats2bfloat162_rn(v0, v1);
                    pw[e] = *reinterpret_cast<uint32_t*>(&pair);
                }
                if (r < n) {
                    reinterpret_cast<uint4*>(out_row + kChunk * c)[0] = packed[0];
                    reinterpret_cast<uint4*>(out_row + kChunk * c)[1] = packed[1];
                }
            }
            if (args.lse != nullptr && r < n) args.lse[head * args.seq_q + token0 + r] = m + log2f(l);
        }
    }

    // ---- teardown ------------------------------------------------------------------------------
    tc::fence_before_sync();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, kTmemColumns);
    }
    if (tid == 0 && *abort_flag) raise_device_error(args.error, ABX_ERR_DEVICE_TIMEOUT);
}

}  // namespace

static int64_t rows_or(int64_t rows, int64_t fallback) { return rows > 0 ? rows : fallback; }

cudaError_t launch_prefill(const bf16* q, int64_t q_tokens, const bf16* k, const bf16* v, int64_t bh, int64_t seq,
                           const int32_t* ids, const float* log_weights, int64_t samples,
                           const bf16* text_k, const bf16* text_v, int64_t text_tokens, bf16* o,
                           float* lse, cudaStream_t stream) {
    PrefillArgs args{};
    args.q = q;
    args.k = k;
    args.v = v;
    args.ids = ids;
    args.logw = log_weights;
    args.text_k = text_k;
    args.text_v = text_v;
    args.o = o;
    args.lse = lse;
    args.seq = seq;
    args.seq_q = q_tokens;
    args.qb = ceil_div(q_tokens, kQueryBlock);
    args.text_tokens = text_tokens;
    args.text_tail = static_cast<int>(text_tokens % kKv4);
    args.samples = static_cast<int>(samples);
    args.granules = static_cast<int>(samples + ceil_div(text_tokens, kKv4));
    args.fine_blocks = static_cast<int>(seq / kKv4);
    args.text_rows = bh * text_tokens;
    args.kappa = qk_scale_log2();
    args.error = device_error_word();
    PrefillMaps maps;
    cudaError_t err;
    if ((err = encode_rows(&maps.q, q, bh * q_tokens, 128)) != cudaSuccess) return err;
    const bool has_text = text_tokens > 0 && text_k != nullptr && text_v != nullptr;
    const void* sources[2][2] = {{k, has_text ? text_k : k}, {v, has_text ? text_v : v}};
    const bool has_video = seq > 0;
    if (!has_video) sources[0][0] = sources[1][0] = has_text ? text_k : q;  // never read: no video slots
    const int64_t rows[2] = {has_video ? bh * seq : bh, has_text ? bh * text_tokens : rows_or(bh * seq, bh)};
    args.kv_rows = rows[0];  // first row past the video map: padding slots read zeros there
    for (int op = 0; op < 2; ++op) {
        for (int src = 0; src < 2; ++src)
            if ((err = encode_rows(&maps.kv[op][src], sources[op][src], rows[src], kKv4)) != cudaSuccess) return err;
        if ((err = encode_rows(&maps.kv_dense[op], sources[op][0], rows[0], kTileKeys)) != cudaSuccess) return err;
    }
    err = cudaFuncSetAttribute(prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(kSmemBytes));
    if (err != cudaSuccess) return err;
    // The setmaxnreg increase only completes if the launch allocated at least the
    // split's registers; refuse to launch otherwise.
    cudaFuncAttributes attr{};
    if ((err = cudaFuncGetAttributes(&attr, prefill_kernel)) != cudaSuccess) return err;
    if (static_cast<int64_t>(attr.numRegs) * kThreads <
        static_cast<int64_t>(8 * 32 * kSoftmaxRegs + (kThreads - 8 * 32) * kProducerRegs))
        return cudaErrorInvalidConfiguration;
    prefill_kernel<<<static_cast<unsigned>(bh * args.qb), kThreads, kSmemBytes, stream>>>(args, maps);
    return cudaGetLastError();
}

}  // namespace abx
