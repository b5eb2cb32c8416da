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
// One CTA per row, warp-specialised (224 threads, at most two warps per SM
// sub-partition so the softmax warps can hold a whole 128-column S row in registers):
//   warps 0-3  softmax: thread i owns query row i = TMEM lane i, so row max and
//              row sum need no shuffles. Reads S from TMEM, writes P (bf16)
//              back over S for the PV product, rescales O lazily (only when the
//              running max grows by more than 2^8).
//   warp  4    TMEM allocation + MMA issue (one thread): S = Q K^T (both
//              operands in shared memory) and O += P V (P from TMEM).
//   warp  5    gathers Q and the K tiles, warp 6 the V tiles, with TMA: one
//              lane per KV4 granule issues two 4-row x 64-column boxes (the two
//              64-dim slabs) that land, 128-byte swizzled, at the granule's rows
//              of the UMMA operand tile; the stage mbarrier counts the bytes.
//              Granules past the end load from an out-of-range row (zero fill).
// TMEM: O in columns [0,128), S/P double buffer in [128,256) and [256,384).
// Every mbarrier wait is bounded; on expiry the CTA drains its copies and MMAs,
// frees TMEM, records ABX_ERR_DEVICE_TIMEOUT in the device error word and exits.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "ibcs.cuh"
#include "tcgen05.cuh"

#include <cfloat>
#include <mutex>

namespace abx {
namespace {

constexpr int kTileKeys = 128;
constexpr int kTileGranules = kTileKeys / kKv4;
constexpr int kKStages = 3;
constexpr int kVStages = 2;
constexpr uint32_t kSlabBytes = 128 * 128;       // 128 rows x 64 bf16
constexpr uint32_t kTileBytes = 2 * kSlabBytes;  // one 128 x 128 bf16 operand tile
constexpr int kSoftmaxWarps = 4;
constexpr int kMmaWarp = 4;
constexpr int kProducerWarpsPerOperand = 2;  // 1: each lane issues both slab boxes; 2: one slab per warp
constexpr int kKLoadWarp = 5;                                         // first K warp (also loads Q)
constexpr int kVLoadWarp = kKLoadWarp + kProducerWarpsPerOperand;     // first V warp
constexpr int kThreads = (kVLoadWarp + kProducerWarpsPerOperand) * 32;

constexpr uint32_t kTmemColumns = 512;
constexpr uint32_t kColO = 0;
__device__ __forceinline__ constexpr uint32_t col_s(int b) { return 128u + 128u * static_cast<uint32_t>(b); }

// shared memory map (offsets from a 1024-byte aligned base)
constexpr uint32_t kOffQ = 0;
constexpr uint32_t kOffK = kOffQ + kTileBytes;
constexpr uint32_t kOffV = kOffK + kKStages * kTileBytes;
constexpr uint32_t kOffBar = kOffV + kVStages * kTileBytes;
// barrier slots (8 bytes each)
constexpr int kBarQFull = 0;
constexpr int kBarKFull = 1;                      // kKStages
constexpr int kBarKEmpty = kBarKFull + kKStages;  // kKStages
constexpr int kBarVFull = kBarKEmpty + kKStages;  // kVStages
constexpr int kBarVEmpty = kBarVFull + kVStages;  // kVStages
constexpr int kBarSFull = kBarVEmpty + kVStages;  // 2
constexpr int kBarPFull = kBarSFull + 2;          // 2
constexpr int kBarPv = kBarPFull + 2;
constexpr int kBarOFinal = kBarPv + 1;
constexpr int kBarDrain = kBarOFinal + 1;
constexpr int kNumBars = kBarDrain + 1;
constexpr uint32_t kOffTmemSlot = kOffBar + kNumBars * 8;
constexpr uint32_t kOffAbort = kOffTmemSlot + 4;
constexpr uint32_t kSmemUsed = kOffAbort + 4;
constexpr uint32_t kSmemBytes = kSmemUsed + 1024;  // slack for aligning the base

constexpr uint64_t kWaitLimit = 400ull * 1000 * 1000;  // SM cycles per wait (~0.2 s)
constexpr float kRescaleThreshold = 8.0f;                // log2 units: rescale O when max grows > 2^8

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
    int64_t seq;
    int64_t qb;
    int64_t text_tokens;
    int samples;
    int granules;         // samples + text_tokens / 4
    int fine_blocks;      // seq / 4: valid ids are [0, fine_blocks)
    int64_t kv_rows;      // bh * seq: rows of the K/V tensor maps (an index >= this reads zeros)
    int64_t text_rows;    // bh * text_tokens
    float kappa;          // 128^-0.5 * log2(e)
    int* error;           // device error word
};

// Tensor maps over [rows, 128] bf16 with 64-column boxes and 128-byte swizzle.
struct PrefillMaps {
    CUtensorMap q;       // box 64 x 128 rows
    CUtensorMap k, v;    // box 64 x 4 rows (one granule)
    CUtensorMap tk, tv;  // text keys / values, box 64 x 4 rows
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

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int64_t row = blockIdx.x;
    const int64_t head = row / args.qb;
    const int64_t token0 = (row - head * args.qb) * kQueryBlock;
    const int n = static_cast<int>(min(static_cast<int64_t>(kQueryBlock), args.seq - token0));
    const int tiles = (args.granules + kTileGranules - 1) / kTileGranules;
    const int32_t* row_ids = args.ids ? args.ids + row * args.samples : nullptr;
    const float* row_w = args.logw ? args.logw + row * args.samples : nullptr;

    // ---- set-up: barriers, TMEM ------------------------------------------------------
    if (tid == 0) {
        *abort_flag = 0;
        tc::mbar_init(bar(kBarQFull), 1);
        for (int s = 0; s < kKStages; ++s) {
            tc::mbar_init(bar(kBarKFull + s), kProducerWarpsPerOperand);
            tc::mbar_init(bar(kBarKEmpty + s), 1);
        }
        for (int s = 0; s < kVStages; ++s) {
            tc::mbar_init(bar(kBarVFull + s), kProducerWarpsPerOperand);
            tc::mbar_init(bar(kBarVEmpty + s), 1);
        }
        for (int b = 0; b < 2; ++b) {
            tc::mbar_init(bar(kBarSFull + b), 1);
            tc::mbar_init(bar(kBarPFull + b), kSoftmaxWarps * 32);
        }
        tc::mbar_init(bar(kBarPv), 1);
        tc::mbar_init(bar(kBarOFinal), 1);
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

    if (warp >= kKLoadWarp) {
        // ---- producers: one lane per granule, one TMA box per 64-dim slab ----------------------
        const bool is_k = warp < kVLoadWarp;
        const int part = warp - (is_k ? kKLoadWarp : kVLoadWarp);  // which slab, when split
        const int slab0 = kProducerWarpsPerOperand == 2 ? part : 0;
        const int nslabs = kProducerWarpsPerOperand == 2 ? 1 : 2;
        if (warp == kKLoadWarp && lane == 0) {
            // Q tile: two 128-row x 64-column boxes (rows past the block are never stored).
            tc::mbar_arrive_expect_tx(bar(kBarQFull), kTileBytes);
            const int32_t qy = static_cast<int32_t>(head * args.seq + token0);
            tc::tma_load_2d(base + kOffQ, &maps.q, 0, qy, bar(kBarQFull));
            tc::tma_load_2d(base + kOffQ + kSlabBytes, &maps.q, 64, qy, bar(kBarQFull));
        }
        const CUtensorMap* main_map = is_k ? &maps.k : &maps.v;
        const CUtensorMap* text_map = is_k ? &maps.tk : &maps.tv;
        const int stages = is_k ? kKStages : kVStages;
        const uint32_t ring = base + (is_k ? kOffK : kOffV);
        const int bar_full = is_k ? kBarKFull : kBarVFull;
        const int bar_empty = is_k ? kBarKEmpty : kBarVEmpty;
        int issued = 0;
        int next_id = granule_id(args, row_ids, lane);  // ids are read one tile ahead
        for (int t = 0; t < tiles; ++t) {
            const int st = t % stages;
            const int use = t / stages;
            const int slot = t * kTileGranules + lane;
            const int id = next_id;
            if (t + 1 < tiles) next_id = granule_id(args, row_ids, slot + kTileGranules);
            const bool free_ok =
                use == 0 || tc::mbar_wait(bar(bar_empty + st), (use - 1) & 1, abort_flag, kWaitLimit);
            if (!__all_sync(0xffffffffu, free_ok)) break;
            issued = t + 1;
            if (lane == 0) tc::mbar_arrive_expect_tx(bar(bar_full + st), nslabs * kSlabBytes);
            __syncwarp();
            bool text;
            const int64_t y = granule_row(args, head, slot, id, text);
            const CUtensorMap* map = text ? text_map : main_map;
            const uint32_t dst = ring + st * kTileBytes + lane * (kKv4 * 128);
            for (int sl = slab0; sl < slab0 + nslabs; ++sl)
                tc::tma_load_2d(dst + sl * kSlabBytes, map, 64 * sl, static_cast<int32_t>(y), bar(bar_full + st));
        }
        // Drain: every box issued above has landed before the CTA may exit (on the
        // normal path the MMA warp consumed them all and these waits return at once).
        if (lane == 0) {
            for (int st = 0; st < stages && st < issued; ++st) {
                const int last_use = (issued - 1 - st) / stages;
                tc::mbar_wait(bar(bar_full + st), last_use & 1, abort_flag, kWaitLimit, /*honor_abort=*/false);
            }
            if (warp == kKLoadWarp) tc::mbar_wait(bar(kBarQFull), 0, abort_flag, kWaitLimit, /*honor_abort=*/false);
        }
        __syncwarp();
    } else if (warp == kMmaWarp) {
        // ---- MMA issue ------------------------------------------------------------------------
        if (lane == 0) {
            bool ok = tc::mbar_wait(bar(kBarQFull), 0, abort_flag, kWaitLimit);
            const uint32_t q_base = base + kOffQ;
            auto issue_pv = [&](int u) -> bool {
                const int b = u & 1;
                const int vst = u % kVStages;
                if (!tc::mbar_wait(bar(kBarVFull + vst), (u / kVStages) & 1, abort_flag, kWaitLimit)) return false;
                if (!tc::mbar_wait(bar(kBarPFull + b), (u >> 1) & 1, abort_flag, kWaitLimit)) return false;
                tc::fence_after_sync();
                const uint32_t v_base = base + kOffV + vst * kTileBytes;
#pragma unroll
                for (int j = 0; j < kTileKeys / 16; ++j) {
                    // 16 keys per step: P columns [8j, 8j+8); V rows [16j, 16j+16) (MN-major,
                    // leading offset = the second 64-dim slab, stride offset = 8-row atom).
                    const uint64_t bdesc = tc::smem_desc(v_base + j * 16 * 128, kSlabBytes, 1024, tc::kSwizzle128B);
                    tc::mma_ts(tmem + kColO, tmem + col_s(b) + 8 * j, bdesc, kIdescPV, (u > 0 || j > 0) ? 1u : 0u);
                }
                tc::mma_commit(bar(kBarVEmpty + vst));
                tc::mma_commit(bar(kBarPv));
                return true;
            };
            for (int t = 0; ok && t < tiles; ++t) {
                const int b = t & 1;
                const int kst = t % kKStages;
                if (!tc::mbar_wait(bar(kBarKFull + kst), (t / kKStages) & 1, abort_flag, kWaitLimit)) {
                    ok = false;
                    break;
                }
                const uint32_t k_base = base + kOffK + kst * kTileBytes;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    // 16 dims per step inside a 64-dim slab: advance the start by 32 bytes.
                    const uint32_t off = (j >> 2) * kSlabBytes + (j & 3) * 32;
                    const uint64_t adesc = tc::smem_desc(q_base + off, 16, 1024, tc::kSwizzle128B);
                    const uint64_t bdesc = tc::smem_desc(k_base + off, 16, 1024, tc::kSwizzle128B);
                    tc::mma_ss(tmem + col_s(b), adesc, bdesc, kIdescS, j > 0 ? 1u : 0u);
                }
                tc::mma_commit(bar(kBarKEmpty + kst));
                tc::mma_commit(bar(kBarSFull + b));
                if (t > 0 && !issue_pv(t - 1)) ok = false;
            }
            if (ok && !issue_pv(tiles - 1)) ok = false;
            if (ok) tc::mma_commit(bar(kBarOFinal));
            // Drain: every MMA issued above has completed before TMEM is freed.
            tc::mma_commit(bar(kBarDrain));
            tc::mbar_wait(bar(kBarDrain), 0, abort_flag, kWaitLimit, /*honor_abort=*/false);
        }
        __syncwarp();
    } else {
        // ---- softmax (thread = query row = TMEM lane) -------------------------------------------
        const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
        float m_used = -INFINITY;
        float l_sum = 0.f;
        bool ok = true;
        // Lane j holds the weight of granule j of the current tile; the next
        // tile's weights are read one tile ahead.
        float w_next = slot_weight(args, row_w, lane);
        for (int t = 0; t < tiles; ++t) {
            const int b = t & 1;
            const float w_lane = w_next;
            if (t + 1 < tiles) w_next = slot_weight(args, row_w, (t + 1) * kTileGranules + lane);
            if (!tc::mbar_wait_warp(bar(kBarSFull + b), (t >> 1) & 1, abort_flag, kWaitLimit)) {
                ok = false;
                break;
            }
            tc::fence_after_sync();
            const uint32_t s_col = lane_base + col_s(b);
            // Pass 1: row max of x = s * kappa + w over the tile, streaming S from TMEM
            // 32 columns at a time (double-buffered loads, 8 independent max chains).
            float part_max[8];
#pragma unroll
            for (int g = 0; g < 8; ++g) part_max[g] = -INFINITY;
            {
                uint32_t buf[2][32];
                tc::tmem_ld32(s_col, buf[0]);
                tc::tmem_wait_ld();
                tc::tmem_reg_fence(buf[0]);
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    if (c + 1 < 4) tc::tmem_ld32(s_col + 32 * (c + 1), buf[(c + 1) & 1]);
#pragma unroll
                    for (int g = 0; g < 8; ++g) {
                        const float w = __shfl_sync(0xffffffffu, w_lane, c * 8 + g);
#pragma unroll
                        for (int e = 0; e < 4; ++e)
                            part_max[g] = fmaxf(part_max[g], fmaf(__uint_as_float(buf[c & 1][4 * g + e]), args.kappa, w));
                    }
                    if (c + 1 < 4) {
                        tc::tmem_wait_ld();
                        tc::tmem_reg_fence(buf[(c + 1) & 1]);
                    }
                }
            }
#pragma unroll
            for (int width = 4; width > 0; width >>= 1)
#pragma unroll
                for (int g = 0; g < width; ++g) part_max[g] = fmaxf(part_max[g], part_max[g + width]);
            const float tile_max = part_max[0];
            // Lazy rescale, decided per warp (tcgen05.ld/st are warp-collective):
            // a row whose max grew by more than 2^8 moves its reference max and
            // scales its O row and sum; the other rows of the warp scale by 1.
            const bool grow = tile_max > m_used + kRescaleThreshold;
            if (__any_sync(0xffffffffu, grow)) {
                const float m_new = grow ? tile_max : m_used;
                const float scale = grow ? exp2f(m_used - m_new) : 1.0f;
                l_sum *= scale;
                if (t > 0) {
                    // O holds PV(0..t-1): wait for PV(t-1), then rescale the rows in place.
                    if (!tc::mbar_wait_warp(bar(kBarPv), (t - 1) & 1, abort_flag, kWaitLimit)) {
                        ok = false;
                        break;
                    }
                    tc::fence_after_sync();
#pragma unroll 1
                    for (int c = 0; c < 8; ++c) {  // 16 columns at a time: S is still live in registers
                        uint32_t o[16];
                        tc::tmem_ld16(lane_base + kColO + 16 * c, o);
                        tc::tmem_wait_ld();
                        tc::tmem_reg_fence(o);
#pragma unroll
                        for (int e = 0; e < 16; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * scale);
                        tc::tmem_st16(lane_base + kColO + 16 * c, o);
                    }
                }
                m_used = m_new;
            }
            // Pass 2: P = 2^(s * kappa + (w - m)) as bf16 pairs, re-reading S in
            // 32-column chunks; chunk c's 16 packed words overwrite S columns
            // [16c, 16c + 16), which no later chunk reads.
            float part_sum[4] = {0.f, 0.f, 0.f, 0.f};
            {
                uint32_t buf[2][32];
                tc::tmem_ld32(s_col, buf[0]);
                tc::tmem_wait_ld();
                tc::tmem_reg_fence(buf[0]);
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    if (c + 1 < 4) tc::tmem_ld32(s_col + 32 * (c + 1), buf[(c + 1) & 1]);
                    uint32_t packed[16];
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        const float wm = __shfl_sync(0xffffffffu, w_lane, c * 8 + (e >> 1)) - m_used;
                        const float p0 = exp2f(fmaf(__uint_as_float(buf[c & 1][2 * e]), args.kappa, wm));
                        const float p1 = exp2f(fmaf(__uint_as_float(buf[c & 1][2 * e + 1]), args.kappa, wm));
                        part_sum[e & 3] += p0 + p1;
                        __nv_bfloat162 pair = __floats2bfloat162_rn(p0, p1);
                        packed[e] = *reinterpret_cast<uint32_t*>(&pair);
                    }
                    tc::tmem_st16(s_col + 16 * c, packed);
                    if (c + 1 < 4) {
                        tc::tmem_wait_ld();
                        tc::tmem_reg_fence(buf[(c + 1) & 1]);
                    }
                }
            }
            l_sum += (part_sum[0] + part_sum[1]) + (part_sum[2] + part_sum[3]);
            tc::tmem_wait_st();
            tc::fence_before_sync();
            tc::mbar_arrive(bar(kBarPFull + b));
        }
        if (ok && tc::mbar_wait_warp(bar(kBarOFinal), 0, abort_flag, kWaitLimit)) {
            tc::fence_after_sync();
            const int r = tid;  // query row
            const float inv = 1.f / l_sum;
            bf16* out_row = args.o + (head * args.seq + token0 + r) * kHeadDim;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                uint32_t o[32];
                tc::tmem_ld32(lane_base + kColO + 32 * c, o);
                tc::tmem_wait_ld();
                tc::tmem_reg_fence(o);
                if (r < n) {
#pragma unroll
                    for (int v = 0; v < 4; ++v) {
                        uint4 packed;
                        uint32_t* pw = reinterpret_cast<uint32_t*>(&packed);
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            __nv_bfloat162 pair = __floats2bfloat162_rn(__uint_as_float(o[8 * v + 2 * e]) * inv,
                                                                        __uint_as_float(o[8 * v + 2 * e + 1]) * inv);
                            pw[e] = *reinterpret_cast<uint32_t*>(&pair);
                        }
                        *reinterpret_cast<uint4*>(out_row + 32 * c + 8 * v) = packed;
                    }
                }
            }
            if (args.lse != nullptr && r < n) args.lse[head * args.seq + token0 + r] = m_used + log2f(l_sum);
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

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link).
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static std::once_flag once;
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult status;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &status) == cudaSuccess &&
            status == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    });
    return fn;
}

// [rows, 128] bf16 row-major, box = 64 columns x box_rows rows, 128-byte swizzle.
static cudaError_t encode_rows(CUtensorMap* map, const void* base, int64_t rows, uint32_t box_rows) {
    auto encode = tensor_map_encoder();
    if (encode == nullptr) return cudaErrorNotSupported;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(kHeadDim), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(kHeadDim) * 2};
    const cuuint32_t box[2] = {64, box_rows};
    const cuuint32_t elem_strides[2] = {1, 1};
    const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                              elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t launch_prefill(const bf16* q, const bf16* k, const bf16* v, int64_t bh, int64_t seq,
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
    args.qb = ceil_div(seq, kQueryBlock);
    args.text_tokens = text_tokens;
    args.samples = static_cast<int>(samples);
    args.granules = static_cast<int>(samples + text_tokens / kKv4);
    args.fine_blocks = static_cast<int>(seq / kKv4);
    args.kv_rows = bh * seq;
    args.text_rows = bh * text_tokens;
    args.kappa = qk_scale_log2();
    args.error = device_error_word();
    PrefillMaps maps;
    cudaError_t err;
    if ((err = encode_rows(&maps.q, q, bh * seq, 128)) != cudaSuccess) return err;
    if ((err = encode_rows(&maps.k, k, bh * seq, kKv4)) != cudaSuccess) return err;
    if ((err = encode_rows(&maps.v, v, bh * seq, kKv4)) != cudaSuccess) return err;
    const bool has_text = text_tokens > 0 && text_k != nullptr && text_v != nullptr;
    if ((err = encode_rows(&maps.tk, has_text ? text_k : k, has_text ? bh * text_tokens : bh * seq, kKv4)) !=
        cudaSuccess)
        return err;
    if ((err = encode_rows(&maps.tv, has_text ? text_v : v, has_text ? bh * text_tokens : bh * seq, kKv4)) !=
        cudaSuccess)
        return err;
    err = cudaFuncSetAttribute(prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(kSmemBytes));
    if (err != cudaSuccess) return err;
    const int64_t rows = bh * args.qb;
    prefill_kernel<<<static_cast<unsigned>(rows), kThreads, kSmemBytes, stream>>>(args, maps);
    return cudaGetLastError();
}

}  // namespace abx
