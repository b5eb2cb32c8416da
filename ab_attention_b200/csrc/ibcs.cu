// IBCS (intra-block clustering selector) for sm_100a.
//
// Stages, each reproducing the float arithmetic of the reference kernel it
// replaces (rounding points, reduction orders and `--use_fast_math` semantics
// are kept identical so the downstream page selection is bit-exact):
//   cluster_kernel  <- cluster_queries_kernel  csrc/ibcs.cu:106-238
//   pool_kernel     <- pool_keys_kernel        csrc/ibcs.cu:244-266
//   lse_kernel      <- ibcs_lse_kernel         csrc/ibcs.cu:370-489 (tcgen05 + TMEM)
//   mix_kernel      <- ibcs_scores_kernel      csrc/ibcs.cu:495-538
//
// What differs is the work decomposition: one thread per query for the
// clustering distances (the 32-lane partial sums and the xor-butterfly are
// evaluated inside the thread, in the reference's order), 16-byte vector
// loads and stores throughout, the scorer on tcgen05 (TMA key tiles, TMEM
// accumulators, one thread per centroid row running the reference's four
// lane-class chains), and a padded fp16 LSE scratch with 16-byte aligned rows.
// This file must be compiled with --use_fast_math (as csrc/ibcs.cu is).
#include "common.cuh"
#include "ibcs.cuh"
#include "f32x2.cuh"
#include "mix.cuh"
#include "tcgen05.cuh"
#include "tma_host.cuh"

#include <cfloat>
#include <cmath>

namespace abx {

namespace {

// ---------------------------------------------------------------------------
// Clustering
// ---------------------------------------------------------------------------

// Element (i, d) of a swizzled [128][128] bf16 tile stored as 16-byte chunks:
// chunk c of row i lives at slot i*16 + (c ^ (i & 7)), so a thread-per-row
// sweep and a thread-per-column sweep are both free of bank conflicts.
__device__ __forceinline__ int chunk_slot(int i, int c) { return i * 16 + (c ^ (i & 7)); }

__device__ __forceinline__ float tile_elem(const uint4* tile, int i, int d) {
    const bf16* chunk = reinterpret_cast<const bf16*>(tile + chunk_slot(i, d >> 3));
    return __bfloat162float(chunk[d & 7]);
}

// Squared distance of query row `i` to `center` (float[128], shared), summed the
// way the reference's warp does it (csrc/ibcs.cu:143-151,173-181): lane p folds
// dims p, p+32, p+64, p+96 in order, then the xor-butterfly 16,8,4,2,1 as seen
// from lane 0.
// The two bf16 of a 32-bit word as an f32x2 pair (low element in the low half).
__device__ __forceinline__ uint64_t bf16x2_to_f32x2(uint32_t w) {
    return (static_cast<uint64_t>(w & 0xffff0000u) << 32) | static_cast<uint64_t>(w << 16);
}

__device__ __forceinline__ float block_distance(const uint4* tile, int i, const float* center) {
    // part[q] holds lane partials (2q, 2q + 1): packed f32x2 operations apply to
    // each the same subtract and fused multiply-add, in the same order.
    uint64_t part[16];
#pragma unroll
    for (int q = 0; q < 16; ++q) part[q] = kZeros2;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const uint4 raw = tile[chunk_slot(i, 4 * k + c)];
            const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
            const float4 c0 = reinterpret_cast<const float4*>(center + 32 * k + 8 * c)[0];
            const float4 c1 = reinterpret_cast<const float4*>(center + 32 * k + 8 * c)[1];
            const uint64_t cp[4] = {pack2(c0.x, c0.y), pack2(c0.z, c0.w), pack2(c1.x, c1.y), pack2(c1.z, c1.w)};
#pragma unroll
            for (int h = 0; h < 4; ++h) {
                const uint64_t delta = sub2(bf16x2_to_f32x2(w[h]), cp[h]);
                part[4 * c + h] = fma2(delta, delta, part[4 * c + h]);
            }
        }
    }
    // xor-butterfly 16, 8, 4, 2 on pairs, then 1
#pragma unroll
    for (int width = 8; width > 0; width >>= 1) {
#pragma unroll
        for (int q = 0; q < width; ++q) part[q] = add2(part[q], part[q + width]);
    }
    const float2 last = unpack2(part[0]);
    return last.x + last.y;
}

// Block-wide argmax over one (value, index) per thread of a 128-thread block:
// largest value, ties to the smallest index (the cub::ArgMax rule the reference
// uses, csrc/ibcs.cu:94-102). The result is unique, so the reduction order is free.
__device__ __forceinline__ int argmax128(float value, int index, float* red_val, int* red_idx) {
#pragma unroll
    for (int mask = 16; mask > 0; mask >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, value, mask);
        const int oi = __shfl_xor_sync(0xffffffffu, index, mask);
        if (ov > value || (ov == value && oi < index)) {
            value = ov;
            index = oi;
        }
    }
    const int warp = threadIdx.x >> 5;
    __syncthreads();  // previous readers of red_* are done
    if ((threadIdx.x & 31) == 0) {
        red_val[warp] = value;
        red_idx[warp] = index;
    }
    __syncthreads();
    float best = red_val[0];
    int best_index = red_idx[0];
#pragma unroll
    for (int w = 1; w < 4; ++w) {
        if (red_val[w] > best || (red_val[w] == best && red_idx[w] < best_index)) {
            best = red_val[w];
            best_index = red_idx[w];
        }
    }
    return best_index;
}

// The pooled representatives of one KV4 block's 8-dim chunk (pool_keys_kernel,
// csrc/ibcs.cu:244-266): p_t = bf16_rn(0.5f * (k_{2t} + k_{2t+1})), t = 0, 1.
__device__ __forceinline__ void pool_chunk(const bf16* __restrict__ k, bf16* __restrict__ pooled, int64_t block,
                                           int chunk) {
    const uint4* src = reinterpret_cast<const uint4*>(k + block * kKv4 * kHeadDim) + chunk;
    uint4 rows[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) rows[r] = __ldg(src + r * 16);
    uint4 out[2];
#pragma unroll
    for (int rep = 0; rep < 2; ++rep) {
        const bf16* a = reinterpret_cast<const bf16*>(&rows[2 * rep]);
        const bf16* b = reinterpret_cast<const bf16*>(&rows[2 * rep + 1]);
        bf16* o = reinterpret_cast<bf16*>(&out[rep]);
#pragma unroll
        for (int e = 0; e < 8; ++e)
            o[e] = __float2bfloat16_rn(0.5f * (__bfloat162float(a[e]) + __bfloat162float(b[e])));
    }
    uint4* dst = reinterpret_cast<uint4*>(pooled + block * kReps * kHeadDim) + chunk;
    dst[0] = out[0];
    dst[16] = out[1];
}

// k / pooled (both or neither): the CTA of query block r also pools the KV4
// blocks of the same 128 tokens (blocks 32r .. 32r + 31 of the head), so the
// key pooling rides on the clustering's latency-bound pass instead of a launch
// of its own.
__global__ __launch_bounds__(128) void cluster_kernel(
    const bf16* __restrict__ q, int64_t seq, int64_t qb, bf16* __restrict__ centroids,
    bf16* __restrict__ scaled, float* __restrict__ populations,
    int32_t* __restrict__ assignments, float kappa, const bf16* __restrict__ k,
    bf16* __restrict__ pooled) {
    __shared__ uint4 tile[128 * 16];
    __shared__ __align__(16) float center[kHeadDim];
    __shared__ int members[kQueryBlock];
    __shared__ float red_val[4];
    __shared__ int red_idx[4];
    __shared__ int counts[kCentroids];

    const int tid = threadIdx.x;
    const int64_t row = blockIdx.x;
    const int64_t head = row / qb;
    const int64_t token0 = (row - head * qb) * kQueryBlock;
    const int n = static_cast<int>(min(static_cast<int64_t>(kQueryBlock), seq - token0));
    const uint4* src = reinterpret_cast<const uint4*>(q + (head * seq + token0) * kHeadDim);

    // 32 KB block, 16-byte coalesced loads; rows past the end read as zero.
#pragma unroll 4
    for (int p = 0; p < 16; ++p) {
        const int i = (tid >> 4) + 8 * p;
        const int c = tid & 15;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (i < n) v = src[i * 16 + c];
        tile[chunk_slot(i, c)] = v;
    }
    if (pooled != nullptr) {
        // n is a multiple of 4 (seq % 4 == 0, token0 % 128 == 0): whole KV4 blocks
        const int64_t block0 = head * (seq / kKv4) + token0 / kKv4;
        const int items = (n / kKv4) * 16;
        for (int it = tid; it < items; it += 128) pool_chunk(k, pooled, block0 + (it >> 4), it & 15);
    }
    __syncthreads();

    // Block mean, sequential over queries (csrc/ibcs.cu:130-140).
    {
        float sum = 0.0f;
        for (int i = 0; i < n; ++i) sum += tile_elem(tile, i, tid);
        center[tid] = sum / static_cast<float>(n);
    }
    __syncthreads();

    const bool valid = tid < n;
    float distance = block_distance(tile, tid, center);
    int next = argmax128(valid ? distance : -INFINITY, tid, red_val, red_idx);

    // Farthest-first centres with strict-< assignment (csrc/ibcs.cu:165-197).
    float min_distance = INFINITY;
    int assignment = 0;
#pragma unroll 1
    for (int slot = 0; slot < kCentroids; ++slot) {
        __syncthreads();  // all threads are done with the previous centre row
        center[tid] = tile_elem(tile, next, tid);
        __syncthreads();
        distance = block_distance(tile, tid, center);
        if (valid && distance < min_distance) {
            min_distance = distance;
            assignment = slot;
        }
        if (slot + 1 < kCentroids) {
            next = argmax128(valid ? min_distance : -INFINITY, tid, red_val, red_idx);
        }
    }

    if (tid < kCentroids) counts[tid] = 0;
    members[tid] = valid ? assignment : -1;
    __syncthreads();
    if (valid) atomicAdd(&counts[assignment], 1);
    __syncthreads();
    if (tid < kCentroids) populations[row * kCentroids + tid] = static_cast<float>(counts[tid]);
    if (assignments != nullptr) assignments[row * kQueryBlock + tid] = members[tid];

    // Member sums per (centroid, 8-dim chunk), sequential over queries
    // (csrc/ibcs.cu:213-227); centroid = bf16_rn(sum / count) (:228-237).
    const int cluster = tid >> 4;
    const int chunk = tid & 15;
    uint64_t acc2[4] = {kZeros2, kZeros2, kZeros2, kZeros2};  // dims (2h, 2h + 1) of the chunk
    for (int i = 0; i < n; ++i) {
        if (members[i] == cluster) {
            const uint4 raw = tile[chunk_slot(i, chunk)];
            acc2[0] = add2(acc2[0], bf16x2_to_f32x2(raw.x));
            acc2[1] = add2(acc2[1], bf16x2_to_f32x2(raw.y));
            acc2[2] = add2(acc2[2], bf16x2_to_f32x2(raw.z));
            acc2[3] = add2(acc2[3], bf16x2_to_f32x2(raw.w));
        }
    }
    float acc[8];
#pragma unroll
    for (int h = 0; h < 4; ++h) {
        const float2 pair = unpack2(acc2[h]);
        acc[2 * h] = pair.x;
        acc[2 * h + 1] = pair.y;
    }
    const int count = counts[cluster];
    uint4 plain, pre;
    bf16* pv = reinterpret_cast<bf16*>(&plain);
    bf16* sv = reinterpret_cast<bf16*>(&pre);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        pv[e] = count > 0 ? __float2bfloat16_rn(acc[e] / static_cast<float>(count))
                          : __float2bfloat16_rn(0.0f);
        // MMA operand pre-scaled by 128^-0.5*log2(e) and rounded (csrc/ibcs.cu:293-295).
        sv[e] = __float2bfloat16_rn(__bfloat162float(pv[e]) * kappa);
    }
    const int64_t out = (row * kCentroids + cluster) * kHeadDim + chunk * 8;
    if (centroids != nullptr) *reinterpret_cast<uint4*>(centroids + out) = plain;
    if (scaled != nullptr) *reinterpret_cast<uint4*>(scaled + out) = pre;
}

// ---------------------------------------------------------------------------
// Key pooling: one thread per (KV4 block, 8-dim chunk), 16-byte loads/stores.
// ---------------------------------------------------------------------------

__global__ __launch_bounds__(256) void pool_kernel(const bf16* __restrict__ k, int64_t chunks,
                                                   bf16* __restrict__ pooled) {
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= chunks) return;
    pool_chunk(k, pooled, idx >> 4, static_cast<int>(idx & 15));
}

// ---------------------------------------------------------------------------
// Centroid x pooled-key scoring with per-centroid normalizers (tcgen05).
//
// One CTA scores 128 scaled-centroid rows of one head against every pooled key
// of that head: S = C K^T on the tensor cores (M = 128 rows, N = 64 keys = 32
// KV4 blocks per tile, K = 128 in eight k16 steps, f32 accumulators in TMEM),
// with the reference's epilogue per element. tcgen05.mma with this shape
// accumulates bit-identically to the reference's chain of eight
// mma.sync.m16n8k16 (checked on this hardware over 2M products, and covered
// by the bit-exact tests against the reference kernels).
//
//   warps 0-3  epilogue: thread m owns centroid row m (TMEM lane m) and reads
//              its row's 64 accumulators per tile; per KV4 block it forms the
//              pair LSE, rounds it to fp16, stores it, and folds it into one of
//              four running (max, den) chains by block index mod 4 (the
//              reference's four lane classes, csrc/ibcs.cu:329-335,454-462),
//              merged at the end as (c0 + c1) + (c2 + c3) (:468-477).
//   warp 4     allocates and frees TMEM; one thread loads the 32 KB centroid
//              tile once and 16 KB key tiles into a 2-stage ring (TMA), and
//              issues the MMAs into two TMEM buffers.
// Each epilogue warp stages its 32 rows x 32 blocks of fp16 per tile in shared
// memory (64-byte swizzle) and writes them with one TMA store: 64-byte row
// segments instead of 32 scattered 16-byte stores per instruction.
// 74 KB of shared memory, 128 TMEM columns and 160 threads: three CTAs per SM.
// ---------------------------------------------------------------------------

constexpr int kLseRows = 128;                          // centroid rows per CTA = TMEM lanes
constexpr int kLseTileBlocks = 32;                     // KV4 blocks per key tile
constexpr int kLseTileKeys = kLseTileBlocks * kReps;  // 64 pooled rows = MMA N
constexpr int kLseStages = 2;
constexpr int kLseCtlWarp = 4;  // TMEM allocation, TMA and MMA issue
constexpr int kLseThreads = 5 * 32;
constexpr uint32_t kLseSlabA = kLseRows * 128;      // 128 rows x 64 bf16
constexpr uint32_t kLseSlabB = kLseTileKeys * 128;  // 64 rows x 64 bf16
constexpr uint32_t kLseStageBytes = 2 * kLseSlabB;
constexpr uint32_t kLseOffA = 0;
constexpr uint32_t kLseOffB = 2 * kLseSlabA;
constexpr uint32_t kLseStageRowBytes = kLseTileBlocks * 2;                // 64 B of fp16 per row and tile
constexpr uint32_t kLseOutBufBytes = 32 * kLseStageRowBytes;                // one warp's 32 rows
constexpr uint32_t kLseOffOut = kLseOffB + kLseStages * kLseStageBytes;   // one buffer per epilogue warp
constexpr uint32_t kLseOffBar = kLseOffOut + 4 * kLseOutBufBytes;
constexpr int kLseBarAFull = 0;
constexpr int kLseBarBFull = 1;                            // kLseStages
constexpr int kLseBarBEmpty = kLseBarBFull + kLseStages;  // kLseStages
constexpr int kLseBarTFull = kLseBarBEmpty + kLseStages;  // 2 TMEM buffers
constexpr int kLseBarTEmpty = kLseBarTFull + 2;           // 2
constexpr int kLseBarDrain = kLseBarTEmpty + 2;
constexpr int kLseNumBars = kLseBarDrain + 1;
constexpr uint32_t kLseOffTmemSlot = kLseOffBar + kLseNumBars * 8;
constexpr uint32_t kLseOffAbort = kLseOffTmemSlot + 4;
constexpr uint32_t kLseSmemBytes = kLseOffAbort + 4 + 1024;  // slack for aligning the base
constexpr uint32_t kLseTmemColumns = 2 * kLseTileKeys;
constexpr uint32_t kLseIdesc = tc::idesc_bf16_f32(kLseRows, kLseTileKeys, 0, 0);  // both K-major
constexpr uint64_t kLseWaitLimit = 400ull * 1000 * 1000;  // SM cycles per wait (~0.2 s)

struct LseMaps {
    CUtensorMap centroids;  // [bh * qb * 8, 128], box 64 x 128 rows
    CUtensorMap keys;       // [bh * F * 2, 128], box 64 x 64 rows
    CUtensorMap out;        // fp16 [bh][qb * 8][ld] (F columns), box 32 x 32 rows (vector_rows only)
};

struct LseArgs {
    int64_t head_rows;  // qb * 8
    int64_t ld;         // fp16 LSE row stride (elements)
    int fine_blocks;
    int tiles;
    half* lse;
    float* lse_max;
    float* lse_den;
    int* error;
    bool vector_rows;   // every LSE row starts on a 16-byte boundary
};

// 2^(x - x) without a MUFU op: x * 0 + 1 is exactly 1 for finite x (and ex2 of
// +/-0 is exactly 1, a documented special value of ex2.approx); for an infinite
// or NaN x both are NaN. Inline PTX keeps the compiler from folding x * 0.
__device__ __forceinline__ float unit_exp(float x) {
    float r;
    asm("fma.rn.f32 %0, %1, 0f00000000, 0f3F800000;" : "=f"(r) : "f"(x));
    return r;
}

// The reference's accumulate_lse (csrc/ibcs.cu:329-335):
//   next = fmax(max, v); den = den * 2^(max - next) + 2^(v - next); max = next.
// One exponent is next - next (ex2 = unit_exp(next)), the other -|max - v|;
// the multiply-add keeps the reference's shape (one FFMA).
__device__ __forceinline__ void accumulate_lse(float& maximum, float& denominator, float value) {
    const float next_max = fmaxf(maximum, value);
    const bool keep = next_max == maximum;
    const float e = exp2f(-fabsf(maximum - value));
    const float unit = unit_exp(next_max);
    denominator = denominator * (keep ? unit : e) + (keep ? e : unit);
    maximum = next_max;
}

__device__ __forceinline__ void combine_lse(float& maximum, float& denominator, float other_max,
                                            float other_den) {
    const float next = fmaxf(maximum, other_max);
    denominator = denominator * exp2f(maximum - next) + other_den * exp2f(other_max - next);
    maximum = next;
}


// The reference's pair_lse (csrc/ibcs.cu:339-343) for two blocks A and B, from
// their raw representative scores with its "+ 1" (log2 of the representative
// size) applied first:
//   M = fmax(l, r); M + log2(fmax(2^(l - M) + 2^(r - M), 1e-20)).
// The term of the operand equal to M is 2^(M - M) = unit_exp(M); the other is
// 2^(-|l - r|) (l - r and r - l differ only in sign); the addition commutes.
__device__ __forceinline__ float2 pair_lse2(uint32_t a0, uint32_t a1, uint32_t b0, uint32_t b1) {
    const float2 la = unpack2(add2((static_cast<uint64_t>(a1) << 32) | a0, kOnes2));  // (l_A, r_A)
    const float2 lb = unpack2(add2((static_cast<uint64_t>(b1) << 32) | b0, kOnes2));
    const uint64_t m = pack2(fmaxf(la.x, la.y), fmaxf(lb.x, lb.y));
    const uint64_t e = pack2(exp2f(-fabsf(la.x - la.y)), exp2f(-fabsf(lb.x - lb.y)));
    const float2 sum = unpack2(add2(fma2(m, kZeros2, kOnes2), e));  // unit_exp(M) + e
    return unpack2(add2(m, pack2(log2f(fmaxf(sum.x, 1.0e-20f)), log2f(fmaxf(sum.y, 1.0e-20f)))));
}

// accumulate_lse on two chains at once: chain pair (max, den) and one value each.
__device__ __forceinline__ void accumulate_lse2(uint64_t& mx, uint64_t& dn, uint64_t v) {
    const float2 m = unpack2(mx);
    const float2 x = unpack2(v);
    const float n0 = fmaxf(m.x, x.x);
    const float n1 = fmaxf(m.y, x.y);
    const float2 d = unpack2(sub2(mx, v));
    const float e0 = exp2f(-fabsf(d.x));
    const float e1 = exp2f(-fabsf(d.y));
    const uint64_t n = pack2(n0, n1);
    const float2 u = unpack2(fma2(n, kZeros2, kOnes2));
    const bool k0 = n0 == m.x;
    const bool k1 = n1 == m.y;
    dn = fma2(dn, pack2(k0 ? u.x : e0, k1 ? u.y : e1), pack2(k0 ? e0 : u.x, k1 ? e1 : u.y));
    mx = n;
}

// One tile of a row: 32 KV4 blocks from 64 accumulators (block k = columns 2k,
// 2k + 1: the two pooled representatives). kFull: all 32 blocks are < F. The
// chains are held as pairs (c0, c1) and (c2, c3): mx[0..1], dn[0..1].
// kTma: the row's 16-byte chunks go to its 64-byte staging row (chunk c at
// c ^ ((lane >> 1) & 3), the 64-byte swizzle of the store's tensor map);
// otherwise straight to the row in global memory (rows not 16-byte aligned).
template <bool kFull, bool kTma>
__device__ __forceinline__ void lse_tile(const uint32_t (&acc)[32], int j0, int fine_blocks, half* out,
                                         bool store, uint32_t stage_row, int chunk0, int swz,
                                         uint64_t (&mx)[2], uint64_t (&dn)[2]) {
#pragma unroll
    for (int q = 0; q < 2; ++q) {
        uint32_t packed[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int k = 8 * q + 2 * e;
            const float2 p = pair_lse2(acc[2 * k], acc[2 * k + 1], acc[2 * k + 2], acc[2 * k + 3]);
            // One packed cvt.rn.f16x2 rounds both (the same round-to-nearest as a
            // scalar conversion); the rounded values are what the chains see.
            const half2 h = __floats2half2_rn(p.x, p.y);
            const float2 r = __half22float2(h);
            const int j = j0 + k;  // j % 4 == 2 * (e & 1): chains (0, 1) or (2, 3)
            const int c = e & 1;
            if (kFull) {
                accumulate_lse2(mx[c], dn[c], pack2(r.x, r.y));
            } else {
                float2 m2 = unpack2(mx[c]), d2 = unpack2(dn[c]);
                if (j < fine_blocks) accumulate_lse(m2.x, d2.x, r.x);
                if (j + 1 < fine_blocks) accumulate_lse(m2.y, d2.y, r.y);
                mx[c] = pack2(m2.x, m2.y);
                dn[c] = pack2(d2.x, d2.y);
            }
            packed[e] = *reinterpret_cast<const uint32_t*>(&h);
        }
        if constexpr (kTma) {
            const uint32_t dst = stage_row + (static_cast<uint32_t>((chunk0 + q) ^ swz) << 4);
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};\n" ::"r"(dst), "r"(packed[0]), "r"(packed[1]),
                         "r"(packed[2]), "r"(packed[3])
                         : "memory");
        } else {
            const int jb = j0 + 8 * q;
            if (store && (kFull || jb < fine_blocks)) {
                const half* hv = reinterpret_cast<const half*>(packed);
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    if (kFull || jb + i < fine_blocks) out[jb + i] = hv[i];
            }
        }
    }
}

// grid (ceil(qb * 8 / 128), bh)
__global__ __launch_bounds__(kLseThreads, 3) void lse_kernel(const __grid_constant__ LseMaps maps,
                                                             const LseArgs args) {
    extern __shared__ __align__(1024) unsigned char lse_smem[];
    const uint32_t raw = smem_addr(lse_smem);
    const uint32_t base = (raw + 1023u) & ~1023u;
    unsigned char* base_ptr = lse_smem + (base - raw);
    auto bar = [&](int i) { return base + kLseOffBar + 8u * static_cast<uint32_t>(i); };
    volatile int* abort_flag = reinterpret_cast<volatile int*>(base_ptr + kLseOffAbort);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base_ptr + kLseOffTmemSlot);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int64_t head = blockIdx.y;
    const int64_t row0 = static_cast<int64_t>(blockIdx.x) * kLseRows;
    const int tiles = args.tiles;

    if (threadIdx.x == 0) {
        *abort_flag = 0;
        tc::mbar_init(bar(kLseBarAFull), 1);
        for (int s = 0; s < kLseStages; ++s) {
            tc::mbar_init(bar(kLseBarBFull + s), 1);
            tc::mbar_init(bar(kLseBarBEmpty + s), 1);
        }
        for (int b = 0; b < 2; ++b) {
            tc::mbar_init(bar(kLseBarTFull + b), 1);
            tc::mbar_init(bar(kLseBarTEmpty + b), kLseRows);
        }
        tc::mbar_init(bar(kLseBarDrain), 1);
        tc::mbar_init_fence();
    }
    if (warp == kLseCtlWarp) {
        tc::tmem_alloc(smem_addr(tmem_slot), kLseTmemColumns);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    if (warp == kLseCtlWarp) {
        if (lane == 0) {
            const int64_t key0 = head * static_cast<int64_t>(args.fine_blocks) * kReps;
            auto load = [&](int t) {
                const int st = t % kLseStages;
                tc::mbar_arrive_expect_tx(bar(kLseBarBFull + st), kLseStageBytes);
                const int32_t y = static_cast<int32_t>(key0 + static_cast<int64_t>(t) * kLseTileKeys);
                const uint32_t dst = base + kLseOffB + st * kLseStageBytes;
                tc::tma_load_2d(dst, &maps.keys, 0, y, bar(kLseBarBFull + st));
                tc::tma_load_2d(dst + kLseSlabB, &maps.keys, 64, y, bar(kLseBarBFull + st));
            };
            tc::mbar_arrive_expect_tx(bar(kLseBarAFull), 2 * kLseSlabA);
            const int32_t ay = static_cast<int32_t>(head * args.head_rows + row0);
            tc::tma_load_2d(base + kLseOffA, &maps.centroids, 0, ay, bar(kLseBarAFull));
            tc::tma_load_2d(base + kLseOffA + kLseSlabA, &maps.centroids, 64, ay, bar(kLseBarAFull));
            int issued = 0;
            for (; issued < kLseStages && issued < tiles; ++issued) load(issued);
            bool ok = tc::mbar_wait(bar(kLseBarAFull), 0, abort_flag, kLseWaitLimit);
            for (int t = 0; ok && t < tiles; ++t) {
                const int st = t % kLseStages;
                const int b = t & 1;
                if (!tc::mbar_wait(bar(kLseBarBFull + st), (t / kLseStages) & 1, abort_flag, kLseWaitLimit, true,
                                   tc::kLongWaitHintNs) ||
                    (t >= 2 && !tc::mbar_wait(bar(kLseBarTEmpty + b), ((t >> 1) - 1) & 1, abort_flag,
                                              kLseWaitLimit, true, tc::kLongWaitHintNs))) {
                    ok = false;
                    break;
                }
                tc::fence_after_sync();
                const uint32_t b_base = base + kLseOffB + st * kLseStageBytes;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    // 16 dims per step inside a 64-dim slab: advance the start by 32 bytes.
                    const uint64_t adesc =
                        tc::smem_desc(base + kLseOffA + (j >> 2) * kLseSlabA + (j & 3) * 32, 16, 1024, tc::kSwizzle128B);
                    const uint64_t bdesc =
                        tc::smem_desc(b_base + (j >> 2) * kLseSlabB + (j & 3) * 32, 16, 1024, tc::kSwizzle128B);
                    tc::mma_ss(tmem + b * kLseTileKeys, adesc, bdesc, kLseIdesc, j > 0 ? 1u : 0u);
                }
                tc::mma_commit(bar(kLseBarBEmpty + st));
                tc::mma_commit(bar(kLseBarTFull + b));
                // Refill the stage of tile t - 1 (its MMAs were queued before this
                // tile's, so the tensor pipe stays busy meanwhile).
                if (t >= 1 && issued < tiles) {
                    const int prev = t - 1;
                    if (!tc::mbar_wait(bar(kLseBarBEmpty + prev % kLseStages), (prev / kLseStages) & 1, abort_flag,
                                       kLseWaitLimit, true, tc::kLongWaitHintNs)) {
                        ok = false;
                        break;
                    }
                    load(issued++);
                }
            }
            // Drain: every MMA issued above has completed before TMEM is freed,
            // and every key tile issued has landed before the CTA may exit.
            tc::mma_commit(bar(kLseBarDrain));
            tc::mbar_wait(bar(kLseBarDrain), 0, abort_flag, kLseWaitLimit, false);
            for (int st = 0; st < kLseStages && st < issued; ++st) {
                const int last_use = (issued - 1 - st) / kLseStages;
                tc::mbar_wait(bar(kLseBarBFull + st), last_use & 1, abort_flag, kLseWaitLimit, false);
            }
            tc::mbar_wait(bar(kLseBarAFull), 0, abort_flag, kLseWaitLimit, false);
        }
        __syncwarp();
    } else {
        const int m = threadIdx.x;  // TMEM lane = centroid row row0 + m
        const int64_t row = row0 + m;
        const bool valid = row < args.head_rows;
        const int64_t global_row = head * args.head_rows + row;
        half* out = args.lse + global_row * args.ld;
        const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
        uint64_t mx[2] = {pack2(-FLT_MAX, -FLT_MAX), pack2(-FLT_MAX, -FLT_MAX)};
        uint64_t dn[2] = {0, 0};
        const bool tma_out = args.vector_rows;
        const int swz = (lane >> 1) & 3;
        // TMEM reads overlap the arithmetic: the high half of tile t is read while
        // the low half is evaluated, and the low half of tile t + 1 while the high
        // half of tile t is.
        uint32_t lo[32], hi[32];
        bool ok = tiles > 0 && tc::mbar_wait_warp(bar(kLseBarTFull), 0, abort_flag, kLseWaitLimit,
                                                  tc::kLongWaitHintNs);
        if (ok) {
            tc::fence_after_sync();
            tc::tmem_ld32(lane_base, lo);
            tc::tmem_wait_ld();
            tc::tmem_reg_fence(lo);
        }
        for (int t = 0; ok && t < tiles; ++t) {
            const int b = t & 1;
            tc::tmem_ld32(lane_base + b * kLseTileKeys + 32, hi);
            const int j0 = t * kLseTileBlocks;
            const bool full = j0 + kLseTileBlocks <= args.fine_blocks;
            const uint32_t buf = base + kLseOffOut + warp * kLseOutBufBytes;
            const uint32_t row_addr = buf + lane * kLseStageRowBytes;
            if (tma_out) {
                // This warp's staging buffer: the store issued from it for the
                // previous tile must have finished reading it.
                if (lane == 0) tc::bulk_wait_read<0>();
                __syncwarp();
                if (full)
                    lse_tile<true, true>(lo, j0, args.fine_blocks, out, valid, row_addr, 0, swz, mx, dn);
                else
                    lse_tile<false, true>(lo, j0, args.fine_blocks, out, valid, row_addr, 0, swz, mx, dn);
            } else if (full) {
                lse_tile<true, false>(lo, j0, args.fine_blocks, out, valid, 0, 0, 0, mx, dn);
            } else {
                lse_tile<false, false>(lo, j0, args.fine_blocks, out, valid, 0, 0, 0, mx, dn);
            }
            tc::tmem_wait_ld();
            tc::tmem_reg_fence(hi);
            tc::fence_before_sync();
            tc::mbar_arrive(bar(kLseBarTEmpty + b));
            const bool next = t + 1 < tiles;
            if (next) {
                const int nb = (t + 1) & 1;
                if (tc::mbar_wait_warp(bar(kLseBarTFull + nb), ((t + 1) >> 1) & 1, abort_flag, kLseWaitLimit,
                                       tc::kLongWaitHintNs)) {
                    tc::fence_after_sync();
                    tc::tmem_ld32(lane_base + nb * kLseTileKeys, lo);
                } else {
                    ok = false;
                }
            }
            if (tma_out) {
                if (full)
                    lse_tile<true, true>(hi, j0 + 16, args.fine_blocks, out, valid, row_addr, 2, swz, mx, dn);
                else
                    lse_tile<false, true>(hi, j0 + 16, args.fine_blocks, out, valid, row_addr, 2, swz, mx, dn);
                tc::fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tc::tma_store_3d(&maps.out, buf, j0, static_cast<int32_t>(row0 + warp * 32),
                                     static_cast<int32_t>(head));
                    tc::bulk_commit();
                }
            } else if (full) {
                lse_tile<true, false>(hi, j0 + 16, args.fine_blocks, out, valid, 0, 0, 0, mx, dn);
            } else {
                lse_tile<false, false>(hi, j0 + 16, args.fine_blocks, out, valid, 0, 0, 0, mx, dn);
            }
            if (next && ok) {
                tc::tmem_wait_ld();
                tc::tmem_reg_fence(lo);
            }
        }
        // Every store issued above has completed before the CTA may exit.
        if (tma_out && lane == 0) tc::bulk_wait<0>();
        __syncwarp();
        if (ok && valid) {
            // (c0 + c1) + (c2 + c3), each merge in the reference's operand order.
            const float2 m0 = unpack2(mx[0]), m1 = unpack2(mx[1]);
            const float2 d0 = unpack2(dn[0]), d1 = unpack2(dn[1]);
            float m01 = m0.x, d01 = d0.x;
            combine_lse(m01, d01, m0.y, d0.y);
            float m23 = m1.x, d23 = d1.x;
            combine_lse(m23, d23, m1.y, d1.y);
            combine_lse(m01, d01, m23, d23);
            args.lse_max[global_row] = m01;
            args.lse_den[global_row] = d01;
        }
    }

    tc::fence_before_sync();
    __syncthreads();
    if (warp == kLseCtlWarp) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, kLseTmemColumns);
    }
    if (threadIdx.x == 0 && *abort_flag) raise_device_error(args.error, ABX_ERR_DEVICE_TIMEOUT);
}

// ---------------------------------------------------------------------------
// Population-weighted mixture (csrc/ibcs.cu:495-538): the third pass of IBCS.
// ---------------------------------------------------------------------------

constexpr int kMixThreads = 256;
constexpr int kMixPerThread = 8;  // consecutive KV4 blocks per thread: one 16-byte load per centroid

// grid (rows, ceil(F / 2048)): a CTA covers 2048 consecutive KV4 blocks of one row.
// kVector: every LSE row starts on a 16-byte boundary (ld % 8 == 0, aligned base);
// loads then cover [j0, j0 + 8) and may read the row's padding past F.
template <bool kVector>
__global__ __launch_bounds__(kMixThreads) void mix_kernel(const half* __restrict__ lse, int64_t ld,
                                                          const float* __restrict__ populations,
                                                          const float* __restrict__ lse_max,
                                                          const float* __restrict__ lse_den, int fine_blocks,
                                                          float* __restrict__ scores) {
    __shared__ float row_max[kCentroids];
    __shared__ float row_den[kCentroids];
    __shared__ float row_weight[kCentroids];
    const int64_t row = blockIdx.x;
    if (threadIdx.x < kCentroids) {
        row_max[threadIdx.x] = lse_max[row * kCentroids + threadIdx.x];
        row_den[threadIdx.x] = mix_reciprocal(lse_den[row * kCentroids + threadIdx.x]);  // 1 / den
        row_weight[threadIdx.x] = populations[row * kCentroids + threadIdx.x];
    }
    __syncthreads();
    const int j0 = (blockIdx.y * kMixThreads + threadIdx.x) * kMixPerThread;
    if (j0 >= fine_blocks) return;
    const half* base = lse + row * kCentroids * ld + j0;
    half value[kCentroids][kMixPerThread];
    if constexpr (kVector) {
#pragma unroll
        for (int c = 0; c < kCentroids; ++c)
            *reinterpret_cast<uint4*>(value[c]) = __ldg(reinterpret_cast<const uint4*>(base + c * ld));
    } else {
        const int last = fine_blocks - 1 - j0;
#pragma unroll
        for (int c = 0; c < kCentroids; ++c)
#pragma unroll
            for (int e = 0; e < kMixPerThread; ++e) value[c][e] = base[c * ld + min(e, last)];
    }
    const float total_weight = mix_total_weight(row_weight);
    float out[kMixPerThread];
#pragma unroll
    for (int e = 0; e < kMixPerThread; ++e) {
        half v[kCentroids];
#pragma unroll
        for (int c = 0; c < kCentroids; ++c) v[c] = value[c][e];
        out[e] = mix_score(v, row_max, row_den, row_weight, total_weight);
    }
    float* dst = scores + row * fine_blocks + j0;
    if (j0 + kMixPerThread <= fine_blocks && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
        reinterpret_cast<float4*>(dst)[0] = make_float4(out[0], out[1], out[2], out[3]);
        reinterpret_cast<float4*>(dst)[1] = make_float4(out[4], out[5], out[6], out[7]);
    } else {
#pragma unroll
        for (int e = 0; e < kMixPerThread; ++e)
            if (j0 + e < fine_blocks) dst[e] = out[e];
    }
}

}  // namespace

// ---------------------------------------------------------------------------
// Launchers (validated by the C ABI layer).
// ---------------------------------------------------------------------------

cudaError_t launch_cluster(const bf16* q, int64_t bh, int64_t seq, bf16* centroids, bf16* scaled,
                           float* populations, int32_t* assignments, cudaStream_t stream, const bf16* k,
                           bf16* pooled) {
    if ((k == nullptr) != (pooled == nullptr)) return cudaErrorInvalidValue;
    const int64_t qb = ceil_div(seq, kQueryBlock);
    const int64_t rows = bh * qb;
    cluster_kernel<<<static_cast<unsigned>(rows), 128, 0, stream>>>(
        q, seq, qb, centroids, scaled, populations, assignments, qk_scale_log2(), k, pooled);
    return cudaGetLastError();
}

cudaError_t launch_pool(const bf16* k, int64_t bh, int64_t seq, bf16* pooled, cudaStream_t stream) {
    const int64_t chunks = bh * (seq / kKv4) * 16;
    const unsigned grid = static_cast<unsigned>(ceil_div(chunks, 256));
    pool_kernel<<<grid, 256, 0, stream>>>(k, chunks, pooled);
    return cudaGetLastError();
}

size_t lse_smem_bytes() { return kLseSmemBytes; }

cudaError_t launch_lse(const bf16* scaled, const bf16* pooled, int64_t bh, int64_t qb,
                       int64_t fine_blocks, int64_t ld, half* lse, float* lse_max, float* lse_den,
                       cudaStream_t stream) {
    LseMaps maps{};
    cudaError_t err;
    const int64_t head_rows = qb * kCentroids;
    if ((err = encode_rows(&maps.centroids, scaled, bh * head_rows, kLseRows)) != cudaSuccess) return err;
    if ((err = encode_rows(&maps.keys, pooled, bh * fine_blocks * kReps, kLseTileKeys)) != cudaSuccess) return err;
    const bool vector_rows = ld % 8 == 0 && (reinterpret_cast<uintptr_t>(lse) & 15) == 0;
    if (vector_rows &&
        (err = encode_half_rows3d(&maps.out, lse, fine_blocks, head_rows, bh, ld, kLseTileBlocks, 32)) != cudaSuccess)
        return err;
    LseArgs args{};
    args.head_rows = head_rows;
    args.ld = ld;
    args.fine_blocks = static_cast<int>(fine_blocks);
    args.tiles = static_cast<int>(ceil_div(fine_blocks, kLseTileBlocks));
    args.lse = lse;
    args.lse_max = lse_max;
    args.lse_den = lse_den;
    args.error = device_error_word();
    args.vector_rows = vector_rows;
    err = cudaFuncSetAttribute(lse_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(kLseSmemBytes));
    if (err != cudaSuccess) return err;
    const dim3 grid(static_cast<unsigned>(ceil_div(head_rows, kLseRows)), static_cast<unsigned>(bh));
    lse_kernel<<<grid, kLseThreads, kLseSmemBytes, stream>>>(maps, args);
    return cudaGetLastError();
}

cudaError_t launch_mix(const half* lse, int64_t ld, const float* populations, const float* lse_max,
                       const float* lse_den, int64_t rows, int64_t fine_blocks, float* scores,
                       cudaStream_t stream) {
    const dim3 grid(static_cast<unsigned>(rows),
                    static_cast<unsigned>(ceil_div(fine_blocks, kMixThreads * kMixPerThread)));
    const bool vector = ld % 8 == 0 && (reinterpret_cast<uintptr_t>(lse) & 15) == 0;
    if (vector)
        mix_kernel<true><<<grid, kMixThreads, 0, stream>>>(lse, ld, populations, lse_max, lse_den,
                                                           static_cast<int>(fine_blocks), scores);
    else
        mix_kernel<false><<<grid, kMixThreads, 0, stream>>>(lse, ld, populations, lse_max, lse_den,
                                                            static_cast<int>(fine_blocks), scores);
    return cudaGetLastError();
}

}  // namespace abx
