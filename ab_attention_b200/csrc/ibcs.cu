// IBCS (intra-block clustering selector) for sm_100a.
//
// Stages, each reproducing the float arithmetic of the reference kernel it
// replaces (rounding points, reduction orders and `--use_fast_math` semantics
// are kept identical so the downstream page selection is bit-exact):
//   cluster_kernel  <- cluster_queries_kernel  csrc/ibcs.cu:106-238
//   pool_kernel     <- pool_keys_kernel        csrc/ibcs.cu:244-266
//   lse_kernel      <- ibcs_lse_kernel         csrc/ibcs.cu:370-489
//   mix_kernel      <- ibcs_scores_kernel      csrc/ibcs.cu:495-538
//
// What differs is the work decomposition: one thread per query for the
// clustering distances (the 32-lane partial sums and the xor-butterfly are
// evaluated inside the thread, in the reference's order), 16-byte vector
// loads and stores throughout, 128 centroid rows per CTA in the scorer with a
// 64-block key tile, and a padded fp16 LSE scratch written in 128-byte rows.
// This file must be compiled with --use_fast_math (as csrc/ibcs.cu is).
#include "common.cuh"
#include "ibcs.cuh"

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
__device__ __forceinline__ float block_distance(const uint4* tile, int i, const float* center) {
    float part[32];
#pragma unroll
    for (int p = 0; p < 32; ++p) part[p] = 0.0f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const uint4 raw = tile[chunk_slot(i, 4 * k + c)];
            const bf16* vals = reinterpret_cast<const bf16*>(&raw);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const int p = c * 8 + e;
                const float delta = __bfloat162float(vals[e]) - center[32 * k + p];
                part[p] += delta * delta;
            }
        }
    }
#pragma unroll
    for (int width = 16; width > 0; width >>= 1) {
#pragma unroll
        for (int p = 0; p < width; ++p) part[p] = part[p] + part[p + width];
    }
    return part[0];
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

__global__ __launch_bounds__(128) void cluster_kernel(
    const bf16* __restrict__ q, int64_t seq, int64_t qb, bf16* __restrict__ centroids,
    bf16* __restrict__ scaled, float* __restrict__ populations,
    int32_t* __restrict__ assignments, float kappa) {
    __shared__ uint4 tile[128 * 16];
    __shared__ float center[kHeadDim];
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
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.0f;
    for (int i = 0; i < n; ++i) {
        if (members[i] == cluster) {
            const uint4 raw = tile[chunk_slot(i, chunk)];
            const bf16* vals = reinterpret_cast<const bf16*>(&raw);
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[e] += __bfloat162float(vals[e]);
        }
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
    const int64_t block = idx >> 4;
    const int chunk = static_cast<int>(idx & 15);
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

// ---------------------------------------------------------------------------
// Centroid x pooled-key scoring with per-centroid normalizers.
// ---------------------------------------------------------------------------

constexpr int kLseWarps = 8;
constexpr int kLseThreads = kLseWarps * 32;
constexpr int kLseRowsPerCta = 16 * kLseWarps;  // centroid rows per CTA
constexpr int kLseTileBlocks = 64;              // KV4 blocks per key tile
constexpr int kLseTileKeys = kLseTileBlocks * kReps;
constexpr int kLseStageChunks = kLseTileKeys * 16;  // 16-byte chunks per stage (32 KB)
constexpr int kLseStagingStride = kLseTileBlocks + 8;  // padded row (144 B) avoids bank conflicts
constexpr int kLseStagingHalfs = 16 * kLseStagingStride;  // per-warp LSE staging tile

__device__ __forceinline__ void accumulate_lse(float& maximum, float& denominator, float value) {
    const float next_max = fmaxf(maximum, value);
    denominator = denominator * exp2f(maximum - next_max) + exp2f(value - next_max);
    maximum = next_max;
}

__device__ __forceinline__ float pair_lse(float left, float right) {
    const float maximum = fmaxf(left, right);
    return maximum + log2f(fmaxf(exp2f(left - maximum) + exp2f(right - maximum), 1.0e-20f));
}

__device__ __forceinline__ void combine_lse(float& maximum, float& denominator, float other_max,
                                            float other_den) {
    const float next = fmaxf(maximum, other_max);
    denominator = denominator * exp2f(maximum - next) + other_den * exp2f(other_max - next);
    maximum = next;
}

__device__ __forceinline__ void stage_key_tile(const bf16* __restrict__ pooled_head, uint4* stage,
                                               int tile, int fine_blocks) {
    // 128 pooled rows x 16 chunks; rows past the end are clamped to the last block
    // (their results are never stored, csrc/ibcs.cu:318,355).
    const int last_key = fine_blocks * kReps - 1;
#pragma unroll
    for (int it = 0; it < kLseStageChunks / kLseThreads; ++it) {
        const int idx = it * kLseThreads + threadIdx.x;
        const int key = idx >> 4;
        const int c = idx & 15;
        int src_key = tile * kLseTileKeys + key;
        if (src_key > last_key) src_key = (last_key & ~1) + (key & 1);
        cp_async_16(stage + chunk_slot(key, c), pooled_head + static_cast<int64_t>(src_key) * kHeadDim + c * 8);
    }
}

__global__ __launch_bounds__(kLseThreads) void lse_kernel(
    const bf16* __restrict__ scaled, const bf16* __restrict__ pooled, int64_t qb, int fine_blocks,
    int64_t ld, half* __restrict__ lse, float* __restrict__ lse_max, float* __restrict__ lse_den) {
    extern __shared__ __align__(128) uint4 smem[];
    uint4* stage0 = smem;
    uint4* stage1 = smem + kLseStageChunks;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    half* staging = reinterpret_cast<half*>(smem + 2 * kLseStageChunks) + warp * kLseStagingHalfs;
    const int64_t head = blockIdx.y;
    const int64_t head_rows = qb * kCentroids;
    const int64_t m0 = static_cast<int64_t>(blockIdx.x) * kLseRowsPerCta + warp * 16;
    const int g = lane >> 2;
    const int t = lane & 3;
    const bf16* pooled_head = pooled + head * static_cast<int64_t>(fine_blocks) * kReps * kHeadDim;

    stage_key_tile(pooled_head, stage0, 0, fine_blocks);
    cp_async_commit();

    // A fragments: 16 scaled-centroid rows x 128 dims; rows past the head are zero.
    uint32_t a[8][4];
    {
        const bf16* base = scaled + head * head_rows * kHeadDim;
        const int64_t lo = m0 + g, hi = m0 + g + 8;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
            const int col = 16 * kk + 2 * t;
            a[kk][0] = lo < head_rows ? *reinterpret_cast<const uint32_t*>(base + lo * kHeadDim + col) : 0u;
            a[kk][1] = hi < head_rows ? *reinterpret_cast<const uint32_t*>(base + hi * kHeadDim + col) : 0u;
            a[kk][2] = lo < head_rows ? *reinterpret_cast<const uint32_t*>(base + lo * kHeadDim + col + 8) : 0u;
            a[kk][3] = hi < head_rows ? *reinterpret_cast<const uint32_t*>(base + hi * kHeadDim + col + 8) : 0u;
        }
    }

    // Running normalizers for rows g and g+8, lane class t = KV4 block index mod 4.
    float maximum[2] = {-FLT_MAX, -FLT_MAX};
    float denominator[2] = {0.0f, 0.0f};
    const int tiles = static_cast<int>(ceil_div(fine_blocks, kLseTileBlocks));
    const bool vec_store = (ld % 8) == 0;

    for (int tile = 0; tile < tiles; ++tile) {
        uint4* current = (tile & 1) ? stage1 : stage0;
        uint4* upcoming = (tile & 1) ? stage0 : stage1;
        cp_async_wait<0>();
        __syncthreads();
        if (tile + 1 < tiles) {
            stage_key_tile(pooled_head, upcoming, tile + 1, fine_blocks);
            cp_async_commit();
        }
        const uint32_t stage_base = smem_addr(current);
#pragma unroll 2
        for (int grp = 0; grp < kLseTileKeys / 16; ++grp) {
            float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
            const int key = grp * 16 + (lane >> 4) * 8 + (lane & 7);
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
                const int c = 2 * kk + ((lane >> 3) & 1);
                uint32_t b[4];
                ldmatrix_x4(b, stage_base + chunk_slot(key, c) * 16);
                mma_bf16_16816(acc[0], a[kk], b[0], b[1]);
                mma_bf16_16816(acc[1], a[kk], b[2], b[3]);
            }
            // Lane (g, t) holds rows g / g+8 of KV4 blocks 8*grp + t and 8*grp + t + 4.
#pragma unroll
            for (int r = 0; r < 2; ++r) {
#pragma unroll
                for (int nt = 0; nt < 2; ++nt) {
                    const int local = grp * 8 + nt * 4 + t;
                    const int block = tile * kLseTileBlocks + local;
                    const half stored = __float2half_rn(
                        pair_lse(acc[nt][2 * r] + 1.0f, acc[nt][2 * r + 1] + 1.0f));
                    staging[(g + 8 * r) * kLseStagingStride + local] = stored;
                    if (block < fine_blocks) accumulate_lse(maximum[r], denominator[r], __half2float(stored));
                }
            }
        }
        __syncwarp();
        // Write the warp's 16 x 64 fp16 tile: 16 rows x 8 chunks of 16 bytes.
        const int block0 = tile * kLseTileBlocks;
#pragma unroll
        for (int it = 0; it < 4; ++it) {
            const int idx = it * 32 + lane;
            const int rr = idx >> 3;
            const int c = idx & 7;
            const int64_t m = m0 + rr;
            if (m >= head_rows) continue;
            half* dst = lse + (head * head_rows + m) * ld + block0 + c * 8;
            const half* s = staging + rr * kLseStagingStride + c * 8;
            const int avail = fine_blocks - (block0 + c * 8);
            if (vec_store && avail >= 8) {
                *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(s);
            } else {
                for (int e = 0; e < 8 && e < avail; ++e) dst[e] = s[e];
            }
        }
        __syncwarp();
    }

    // Merge the four lane classes: (c0+c1)+(c2+c3) (csrc/ibcs.cu:468-477).
#pragma unroll
    for (int mask = 1; mask <= 2; mask <<= 1) {
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            combine_lse(maximum[r], denominator[r], __shfl_xor_sync(0xffffffffu, maximum[r], mask),
                        __shfl_xor_sync(0xffffffffu, denominator[r], mask));
        }
    }
    if (t == 0) {
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int64_t m = m0 + g + 8 * r;
            if (m < head_rows) {
                lse_max[head * head_rows + m] = maximum[r];
                lse_den[head * head_rows + m] = denominator[r];
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Population-weighted mixture (standalone; build_plan fuses it into SIP).
// ---------------------------------------------------------------------------

constexpr int kMixThreads = 256;
constexpr int kMixPerThread = 4;  // scores per thread; all 32 fp16 loads are issued before the math

// grid (rows, ceil(F / (256 * 4))): a CTA covers 1024 consecutive KV4 blocks of one row.
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
        row_den[threadIdx.x] = lse_den[row * kCentroids + threadIdx.x];
        row_weight[threadIdx.x] = populations[row * kCentroids + threadIdx.x];
    }
    __syncthreads();
    float total_weight = 0.0f;
#pragma unroll
    for (int c = 0; c < kCentroids; ++c) total_weight += row_weight[c];
    const int j0 = blockIdx.y * (kMixThreads * kMixPerThread) + threadIdx.x;
    const half* base = lse + row * kCentroids * ld;
    half value[kMixPerThread][kCentroids];
#pragma unroll
    for (int u = 0; u < kMixPerThread; ++u) {
        const int j = min(j0 + u * kMixThreads, fine_blocks - 1);
#pragma unroll
        for (int c = 0; c < kCentroids; ++c) value[u][c] = base[c * ld + j];
    }
#pragma unroll
    for (int u = 0; u < kMixPerThread; ++u) {
        const int j = j0 + u * kMixThreads;
        float score = 0.0f;
#pragma unroll
        for (int c = 0; c < kCentroids; ++c) {
            const float probability = exp2f(__half2float(value[u][c]) - row_max[c]) / row_den[c];
            score += row_weight[c] * probability;
        }
        if (j < fine_blocks) scores[row * fine_blocks + j] = score / total_weight;
    }
}

}  // namespace

// ---------------------------------------------------------------------------
// Launchers (validated by the C ABI layer).
// ---------------------------------------------------------------------------

cudaError_t launch_cluster(const bf16* q, int64_t bh, int64_t seq, bf16* centroids, bf16* scaled,
                           float* populations, int32_t* assignments, cudaStream_t stream) {
    const int64_t qb = ceil_div(seq, kQueryBlock);
    const int64_t rows = bh * qb;
    cluster_kernel<<<static_cast<unsigned>(rows), 128, 0, stream>>>(
        q, seq, qb, centroids, scaled, populations, assignments, qk_scale_log2());
    return cudaGetLastError();
}

cudaError_t launch_pool(const bf16* k, int64_t bh, int64_t seq, bf16* pooled, cudaStream_t stream) {
    const int64_t chunks = bh * (seq / kKv4) * 16;
    const unsigned grid = static_cast<unsigned>(ceil_div(chunks, 256));
    pool_kernel<<<grid, 256, 0, stream>>>(k, chunks, pooled);
    return cudaGetLastError();
}

size_t lse_smem_bytes() {
    return 2 * kLseStageChunks * sizeof(uint4) + kLseWarps * kLseStagingHalfs * sizeof(half);
}

cudaError_t launch_lse(const bf16* scaled, const bf16* pooled, int64_t bh, int64_t qb,
                       int64_t fine_blocks, int64_t ld, half* lse, float* lse_max, float* lse_den,
                       cudaStream_t stream) {
    const size_t smem = lse_smem_bytes();
    cudaError_t err = cudaFuncSetAttribute(lse_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem));
    if (err != cudaSuccess) return err;
    const dim3 grid(static_cast<unsigned>(ceil_div(qb * kCentroids, kLseRowsPerCta)),
                    static_cast<unsigned>(bh));
    lse_kernel<<<grid, kLseThreads, smem, stream>>>(scaled, pooled, qb, static_cast<int>(fine_blocks),
                                                    ld, lse, lse_max, lse_den);
    return cudaGetLastError();
}

cudaError_t launch_mix(const half* lse, int64_t ld, const float* populations, const float* lse_max,
                       const float* lse_den, int64_t rows, int64_t fine_blocks, float* scores,
                       cudaStream_t stream) {
    const dim3 grid(static_cast<unsigned>(rows),
                    static_cast<unsigned>(ceil_div(fine_blocks, kMixThreads * kMixPerThread)));
    mix_kernel<<<grid, kMixThreads, 0, stream>>>(lse, ld, populations, lse_max, lse_den,
                                                 static_cast<int>(fine_blocks), scores);
    return cudaGetLastError();
}

}  // namespace abx
