// SIP (sampling with inclusion-probability weighting) for sm_100a.
//
// One 256-thread CTA per row, as in the reference sip_kernel
// (csrc/sip.cu:33-167). Bit-exact page selection needs the same double
// precision sums in the same order, so the per-thread strides, the chunked
// bucket prefix and the CUB block reduction / scans (same algorithms, same
// 256-thread shape) are kept; the arithmetic expressions are written in the
// same form so that --use_fast_math / fmad contraction produce the same
// instructions.
//
// Scores come from a dense f32 [rows, population] array (the caller's scores
// for `_C.sip`), or, for build_plan, straight from the IBCS centroid LSE rows:
// the kernel evaluates the mixture (mix.cuh, the scorer's own expression) into
// shared memory while loading the row, so the score array is never written.
#include <cub/block/block_reduce.cuh>
#include <cub/block/block_scan.cuh>

#include "common.cuh"
#include "ibcs.cuh"
#include "mix.cuh"
#include "tcgen05.cuh"

namespace abx {
namespace {

struct SumMax {
    double sum, maximum;
};
struct SumMaxOp {
    __device__ __forceinline__ SumMax operator()(SumMax a, SumMax b) const {
        return {a.sum + b.sum, fmax(a.maximum, b.maximum)};
    }
};

struct DenseScores {
    static constexpr bool kDense = true;
    const float* scores;
    int64_t population;
    __device__ __forceinline__ const float* row_ptr(int64_t row) const { return scores + row * population; }
    __device__ __forceinline__ float score(int64_t row, int j) const {
        return scores[row * population + j];
    }
};

// The IBCS centroid LSE rows of build_plan: fp16 [rows, kCentroids, ld]
// (ld % 8 == 0, 16-byte aligned rows) with each (row, centroid)'s max, softmax
// denominator and population.
struct MixedScores {
    static constexpr bool kDense = false;
    const half* lse;
    int64_t ld;
    const float* populations;
    const float* lse_max;
    const float* lse_den;
    // One block's score (the rare clamped-weight path), through the same function.
    __device__ float score(int64_t row, int j) const {
        float mx[kCentroids], den[kCentroids], weight[kCentroids];
        half value[kCentroids];
#pragma unroll
        for (int c = 0; c < kCentroids; ++c) {
            mx[c] = lse_max[row * kCentroids + c];
            den[c] = mix_reciprocal(lse_den[row * kCentroids + c]);
            weight[c] = populations[row * kCentroids + c];
            value[c] = lse[(row * kCentroids + c) * ld + j];
        }
        return mix_score(value, mx, den, weight, mix_total_weight(weight));
    }
};

constexpr uint64_t kSipWaitLimit = 400ull * 1000 * 1000;  // SM cycles (~0.2 s) for the row load

// Smallest float f >= 1e-30f with RN(double(f) * s) >= 1. Multiplication by a
// positive double rounds monotonically, so for every stored mass v (>= 1e-30f,
// never NaN) the reference's test `double(v) * s >= 1` equals `v >= f`. Starts
// from the rounded 1/s and steps one float at a time; false when s is not a
// positive finite double or the steps do not settle.
__device__ bool mark_threshold(double s, float& out) {
    if (!(s > 0.0) || !isfinite(s)) return false;
    float f = static_cast<float>(1.0 / s);
    if (!(f >= 1e-30f)) f = 1e-30f;
    for (int i = 0; i < 64 && f > 1e-30f; ++i) {
        const float below = __int_as_float(__float_as_int(f) - 1);
        if (static_cast<double>(below) * s >= 1.) f = below;
        else break;
    }
    for (int i = 0; i < 64; ++i) {
        if (static_cast<double>(f) * s >= 1.) {
            out = f;
            return true;
        }
        if (f == INFINITY) return false;
        f = __int_as_float(__float_as_int(f) + 1);
    }
    return false;
}

using Reduce = cub::BlockReduce<SumMax, kSipThreads>;
using CountScan = cub::BlockScan<int, kSipThreads>;
using MassScan = cub::BlockScan<double, kSipThreads>;
union Scratch {
    Reduce::TempStorage reduce;
    CountScan::TempStorage count;
    MassScan::TempStorage mass;
};

// Dynamic shared memory: the bucket prefix (doubles) then the masses (floats,
// starting on a 16-byte boundary for the float4 chunk sweeps).
// CUB's temporaries live at the start of the prefix region: every block
// reduction and scan finishes before the first prefix entry is written, and
// keeping them out of static shared memory lets two rows share an SM at the
// Wan2.1 shape (F = 18,900).
__host__ __device__ constexpr size_t sip_prefix_region(int64_t population) {
    const size_t prefix = static_cast<size_t>((population + kSipBucket - 1) / kSipBucket + 1) * sizeof(double);
    const size_t region = prefix > sizeof(Scratch) ? prefix : sizeof(Scratch);
    return (region + 15) / 16 * 16;
}

constexpr int kLoadUnroll = 8;  // score loads in flight per thread
// Rows ahead whose LSE rows a CTA prefetches into L2 (build_plan's form). Any
// distance from 0 (the CTA's own row) to 32 measured the same at the Wan2.1
// and HunyuanVideo shapes (SIP 8.0 -> 7.5 ms and 8.4 -> 7.6 ms per layer);
// one or two waves of resident CTAs ahead (148 or 296 rows) measured slower
// than no prefetch.
constexpr int kSipPrefetchAhead = 8;
constexpr int kMarkUnroll = 4;  // masses per thread per step of the marking sweep
constexpr int kDrawGroup = 4;   // draws per thread searched in lockstep

// mass_j = v_j * scale for a residual unit (v_j > 0), 0 for a certain one; the
// expression has the reference's shape (csrc/sip.cu:127,140), so the multiply
// is not fused into the running sum.
#define SIP_MASS(f, s) ((f) > 0.f ? static_cast<double>(f) * (s) : 0.)

template <class Source>
__global__ __launch_bounds__(kSipThreads) void sip_kernel(Source source, const float* __restrict__ offsets,
                                                          int32_t* __restrict__ sampled,
                                                          float* __restrict__ weights, int population,
                                                          int samples, int prefetch_rows,
                                                          int* device_error_word_ptr) {
    extern __shared__ __align__(16) double prefix[];
    Scratch& scratch = *reinterpret_cast<Scratch*>(prefix);
    __shared__ double scale;
    __shared__ int certain;
    __shared__ int added;
    __shared__ int last_residual;
    __shared__ int marking;
    __shared__ int threshold_ok;
    __shared__ float threshold;

    const int buckets = (population + kSipBucket - 1) / kSipBucket;
    float* values = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(prefix) + sip_prefix_region(population));
    const int tid = threadIdx.x;
    const int64_t row = blockIdx.x;
    int32_t* out_ids = sampled + row * samples;
    float* out_logs = weights + row * samples;

    // v_j = max(score_j, 1e-30f) (csrc/sip.cu:58-59), fused with the first
    // iteration's partial sums. Every v_j is positive and its double is above
    // 1e-30, so the reference's `v > 0` test and fmax(v, 1e-30) are identities
    // here; the sums visit j = tid, tid + 256, ... in order as there.
    // The row's scores land in shared memory by one bulk copy (the whole row in
    // flight at once); a ragged tail (or a row not 16-byte aligned) is loaded by
    // the threads. Then v_j = max(score_j, 1e-30f) (csrc/sip.cu:58-59), fused
    // with the first iteration's partial sums. Every v_j is positive and its
    // double is above 1e-30, so the reference's `v > 0` test and fmax(v, 1e-30)
    // are identities here; the sums visit j = tid, tid + 256, ... in order as
    // there, and the max of the doubles is the double of the float max.
    if constexpr (Source::kDense) {
        __shared__ __align__(8) uint64_t load_bar;
        __shared__ int load_abort;
        const float* src = source.row_ptr(row);
        const int bulk = (reinterpret_cast<uintptr_t>(src) & 15) == 0 ? (population & ~3) : 0;
        if (tid == 0) {
            load_abort = 0;
            tc::mbar_init(smem_addr(&load_bar), 1);
            tc::mbar_init_fence();
            if (bulk > 0) {
                tc::mbar_arrive_expect_tx(smem_addr(&load_bar), static_cast<uint32_t>(bulk) * 4u);
                tc::bulk_load(smem_addr(values), src, static_cast<uint32_t>(bulk) * 4u, smem_addr(&load_bar));
            } else {
                tc::mbar_arrive(smem_addr(&load_bar));
            }
        }
        for (int j = bulk + tid; j < population; j += kSipThreads) values[j] = __ldg(src + j);
        __syncthreads();
        if (!tc::mbar_wait(smem_addr(&load_bar), 0, &load_abort, kSipWaitLimit))
            raise_device_error(device_error_word_ptr, ABX_ERR_DEVICE_TIMEOUT);
    } else {
        // Mixture scores of this row, 8 consecutive blocks per step (one 16-byte
        // load per centroid; rows are padded to ld, so the last step stays inside).
        __shared__ float mix_max[kCentroids], mix_den[kCentroids], mix_weight[kCentroids];
        // The LSE rows of the row `prefetch_rows` ahead in launch order go to L2
        // by one bulk prefetch per centroid row (the whole 300 KB at once, where
        // the fill below keeps 64 KB in flight), so that its CTA, starting a
        // little later, fills mostly from L2.
        const int64_t ahead = row + prefetch_rows;
        if (prefetch_rows > 0 && ahead < gridDim.x && tid < kCentroids)
            tc::prefetch_l2(source.lse + (ahead * kCentroids + tid) * source.ld,
                            static_cast<uint32_t>(source.ld * sizeof(half)));
        if (tid < kCentroids) {
            mix_max[tid] = source.lse_max[row * kCentroids + tid];
            mix_den[tid] = mix_reciprocal(source.lse_den[row * kCentroids + tid]);  // 1 / den
            mix_weight[tid] = source.populations[row * kCentroids + tid];
        }
        __syncthreads();
        const float total_weight = mix_total_weight(mix_weight);
        const half* base = source.lse + row * kCentroids * source.ld;
        const int groups = (population + 7) / 8;
        for (int g = tid; g < groups; g += 2 * kSipThreads) {
            // two groups per pass: 16 loads in flight per thread
            uint4 raw[2][kCentroids];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int gg = min(g + h * kSipThreads, groups - 1);
#pragma unroll
                for (int c = 0; c < kCentroids; ++c)
                    raw[h][c] = __ldg(reinterpret_cast<const uint4*>(base + c * source.ld + 8 * gg));
            }
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int j0 = 8 * (g + h * kSipThreads);
                if (j0 >= population) break;
                float out[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    half v[kCentroids];
#pragma unroll
                    for (int c = 0; c < kCentroids; ++c) v[c] = reinterpret_cast<const half*>(&raw[h][c])[e];
                    out[e] = mix_score(v, mix_max, mix_den, mix_weight, total_weight);
                }
                if (j0 + 8 <= population) {
                    reinterpret_cast<float4*>(values + j0)[0] = make_float4(out[0], out[1], out[2], out[3]);
                    reinterpret_cast<float4*>(values + j0)[1] = make_float4(out[4], out[5], out[6], out[7]);
                } else {
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        if (j0 + e < population) values[j0 + e] = out[e];
                }
            }
        }
        __syncthreads();
    }
    double local_sum = 0.;
    double local_max = 0.;
    {
        float fmax_kept = 0.f;
        int j = tid;
        for (; j + (kLoadUnroll - 1) * kSipThreads < population; j += kLoadUnroll * kSipThreads) {
            float f[kLoadUnroll];
#pragma unroll
            for (int u = 0; u < kLoadUnroll; ++u) f[u] = fmaxf(values[j + u * kSipThreads], 1e-30f);
#pragma unroll
            for (int u = 0; u < kLoadUnroll; ++u) {
                values[j + u * kSipThreads] = f[u];
                local_sum += static_cast<double>(f[u]);
                fmax_kept = fmaxf(fmax_kept, f[u]);
            }
        }
        for (; j < population; j += kSipThreads) {
            const float f = fmaxf(values[j], 1e-30f);
            values[j] = f;
            local_sum += static_cast<double>(f);
            fmax_kept = fmaxf(fmax_kept, f);
        }
        local_max = static_cast<double>(fmax_kept);
    }
    if (tid == 0) certain = 0;

    // Iterative certainty: mark every unit whose inclusion probability reaches 1
    // (negated in place) until the residual budget is stable (csrc/sip.cu:62-96).
    // The reference re-sums the uncertain masses after each marking pass; the
    // units a marking pass leaves unmarked are exactly the terms of that sum,
    // visited in the same per-thread order, so the marking pass accumulates the
    // next partial sums itself (adding +0.0 for a skipped unit, which leaves a
    // non-negative sum unchanged) and each iteration is one pass instead of two.
    do {
        const SumMax total = Reduce(scratch.reduce).Reduce(SumMax{local_sum, local_max}, SumMaxOp{});
        if (tid == 0) {
            scale = (samples - certain) / total.sum;
            added = 0;
            marking = total.maximum * scale >= 1.0;
            threshold_ok = marking && mark_threshold(scale, threshold);
        }
        __syncthreads();
        if (marking && threshold_ok) {
            // mark <=> v >= threshold (exactly the reference's double test)
            const float fs = threshold;
            int count = 0;
            local_sum = 0.;
            float fmax_kept = 0.f;
            int j = tid;
            for (; j + (kMarkUnroll - 1) * kSipThreads < population; j += kMarkUnroll * kSipThreads) {
                float f[kMarkUnroll];
#pragma unroll
                for (int u = 0; u < kMarkUnroll; ++u) f[u] = values[j + u * kSipThreads];
#pragma unroll
                for (int u = 0; u < kMarkUnroll; ++u) {
                    const bool live = f[u] > 0.f;
                    const bool mark = live && f[u] >= fs;
                    if (mark) values[j + u * kSipThreads] = -f[u];
                    count += mark;
                    if (live && !mark) {
                        local_sum += static_cast<double>(f[u]);
                        fmax_kept = fmaxf(fmax_kept, f[u]);
                    }
                }
            }
            for (; j < population; j += kSipThreads) {
                const float f = values[j];
                const bool live = f > 0.f;
                const bool mark = live && f >= fs;
                if (mark) values[j] = -f;
                count += mark;
                if (live && !mark) {
                    local_sum += static_cast<double>(f);
                    fmax_kept = fmaxf(fmax_kept, f);
                }
            }
            local_max = static_cast<double>(fmax_kept);
            atomicAdd(&added, count);
        } else if (marking) {
            const double s = scale;
            int count = 0;
            local_sum = 0.;
            local_max = 0.;
            int j = tid;
            for (; j + (kMarkUnroll - 1) * kSipThreads < population; j += kMarkUnroll * kSipThreads) {
                float f[kMarkUnroll];
#pragma unroll
                for (int u = 0; u < kMarkUnroll; ++u) f[u] = values[j + u * kSipThreads];
#pragma unroll
                for (int u = 0; u < kMarkUnroll; ++u) {
                    const bool live = f[u] > 0.f;
                    const double value = static_cast<double>(f[u]);
                    const bool mark = live && value * s >= 1.;
                    if (mark) values[j + u * kSipThreads] = -f[u];
                    count += mark;
                    const double kept = live && !mark ? value : 0.;
                    local_sum += kept;
                    local_max = fmax(local_max, kept);
                }
            }
            for (; j < population; j += kSipThreads) {
                const float f = values[j];
                const bool live = f > 0.f;
                const double value = static_cast<double>(f);
                const bool mark = live && value * s >= 1.;
                if (mark) values[j] = -f;
                count += mark;
                const double kept = live && !mark ? value : 0.;
                local_sum += kept;
                local_max = fmax(local_max, kept);
            }
            atomicAdd(&added, count);
        }
        __syncthreads();
        if (tid == 0) certain += added;
        __syncthreads();
    } while (added != 0);

    // Contiguous chunks of whole buckets per thread (csrc/sip.cu:98-106). The
    // chunk length is a multiple of 4 floats, so a chunk is a run of float4s
    // (conflict-free across a quarter warp) plus, in the last chunk, a tail.
    const int chunk = ((buckets + kSipThreads - 1) / kSipThreads) * kSipBucket;
    const int begin = tid * chunk;
    const int end = min(begin + chunk, population);
    const int quads = end > begin ? (end - begin) / 4 : 0;
    const int tail = begin + 4 * quads;
    const float4* chunk4 = reinterpret_cast<const float4*>(values + begin);
    if (tid == 0) {
        int last = population - 1;
        while (last >= 0 && values[last] <= 0.) --last;
        last_residual = last;
    }
    __syncthreads();
    const double s = scale;

    // Certain units first, ascending, log-weight 0 (csrc/sip.cu:108-124).
    if (certain != 0) {
        int count = 0;
        for (int i = 0; i < quads; ++i) {
            const float4 f = chunk4[i];
            count += (f.x < 0.f) + (f.y < 0.f) + (f.z < 0.f) + (f.w < 0.f);
        }
        for (int j = tail; j < end; ++j) count += values[j] < 0.f;
        int rank = 0;
        CountScan(scratch.count).InclusiveSum(count, rank);
        int slot = rank - count;
        for (int i = 0; i < quads; ++i) {
            const float4 f = chunk4[i];
            const int j = begin + 4 * i;
            if (f.x < 0.f) { out_ids[slot] = j; out_logs[slot++] = 0.f; }
            if (f.y < 0.f) { out_ids[slot] = j + 1; out_logs[slot++] = 0.f; }
            if (f.z < 0.f) { out_ids[slot] = j + 2; out_logs[slot++] = 0.f; }
            if (f.w < 0.f) { out_ids[slot] = j + 3; out_logs[slot++] = 0.f; }
        }
        for (int j = tail; j < end; ++j) {
            if (values[j] < 0.f) {
                out_ids[slot] = j;
                out_logs[slot++] = 0.f;
            }
        }
        __syncthreads();
    }

    // Bucketed prefix of the residual masses (csrc/sip.cu:126-142).
    double chunk_mass = 0.;
    for (int i = 0; i < quads; ++i) {
        const float4 f = chunk4[i];
        chunk_mass += SIP_MASS(f.x, s);
        chunk_mass += SIP_MASS(f.y, s);
        chunk_mass += SIP_MASS(f.z, s);
        chunk_mass += SIP_MASS(f.w, s);
    }
    for (int j = tail; j < end; ++j) chunk_mass += SIP_MASS(values[j], s);
    double cumulative = 0.;
    MassScan(scratch.mass).ExclusiveSum(chunk_mass, cumulative);
    __syncthreads();  // the scan's temporaries overlap the prefix written below
    const int residuals = samples - certain;
    const int last = last_residual;
    if (tid == 0) prefix[buckets] = residuals;
    for (int i = 0; i < quads; ++i) {
        const float4 f = chunk4[i];
        const int j = begin + 4 * i;  // a bucket start
        prefix[j / kSipBucket] = j > last ? residuals : cumulative;
        cumulative += SIP_MASS(f.x, s);
        cumulative += SIP_MASS(f.y, s);
        cumulative += SIP_MASS(f.z, s);
        cumulative += SIP_MASS(f.w, s);
    }
    for (int j = tail; j < end; ++j) {
        if (j % kSipBucket == 0) prefix[j / kSipBucket] = j > last ? residuals : cumulative;
        cumulative += SIP_MASS(values[j], s);
    }
    __syncthreads();

    // Systematic draws at u + k: bucket search, then a walk of at most four
    // masses; the last residual closes roundoff escapes (csrc/sip.cu:144-166).
    // A thread's draws (slots tid, tid + 256, ...) are searched in lockstep
    // groups for instruction-level parallelism; each draw's steps are the
    // reference's.
    const double offset = static_cast<double>(offsets[row]);
    for (int first = tid; first < residuals; first += kDrawGroup * kSipThreads) {
        double threshold[kDrawGroup];
        int lower[kDrawGroup], upper[kDrawGroup];
        bool busy = false;
#pragma unroll
        for (int k = 0; k < kDrawGroup; ++k) {
            const int slot = first + k * kSipThreads;
            threshold[k] = offset + slot;
            lower[k] = 0;
            upper[k] = slot < residuals ? buckets : 0;
            busy |= lower[k] < upper[k];
        }
        while (busy) {
            busy = false;
#pragma unroll
            for (int k = 0; k < kDrawGroup; ++k) {
                if (lower[k] < upper[k]) {
                    const int middle = (lower[k] + upper[k] + 1) / 2;
                    if (prefix[middle] <= threshold[k]) lower[k] = middle;
                    else upper[k] = middle - 1;
                    busy |= lower[k] < upper[k];
                }
            }
        }
        int selected[kDrawGroup];
#pragma unroll
        for (int k = 0; k < kDrawGroup; ++k) {
            const int bucket = min(lower[k], buckets - 1);
            double mass = prefix[bucket];
            selected[k] = last;
            const int stop = min((bucket + 1) * kSipBucket, population);
            for (int j = bucket * kSipBucket; j < stop; ++j) {
                if (values[j] <= 0.f) continue;
                selected[k] = j;
                mass += static_cast<double>(values[j]) * scale;
                if (mass > threshold[k]) break;
            }
        }
#pragma unroll
        for (int k = 0; k < kDrawGroup; ++k) {
            const int slot = first + k * kSipThreads;
            if (slot >= residuals) break;
            // The weight uses the unclamped score; `values` holds max(score, 1e-30f),
            // which equals it unless the clamp was active.
            const float kept = values[selected[k]];
            const float raw = kept == 1e-30f ? source.score(row, selected[k]) : kept;
            out_ids[certain + slot] = selected[k];
            out_logs[certain + slot] = static_cast<float>(-log2(fmax(static_cast<double>(raw), 1e-30) * scale));
        }
    }
}

#undef SIP_MASS

}  // namespace

size_t sip_smem_bytes(int64_t population) {
    return sip_prefix_region(population) + static_cast<size_t>(population) * sizeof(float);
}

int sip_smem_limit() {
    int device = 0, optin = 0;
    cudaGetDevice(&device);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
    cudaFuncAttributes attr{};
    cudaFuncGetAttributes(&attr, sip_kernel<DenseScores>);
    return optin - static_cast<int>(attr.sharedSizeBytes);
}

template <class Source>
static cudaError_t launch_sip_impl(const Source& source, const float* offsets, int64_t rows,
                                   int64_t population, int32_t* ids, float* log_weights,
                                   int64_t samples, cudaStream_t stream) {
    const size_t smem = sip_smem_bytes(population);
    cudaError_t err = cudaFuncSetAttribute(sip_kernel<Source>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem));
    if (err != cudaSuccess) return err;
    const int prefetch_rows = Source::kDense ? 0 : kSipPrefetchAhead;
    sip_kernel<Source><<<static_cast<unsigned>(rows), kSipThreads, smem, stream>>>(
        source, offsets, ids, log_weights, static_cast<int>(population), static_cast<int>(samples),
        prefetch_rows, device_error_word());
    return cudaGetLastError();
}

cudaError_t launch_sip(const float* scores, const float* offsets, int64_t rows, int64_t population,
                       int32_t* ids, float* log_weights, int64_t samples, cudaStream_t stream) {
    DenseScores source{scores, population};
    return launch_sip_impl(source, offsets, rows, population, ids, log_weights, samples, stream);
}

cudaError_t launch_sip_mixed(const half* lse, int64_t ld, const float* populations, const float* lse_max,
                             const float* lse_den, const float* offsets, int64_t rows, int64_t population,
                             int32_t* ids, float* log_weights, int64_t samples, cudaStream_t stream) {
    if (ld % 8 != 0 || ld < population || (reinterpret_cast<uintptr_t>(lse) & 15) != 0) return cudaErrorInvalidValue;
    const MixedScores source{lse, ld, populations, lse_max, lse_den};
    return launch_sip_impl(source, offsets, rows, population, ids, log_weights, samples, stream);
}

}  // namespace abx
