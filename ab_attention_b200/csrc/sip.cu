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
// Two value sources feed it:
//   DenseScores : scores f32 [rows, population] (replaces `_C.sip`)
//   MixedScores : the IBCS population-weighted mixture (csrc/ibcs.cu:495-538)
//                 evaluated in the prologue straight from the fp16 LSE scratch,
//                 so the f32 score array never exists in HBM (build_plan path).
#include <cub/block/block_reduce.cuh>
#include <cub/block/block_scan.cuh>

#include "common.cuh"
#include "ibcs.cuh"

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
    const float* scores;
    int64_t population;
    __device__ __forceinline__ void prepare(int64_t) {}
    __device__ __forceinline__ float score(int64_t row, int j) const {
        return scores[row * population + j];
    }
};

// Mixture of the eight centroid distributions, same expression as the reference
// scores kernel: score_j = (sum_c w_c * 2^(L_cj - max_c) / den_c) / sum_c w_c.
struct MixedScores {
    const half* lse;
    int64_t ld;
    const float* populations;
    const float* lse_max;
    const float* lse_den;
    float row_max[kCentroids];
    float row_den[kCentroids];
    float row_weight[kCentroids];
    float total_weight;

    __device__ __forceinline__ void prepare(int64_t row) {
#pragma unroll
        for (int c = 0; c < kCentroids; ++c) {
            row_max[c] = lse_max[row * kCentroids + c];
            row_den[c] = lse_den[row * kCentroids + c];
            row_weight[c] = populations[row * kCentroids + c];
        }
        total_weight = 0.0f;
#pragma unroll
        for (int c = 0; c < kCentroids; ++c) total_weight += row_weight[c];
    }
    __device__ __forceinline__ float score(int64_t row, int j) const {
        float value_sum = 0.0f;
#pragma unroll
        for (int c = 0; c < kCentroids; ++c) {
            const float value = __half2float(lse[(row * kCentroids + c) * ld + j]);
            const float probability = exp2f(value - row_max[c]) / row_den[c];
            value_sum += row_weight[c] * probability;
        }
        return value_sum / total_weight;
    }
};

template <class Source>
__global__ __launch_bounds__(kSipThreads) void sip_kernel(Source source, const float* __restrict__ offsets,
                                                          int32_t* __restrict__ sampled,
                                                          float* __restrict__ weights, int population,
                                                          int samples) {
    using Reduce = cub::BlockReduce<SumMax, kSipThreads>;
    using CountScan = cub::BlockScan<int, kSipThreads>;
    using MassScan = cub::BlockScan<double, kSipThreads>;
    union Scratch {
        typename Reduce::TempStorage reduce;
        typename CountScan::TempStorage count;
        typename MassScan::TempStorage mass;
    };
    __shared__ Scratch scratch;
    __shared__ double scale;
    __shared__ int certain;
    __shared__ int added;
    __shared__ int last_residual;
    __shared__ int marking;
    extern __shared__ double prefix[];

    const int buckets = (population + kSipBucket - 1) / kSipBucket;
    float* values = reinterpret_cast<float*>(prefix + buckets + 1);
    const int tid = threadIdx.x;
    const int64_t row = blockIdx.x;
    int32_t* out_ids = sampled + row * samples;
    float* out_logs = weights + row * samples;

    source.prepare(row);
    for (int j = tid; j < population; j += kSipThreads) values[j] = fmaxf(source.score(row, j), 1e-30f);
    if (tid == 0) certain = 0;
    __syncthreads();

    // Iterative certainty: mark every unit whose inclusion probability reaches 1
    // (negated in place) until the residual budget is stable (csrc/sip.cu:62-96).
    do {
        double local_sum = 0.;
        double local_max = 0.;
        for (int j = tid; j < population; j += kSipThreads) {
            if (values[j] > 0.f) {
                const double value = fmax(static_cast<double>(values[j]), 1e-30);
                local_sum += value;
                local_max = fmax(local_max, value);
            }
        }
        const SumMax total = Reduce(scratch.reduce).Reduce(SumMax{local_sum, local_max}, SumMaxOp{});
        if (tid == 0) {
            scale = (samples - certain) / total.sum;
            added = 0;
            marking = total.maximum * scale >= 1.0;
        }
        __syncthreads();
        if (marking) {
            int count = 0;
            for (int j = tid; j < population; j += kSipThreads) {
                if (values[j] > 0.f && fmax(static_cast<double>(values[j]), 1e-30) * scale >= 1.) {
                    values[j] = -values[j];
                    ++count;
                }
            }
            atomicAdd(&added, count);
        }
        __syncthreads();
        if (tid == 0) certain += added;
        __syncthreads();
    } while (added != 0);

    // Contiguous chunks of whole buckets per thread (csrc/sip.cu:98-106).
    const int chunk = ((buckets + kSipThreads - 1) / kSipThreads) * kSipBucket;
    const int begin = tid * chunk;
    const int end = min(begin + chunk, population);
    if (tid == 0) {
        int last = population - 1;
        while (last >= 0 && values[last] <= 0.) --last;
        last_residual = last;
    }
    __syncthreads();

    // Certain units first, ascending, log-weight 0 (csrc/sip.cu:108-124).
    if (certain != 0) {
        int count = 0;
        for (int j = begin; j < end; ++j) count += values[j] < 0.f;
        int rank = 0;
        CountScan(scratch.count).InclusiveSum(count, rank);
        int slot = rank - count;
        for (int j = begin; j < end; ++j) {
            if (values[j] < 0.f) {
                out_ids[slot] = j;
                out_logs[slot++] = 0.f;
            }
        }
        __syncthreads();
    }

    // Bucketed prefix of the residual masses (csrc/sip.cu:126-142).
    double chunk_mass = 0.;
    for (int j = begin; j < end; ++j)
        chunk_mass += values[j] > 0.f ? static_cast<double>(values[j]) * scale : 0.;
    double cumulative = 0.;
    MassScan(scratch.mass).ExclusiveSum(chunk_mass, cumulative);
    const int residuals = samples - certain;
    if (tid == 0) prefix[buckets] = residuals;
    for (int j = begin; j < end; ++j) {
        if (j % kSipBucket == 0) prefix[j / kSipBucket] = j > last_residual ? residuals : cumulative;
        cumulative += values[j] > 0.f ? static_cast<double>(values[j]) * scale : 0.;
    }
    __syncthreads();

    // Systematic draws at u + k: bucket search, then a walk of at most four
    // masses; the last residual closes roundoff escapes (csrc/sip.cu:144-166).
    const double offset = static_cast<double>(offsets[row]);
    for (int slot = tid; slot < residuals; slot += kSipThreads) {
        const double threshold = offset + slot;
        int lower = 0, upper = buckets;
        while (lower < upper) {
            const int middle = (lower + upper + 1) / 2;
            if (prefix[middle] <= threshold) lower = middle;
            else upper = middle - 1;
        }
        const int bucket = min(lower, buckets - 1);
        double mass = prefix[bucket];
        int selected = last_residual;
        const int stop = min((bucket + 1) * kSipBucket, population);
        for (int j = bucket * kSipBucket; j < stop; ++j) {
            if (values[j] <= 0.f) continue;
            selected = j;
            mass += static_cast<double>(values[j]) * scale;
            if (mass > threshold) break;
        }
        // The weight uses the unclamped score; `values` holds max(score, 1e-30f),
        // which equals it unless the clamp was active.
        const float kept = values[selected];
        const float raw = kept == 1e-30f ? source.score(row, selected) : kept;
        out_ids[certain + slot] = selected;
        out_logs[certain + slot] = static_cast<float>(-log2(fmax(static_cast<double>(raw), 1e-30) * scale));
    }
}

}  // namespace

size_t sip_smem_bytes(int64_t population) {
    const size_t buckets = static_cast<size_t>((population + kSipBucket - 1) / kSipBucket);
    return population * sizeof(float) + (buckets + 1) * sizeof(double);
}

int sip_smem_limit() {
    int device = 0, optin = 0;
    cudaGetDevice(&device);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
    cudaFuncAttributes attr{};
    cudaFuncGetAttributes(&attr, sip_kernel<MixedScores>);
    cudaFuncAttributes attr2{};
    cudaFuncGetAttributes(&attr2, sip_kernel<DenseScores>);
    const size_t static_bytes = attr.sharedSizeBytes > attr2.sharedSizeBytes ? attr.sharedSizeBytes : attr2.sharedSizeBytes;
    return optin - static_cast<int>(static_bytes);
}

template <class Source>
static cudaError_t launch_sip_impl(const Source& source, const float* offsets, int64_t rows,
                                   int64_t population, int32_t* ids, float* log_weights,
                                   int64_t samples, cudaStream_t stream) {
    const size_t smem = sip_smem_bytes(population);
    cudaError_t err = cudaFuncSetAttribute(sip_kernel<Source>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem));
    if (err != cudaSuccess) return err;
    sip_kernel<Source><<<static_cast<unsigned>(rows), kSipThreads, smem, stream>>>(
        source, offsets, ids, log_weights, static_cast<int>(population), static_cast<int>(samples));
    return cudaGetLastError();
}

cudaError_t launch_sip(const float* scores, const float* offsets, int64_t rows, int64_t population,
                       int32_t* ids, float* log_weights, int64_t samples, cudaStream_t stream) {
    DenseScores source{scores, population};
    return launch_sip_impl(source, offsets, rows, population, ids, log_weights, samples, stream);
}

cudaError_t launch_mix_sip(const half* lse, int64_t ld, const float* populations,
                           const float* lse_max, const float* lse_den, const float* offsets,
                           int64_t rows, int64_t population, int32_t* ids, float* log_weights,
                           int64_t samples, cudaStream_t stream) {
    MixedScores source{};
    source.lse = lse;
    source.ld = ld;
    source.populations = populations;
    source.lse_max = lse_max;
    source.lse_den = lse_den;
    return launch_sip_impl(source, offsets, rows, population, ids, log_weights, samples, stream);
}

}  // namespace abx
