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
// Scores come from a dense f32 [rows, population] array (the IBCS mixture of
// build_plan, or the caller's scores for `_C.sip`).
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

using Reduce = cub::BlockReduce<SumMax, kSipThreads>;
using CountScan = cub::BlockScan<int, kSipThreads>;
using MassScan = cub::BlockScan<double, kSipThreads>;
union Scratch {
    Reduce::TempStorage reduce;
    CountScan::TempStorage count;
    MassScan::TempStorage mass;
};

// Dynamic shared memory: the bucket prefix (doubles) then the masses (floats).
// CUB's temporaries live at the start of the prefix region: every block
// reduction and scan finishes before the first prefix entry is written, and
// keeping them out of static shared memory lets two rows share an SM at the
// Wan2.1 shape (F = 18,900).
__host__ __device__ constexpr size_t sip_prefix_region(int64_t population) {
    const size_t prefix = static_cast<size_t>((population + kSipBucket - 1) / kSipBucket + 1) * sizeof(double);
    return prefix > sizeof(Scratch) ? prefix : (sizeof(Scratch) + 15) / 16 * 16;
}

template <class Source>
__global__ __launch_bounds__(kSipThreads) void sip_kernel(Source source, const float* __restrict__ offsets,
                                                          int32_t* __restrict__ sampled,
                                                          float* __restrict__ weights, int population,
                                                          int samples) {
    extern __shared__ double prefix[];
    Scratch& scratch = *reinterpret_cast<Scratch*>(prefix);
    __shared__ double scale;
    __shared__ int certain;
    __shared__ int added;
    __shared__ int last_residual;
    __shared__ int marking;

    const int buckets = (population + kSipBucket - 1) / kSipBucket;
    float* values = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(prefix) + sip_prefix_region(population));
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
    // The reference re-sums the uncertain masses after each marking pass; the
    // units a marking pass leaves unmarked are exactly the terms of that sum,
    // visited in the same per-thread order, so the marking pass accumulates the
    // next partial sums itself and each iteration is one pass instead of two.
    double local_sum = 0.;
    double local_max = 0.;
    for (int j = tid; j < population; j += kSipThreads) {
        if (values[j] > 0.f) {
            const double value = fmax(static_cast<double>(values[j]), 1e-30);
            local_sum += value;
            local_max = fmax(local_max, value);
        }
    }
    do {
        const SumMax total = Reduce(scratch.reduce).Reduce(SumMax{local_sum, local_max}, SumMaxOp{});
        if (tid == 0) {
            scale = (samples - certain) / total.sum;
            added = 0;
            marking = total.maximum * scale >= 1.0;
        }
        __syncthreads();
        if (marking) {
            int count = 0;
            local_sum = 0.;
            local_max = 0.;
            for (int j = tid; j < population; j += kSipThreads) {
                if (values[j] > 0.f) {
                    const double value = fmax(static_cast<double>(values[j]), 1e-30);
                    if (value * scale >= 1.) {
                        values[j] = -values[j];
                        ++count;
                    } else {
                        local_sum += value;
                        local_max = fmax(local_max, value);
                    }
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
    __syncthreads();  // the scan's temporaries overlap the prefix written below
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
    sip_kernel<Source><<<static_cast<unsigned>(rows), kSipThreads, smem, stream>>>(
        source, offsets, ids, log_weights, static_cast<int>(population), static_cast<int>(samples));
    return cudaGetLastError();
}

cudaError_t launch_sip(const float* scores, const float* offsets, int64_t rows, int64_t population,
                       int32_t* ids, float* log_weights, int64_t samples, cudaStream_t stream) {
    DenseScores source{scores, population};
    return launch_sip_impl(source, offsets, rows, population, ids, log_weights, samples, stream);
}

}  // namespace abx
