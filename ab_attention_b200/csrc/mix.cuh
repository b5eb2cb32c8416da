// The IBCS mixture score of one KV4 block for one query row
// (ibcs_scores_kernel, csrc/ibcs.cu:495-538): the population-weighted mean,
// over the row's centroids, of the centroid's softmax probability
// 2^(lse - max) / den. Both the stand-alone scorer (mix_kernel) and the SIP
// kernel fed directly from the LSE rows evaluate it through this function, so
// they compile to the same operations and produce the same bits.
#pragma once

#include "common.cuh"

namespace abx {

__device__ __forceinline__ float mix_total_weight(const float* row_weight) {
    float total_weight = 0.0f;
#pragma unroll
    for (int c = 0; c < kCentroids; ++c) total_weight += row_weight[c];
    return total_weight;
}

// 1 / den of a centroid, taken once per row: the fast-math quotient x / den is
// x times this reciprocal, so the scores keep their bits.
__device__ __forceinline__ float mix_reciprocal(float den) { return 1.0f / den; }

__device__ __forceinline__ float mix_score(const half (&value)[kCentroids], const float* row_max,
                                           const float* row_rden, const float* row_weight, float total_weight) {
    float score = 0.0f;
#pragma unroll
    for (int c = 0; c < kCentroids; ++c) {
        const float probability = exp2f(__half2float(value[c]) - row_max[c]) * row_rden[c];
        score += row_weight[c] * probability;
    }
    return score / total_weight;
}

}  // namespace abx
