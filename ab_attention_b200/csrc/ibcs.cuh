// Launchers of the IBCS, SIP and prefill kernels (called by the C ABI layer,
// which validates every argument first).
#pragma once

#include "common.cuh"

namespace abx {

// With k and pooled (both or neither), the clustering launch also writes the
// pooled key representatives (what launch_pool writes).
cudaError_t launch_cluster(const bf16* q, int64_t bh, int64_t seq, bf16* centroids, bf16* scaled,
                           float* populations, int32_t* assignments, cudaStream_t stream,
                           const bf16* k = nullptr, bf16* pooled = nullptr);
cudaError_t launch_pool(const bf16* k, int64_t bh, int64_t seq, bf16* pooled, cudaStream_t stream);
size_t lse_smem_bytes();
cudaError_t launch_lse(const bf16* scaled, const bf16* pooled, int64_t bh, int64_t qb,
                       int64_t fine_blocks, int64_t ld, half* lse, float* lse_max, float* lse_den,
                       cudaStream_t stream);
cudaError_t launch_mix(const half* lse, int64_t ld, const float* populations, const float* lse_max,
                       const float* lse_den, int64_t rows, int64_t fine_blocks, float* scores,
                       cudaStream_t stream);

// SIP over a dense score array (csrc/sip.cu).
size_t sip_smem_bytes(int64_t population);
int sip_smem_limit();
cudaError_t launch_sip(const float* scores, const float* offsets, int64_t rows, int64_t population,
                       int32_t* ids, float* log_weights, int64_t samples, cudaStream_t stream);
// SIP fed by the IBCS centroid LSE rows (the mixture is evaluated in the kernel).
cudaError_t launch_sip_mixed(const half* lse, int64_t ld, const float* populations, const float* lse_max,
                             const float* lse_den, const float* offsets, int64_t rows, int64_t population,
                             int32_t* ids, float* log_weights, int64_t samples, cudaStream_t stream);

// Sparse / dense prefill.
cudaError_t launch_prefill(const bf16* q, int64_t q_tokens, const bf16* k, const bf16* v, int64_t bh, int64_t seq,
                           const int32_t* ids, const float* log_weights, int64_t samples,
                           const bf16* text_k, const bf16* text_v, int64_t text_tokens, bf16* o,
                           float* lse, cudaStream_t stream);

// Paired sparse prefill (two adjacent query blocks per CTA over the union of
// their samples); pair_supported() says whether a shape can take it.
bool pair_supported(int64_t seq, int64_t samples, int64_t text_tokens);
size_t pair_workspace_bytes(int64_t bh, int64_t seq, int64_t samples, int64_t text_tokens);
// The two launches of launch_prefill_pair: the union lists of each pair (written
// into the workspace), then the prefill that reads them. A plan reused across
// calls needs its union lists built once.
cudaError_t launch_pair_plan(const int32_t* ids, int64_t bh, int64_t seq, int64_t samples, int64_t text_tokens,
                             void* workspace, size_t workspace_bytes, cudaStream_t stream);
// outs / num_outs (up to kMaxScatterOutputs): write every output row to each of
// these [heads, seq, 128] buffers at head out_head_base + head instead of to o.
constexpr int kMaxScatterOutputs = 8;
cudaError_t launch_pair_prefill(const bf16* q, const bf16* k, const bf16* v, int64_t bh, int64_t seq,
                                const int32_t* ids, const float* log_weights, int64_t samples, const bf16* text_k,
                                const bf16* text_v, int64_t text_tokens, bf16* o, float* lse, void* workspace,
                                size_t workspace_bytes, cudaStream_t stream, bf16* const* outs = nullptr,
                                int num_outs = 0, int64_t out_head_base = 0);
cudaError_t launch_prefill_pair(const bf16* q, const bf16* k, const bf16* v, int64_t bh, int64_t seq,
                                const int32_t* ids, const float* log_weights, int64_t samples, const bf16* text_k,
                                const bf16* text_v, int64_t text_tokens, bf16* o, float* lse, void* workspace,
                                size_t workspace_bytes, cudaStream_t stream);

}  // namespace abx
