// Test-only harness around the reference IBCS kernels (AB-Attention csrc/ibcs.cu).
//
// ORACLE INFRASTRUCTURE: this file is compiled by oracle/build_ref.py into
// oracle/_ref/ and is imported only by tests, smoke() and bench.py's CPU
// baseline leg as a checker. It is never part of the shipped library.
//
// The reference keeps its four IBCS kernels in an anonymous namespace and only
// exports `ibcs_cuda` (csrc/ibcs.cu:549-617). To compare every stage bit for
// bit, this translation unit includes the reference source file where it lies
// (the include path points at the reference checkout; nothing is copied) and
// launches each stage kernel on its own, with the same launch shapes the
// reference wrapper uses (csrc/ibcs.cu:589-614).
//
// Cluster assignments: the reference keeps each query's centroid slot in a
// shared-memory array (`assignments`, csrc/ibcs.cu:116,165-197) and never
// writes it out. To read it without copying or editing the reference source,
// this unit compiles that source with one hook: every `__syncthreads()` in its
// text becomes a barrier followed by a store of the kernel's `assignments`
// array (when a dump buffer is set). Inside cluster_queries_kernel the name
// refers to the kernel's own 128-entry shared array, which shadows the
// one-element namespace-scope stand-in below; in every other kernel it refers
// to the stand-in, whose size disables the store at compile time. The last
// barrier of the kernel (after the populations, csrc/ibcs.cu:211) leaves the
// final assignments in the dump. Headers are included first, so the hook
// reaches only the reference file's own text, not CUB or the CUDA headers.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAException.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cub/block/block_reduce.cuh>
#include <torch/extension.h>

#include "ops.h"
#include "flashinfer/permuted_smem.cuh"

namespace abx_ref_hook {
__device__ int* g_assign_dump = nullptr;

template <size_t kBytes>
__device__ __forceinline__ void sync_and_dump(const int* values) {
    __syncthreads();
    if constexpr (kBytes == 128 * sizeof(int)) {
        int* dump = g_assign_dump;
        if (dump != nullptr && blockDim.x == 128)
            dump[(static_cast<size_t>(blockIdx.y) * gridDim.x + blockIdx.x) * 128 + threadIdx.x] = values[threadIdx.x];
    }
}
}  // namespace abx_ref_hook

__device__ int assignments[1];  // stand-in, shadowed inside cluster_queries_kernel

#define __syncthreads() abx_ref_hook::sync_and_dump<sizeof(assignments)>(assignments)
#include "ibcs.cu"
#undef __syncthreads

#include <tuple>

namespace abx_ref {

std::tuple<torch::Tensor, torch::Tensor> cluster(torch::Tensor q) {
    // q: [BH, S, 128] bf16 contiguous -> packed_q [BH, qb, 8, 128], populations [BH, qb, 8]
    TORCH_CHECK(q.is_cuda() && q.is_contiguous() && q.dim() == 3 && q.size(2) == kHeadDim);
    const int64_t bh = q.size(0), seq = q.size(1);
    const int64_t qb = (seq + kQueryBlockSize - 1) / kQueryBlockSize;
    c10::cuda::CUDAGuard guard(q.device());
    auto packed_q = torch::empty({bh, qb, kQueryCentroids, kHeadDim}, q.options());
    auto pops = torch::empty({bh, qb, kQueryCentroids}, q.options().dtype(torch::kFloat16));
    auto stream = at::cuda::getCurrentCUDAStream();
    cluster_queries_kernel<<<dim3(qb, bh), kHeadDim, 0, stream>>>(
        tensor_ptr<const Bf16>(q), tensor_ptr<Bf16>(packed_q), tensor_ptr<half>(pops), seq, qb);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return {packed_q, pops};
}

std::tuple<torch::Tensor, torch::Tensor, torch::Tensor> cluster_assignments(torch::Tensor q) {
    // cluster() plus the per-query centroid slot [BH, qb, 128] int32 read out of
    // the kernel's shared memory by the hook above; entries past a partial last
    // block are unspecified (the reference never sets them).
    TORCH_CHECK(q.is_cuda() && q.is_contiguous() && q.dim() == 3 && q.size(2) == kHeadDim);
    const int64_t bh = q.size(0), seq = q.size(1);
    const int64_t qb = (seq + kQueryBlockSize - 1) / kQueryBlockSize;
    c10::cuda::CUDAGuard guard(q.device());
    auto assign = torch::full({bh, qb, kQueryBlockSize}, -1, q.options().dtype(torch::kInt32));
    auto stream = at::cuda::getCurrentCUDAStream();
    int* dump = assign.data_ptr<int>();
    C10_CUDA_CHECK(cudaMemcpyToSymbolAsync(abx_ref_hook::g_assign_dump, &dump, sizeof(dump), 0,
                                           cudaMemcpyHostToDevice, stream));
    auto out = cluster(q);
    int* none = nullptr;
    C10_CUDA_CHECK(cudaMemcpyToSymbolAsync(abx_ref_hook::g_assign_dump, &none, sizeof(none), 0,
                                           cudaMemcpyHostToDevice, stream));
    C10_CUDA_CHECK(cudaStreamSynchronize(stream));
    return {std::get<0>(out), std::get<1>(out), assign};
}

torch::Tensor pool(torch::Tensor k) {
    // k: [BH, S, 128] bf16 -> packed_k [BH, S/4, 2, 128]
    TORCH_CHECK(k.is_cuda() && k.is_contiguous() && k.dim() == 3 && k.size(2) == kHeadDim);
    const int64_t bh = k.size(0), fine = k.size(1) / kSamplingBlockSize;
    c10::cuda::CUDAGuard guard(k.device());
    auto packed_k = torch::empty({bh, fine, kKeyRepresentatives, kHeadDim}, k.options());
    auto stream = at::cuda::getCurrentCUDAStream();
    pool_keys_kernel<<<dim3(fine, bh), kHeadDim, 0, stream>>>(
        tensor_ptr<const Bf16>(k), tensor_ptr<Bf16>(packed_k), fine);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return packed_k;
}

std::tuple<torch::Tensor, torch::Tensor, torch::Tensor> lse(
    torch::Tensor packed_q, torch::Tensor packed_k) {
    // packed_q [BH, qb, 8, 128], packed_k [BH, F, 2, 128] -> lse [rows, 8, F] fp16, max/den [rows, 8]
    const int64_t bh = packed_q.size(0), qb = packed_q.size(1), fine = packed_k.size(1);
    const int64_t rows = bh * qb;
    c10::cuda::CUDAGuard guard(packed_q.device());
    auto out = torch::empty({rows, kQueryCentroids, fine}, packed_q.options().dtype(torch::kFloat16));
    auto mx = torch::empty({rows, kQueryCentroids}, packed_q.options().dtype(torch::kFloat32));
    auto den = torch::empty_like(mx);
    const float qk_scale_log2 = static_cast<float>(
        std::pow(static_cast<double>(kHeadDim), -0.5) * 1.4426950408889634);
    const int64_t q_groups = (qb + kQBlocksPerGroup - 1) / kQBlocksPerGroup;
    const int tiles = static_cast<int>((q_groups + kWarps - 1) / kWarps);
    auto stream = at::cuda::getCurrentCUDAStream();
    ibcs_lse_kernel<<<dim3(tiles, bh), kThreads, kSharedBytes, stream>>>(
        tensor_ptr<const Bf16>(packed_q), tensor_ptr<const Bf16>(packed_k),
        tensor_ptr<half>(out), mx.data_ptr<float>(), den.data_ptr<float>(),
        qb, static_cast<int>(fine), qk_scale_log2);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return {out, mx, den};
}

torch::Tensor scores(torch::Tensor lse, torch::Tensor pops, torch::Tensor mx, torch::Tensor den) {
    const int64_t rows = lse.size(0), fine = lse.size(2);
    c10::cuda::CUDAGuard guard(lse.device());
    auto out = torch::empty({rows, fine}, lse.options().dtype(torch::kFloat32));
    auto stream = at::cuda::getCurrentCUDAStream();
    ibcs_scores_kernel<<<static_cast<unsigned>(rows), kScoreThreads, 0, stream>>>(
        tensor_ptr<const half>(lse), tensor_ptr<const half>(pops), mx.data_ptr<float>(),
        den.data_ptr<float>(), out.data_ptr<float>(), static_cast<int>(fine));
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return out;
}

}  // namespace abx_ref
