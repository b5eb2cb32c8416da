// Shared constants and small device helpers for the sm_100a AB-Attention kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>

#include "abx.h"

namespace abx {

using bf16 = __nv_bfloat16;

// Fixed problem constants of the reference path (csrc/ibcs.cu:32-39,
// flashinfer_backend.py:19-21, csrc/sip.cu:23-24).
constexpr int kHeadDim = 128;
constexpr int kQueryBlock = 128;
constexpr int kCentroids = 8;
constexpr int kKv4 = 4;          // tokens per sampling granule
constexpr int kReps = 2;         // pooled key representatives per granule
constexpr int kMaxFineBlocks = 32768;  // csrc/ibcs.cu:567
constexpr int kSipThreads = 256;
constexpr int kSipBucket = 4;

// 128^-0.5 * log2(e), rounded to float as the reference does (csrc/ibcs.cu:601-602).
inline float qk_scale_log2() {
    return static_cast<float>(0.08838834764831845 * 1.4426950408889634);
}

__host__ __device__ constexpr int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Device-side sticky error word (one per device, defined in capi.cu). A kernel
// whose bounded wait expires, or that meets an out-of-range index, records a
// nonzero code through this pointer and returns instead of hanging or faulting.
int* device_error_word();  // host: device address of the word on the current device

__device__ __forceinline__ void raise_device_error(int* word, int code) {
    if (word != nullptr) atomicCAS(word, 0, code);
}

// ---- small PTX wrappers -----------------------------------------------------

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async_16(void* smem, const void* gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_addr(smem)), "l"(gmem));
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }

template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

// D = A*B + C for one m16n8k16 bf16 tile with f32 accumulation.
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4],
                                               uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

}  // namespace abx
