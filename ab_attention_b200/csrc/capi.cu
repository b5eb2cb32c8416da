// extern "C" boundary of libabx (declared in include/abx.h).
//
// Validates every argument on the host, lays out the caller-owned workspace,
// and launches the kernels on the caller's stream. No allocation, no host
// synchronisation (except abx_device_status, which reads the error word).
#include <cuda.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "ibcs.cuh"
#include "tcgen05.cuh"

namespace abx {

__device__ int g_device_error = 0;

int* device_error_word() {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_device_error) != cudaSuccess) return nullptr;
    return static_cast<int*>(ptr);
}

// Two warps wait, bounded by limit_cycles, on an mbarrier that nothing arrives
// at: warp 0 with the library's polling wait, warp 1 with its suspending wait
// (the form the prefill kernels use). Both give up, each on its own abort flag,
// and the kernel records ABX_ERR_DEVICE_TIMEOUT only when both did, exercising
// both timeout paths without a fault.
__global__ void wait_selftest_kernel(uint64_t limit_cycles, int* error) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_flag[2];
    __shared__ int gave_up[2];
    const int w = threadIdx.x >> 5;
    if (threadIdx.x == 0) {
        abort_flag[0] = abort_flag[1] = 0;
        tc::mbar_init(smem_addr(&bar), 1);
        tc::mbar_init_fence();
    }
    __syncthreads();
    const bool ok = w == 0 ? tc::mbar_wait_warp(smem_addr(&bar), 0, &abort_flag[0], limit_cycles)
                           : tc::mbar_wait_warp_suspend(smem_addr(&bar), 0, &abort_flag[1], limit_cycles);
    if ((threadIdx.x & 31) == 0) gave_up[w] = !ok;
    __syncthreads();
    if (threadIdx.x == 0 && gave_up[0] && gave_up[1]) raise_device_error(error, ABX_ERR_DEVICE_TIMEOUT);
}

}  // namespace abx

namespace {

thread_local char g_last_error[512] = "";

int fail(int status, const char* fmt, ...) {
    va_list args;
    va_start(args, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, args);
    va_end(args);
    return status;
}

int check_cuda(cudaError_t err, const char* what) {
    if (err == cudaSuccess) return ABX_OK;
    return fail(ABX_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
}

// A driver API call reached through the runtime's entry-point table (no libcuda link).
template <class Fn>
Fn driver_entry(const char* name) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult status;
    if (cudaGetDriverEntryPoint(name, &ptr, cudaEnableDefault, &status) != cudaSuccess ||
        status != cudaDriverEntryPointSuccess)
        return nullptr;
    return reinterpret_cast<Fn>(ptr);
}

constexpr size_t kAlign = 256;
size_t align_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Workspace of the IBCS stages for (bh, seq).
struct IbcsLayout {
    int64_t qb, rows, fine, ld;
    size_t scaled, populations, pooled, lse, lse_max, lse_den, total;
};

IbcsLayout ibcs_layout(int64_t bh, int64_t seq) {
    IbcsLayout l{};
    l.qb = abx::ceil_div(seq, abx::kQueryBlock);
    l.rows = bh * l.qb;
    l.fine = seq / abx::kKv4;
    l.ld = (l.fine + 7) / 8 * 8;
    size_t off = 0;
    l.scaled = off;
    off = align_up(off + static_cast<size_t>(l.rows) * abx::kCentroids * abx::kHeadDim * 2);
    l.populations = off;
    off = align_up(off + static_cast<size_t>(l.rows) * abx::kCentroids * 4);
    l.pooled = off;
    off = align_up(off + static_cast<size_t>(bh) * l.fine * abx::kReps * abx::kHeadDim * 2);
    l.lse = off;
    off = align_up(off + static_cast<size_t>(l.rows) * abx::kCentroids * l.ld * 2);
    l.lse_max = off;
    off = align_up(off + static_cast<size_t>(l.rows) * abx::kCentroids * 4);
    l.lse_den = off;
    off = align_up(off + static_cast<size_t>(l.rows) * abx::kCentroids * 4);
    // No block-score array: abx_build_plan's SIP evaluates the mixture from the
    // LSE rows, and abx_ibcs_scores writes the caller's scores.
    l.total = off;
    return l;
}

int check_qk_shape(int64_t bh, int64_t seq) {
    if (bh <= 0) return fail(ABX_ERR_INVALID_ARGUMENT, "batch*heads must be positive (got %lld)", (long long)bh);
    if (seq <= 0 || seq % abx::kKv4 != 0)
        return fail(ABX_ERR_INVALID_ARGUMENT, "sequence length must be a positive multiple of 4 (got %lld)", (long long)seq);
    const int64_t fine = seq / abx::kKv4;
    if (fine > abx::kMaxFineBlocks)
        return fail(ABX_ERR_UNSUPPORTED, "KV4 block count must be in [1, 32768] (got %lld)", (long long)fine);
    if (bh * abx::ceil_div(seq, abx::kQueryBlock) > 0x7fffffffLL)
        return fail(ABX_ERR_UNSUPPORTED, "too many query blocks");
    return ABX_OK;
}

int check_sip_shape(int64_t rows, int64_t population, int64_t samples) {
    if (rows <= 0) return fail(ABX_ERR_INVALID_ARGUMENT, "row count must be positive");
    if (samples <= 0 || samples >= population)
        return fail(ABX_ERR_INVALID_ARGUMENT, "sample count must be inside the population (0 < %lld < %lld)",
                    (long long)samples, (long long)population);
    if (population > 0x7fffffffLL) return fail(ABX_ERR_UNSUPPORTED, "population too large");
    const size_t need = abx::sip_smem_bytes(population);
    const int limit = abx::sip_smem_limit();
    if (limit <= 0 || need > static_cast<size_t>(limit))
        return fail(ABX_ERR_UNSUPPORTED, "population exceeds single-block shared memory capacity (%zu > %d bytes)",
                    need, limit);
    return ABX_OK;
}

}  // namespace

extern "C" {

int abx_version(void) { return 1; }

const char* abx_status_string(int status) {
    switch (status) {
        case ABX_OK: return "ok";
        case ABX_ERR_INVALID_ARGUMENT: return "invalid argument";
        case ABX_ERR_UNSUPPORTED: return "unsupported shape";
        case ABX_ERR_WORKSPACE: return "workspace too small or misaligned";
        case ABX_ERR_CUDA: return "CUDA error";
        case ABX_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
        default: return "unknown status";
    }
}

const char* abx_last_error(void) { return g_last_error; }

int abx_device_status(abx_stream_t stream, int clear, int* status_out) {
    if (status_out == nullptr) return fail(ABX_ERR_INVALID_ARGUMENT, "status_out is null");
    int value = 0;
    int st = check_cuda(cudaMemcpyFromSymbolAsync(&value, abx::g_device_error, sizeof(int), 0,
                                                  cudaMemcpyDeviceToHost, stream),
                        "read device status");
    if (st) return st;
    st = check_cuda(cudaStreamSynchronize(stream), "synchronize");
    if (st) return st;
    if (clear) {
        const int zero = 0;
        st = check_cuda(cudaMemcpyToSymbolAsync(abx::g_device_error, &zero, sizeof(int), 0,
                                                cudaMemcpyHostToDevice, stream),
                        "clear device status");
        if (st) return st;
        st = check_cuda(cudaStreamSynchronize(stream), "synchronize");
        if (st) return st;
    }
    *status_out = value;
    return ABX_OK;
}

int abx_ibcs_cluster(const void* q, int64_t bh, int64_t seq, void* centroids, void* scaled_centroids,
                     float* populations, int32_t* assignments, abx_stream_t stream) {
    if (int st = check_qk_shape(bh, seq)) return st;
    if (q == nullptr || populations == nullptr)
        return fail(ABX_ERR_INVALID_ARGUMENT, "q and populations must be non-null");
    if (!aligned16(q) || (centroids && !aligned16(centroids)) || (scaled_centroids && !aligned16(scaled_centroids)))
        return fail(ABX_ERR_INVALID_ARGUMENT, "q and centroid buffers must be 16-byte aligned");
    return check_cuda(abx::launch_cluster(static_cast<const abx::bf16*>(q), bh, seq,
                                          static_cast<abx::bf16*>(centroids),
                                          static_cast<abx::bf16*>(scaled_centroids), populations,
                                          assignments, stream),
                      "cluster launch");
}

int abx_ibcs_pool(const void* k, int64_t bh, int64_t seq, void* pooled, abx_stream_t stream) {
    if (int st = check_qk_shape(bh, seq)) return st;
    if (k == nullptr || pooled == nullptr) return fail(ABX_ERR_INVALID_ARGUMENT, "k and pooled must be non-null");
    if (!aligned16(k) || !aligned16(pooled)) return fail(ABX_ERR_INVALID_ARGUMENT, "k and pooled must be 16-byte aligned");
    return check_cuda(abx::launch_pool(static_cast<const abx::bf16*>(k), bh, seq, static_cast<abx::bf16*>(pooled), stream),
                      "pool launch");
}

int abx_ibcs_lse(const void* scaled_centroids, const void* pooled, int64_t bh, int64_t qb,
                 int64_t fine_blocks, uint16_t* lse, float* lse_max, float* lse_den, abx_stream_t stream) {
    if (bh <= 0 || qb <= 0 || fine_blocks <= 0 || fine_blocks > abx::kMaxFineBlocks)
        return fail(ABX_ERR_INVALID_ARGUMENT, "bad IBCS LSE shape");
    if (!scaled_centroids || !pooled || !lse || !lse_max || !lse_den)
        return fail(ABX_ERR_INVALID_ARGUMENT, "IBCS LSE buffers must be non-null");
    if (!aligned16(scaled_centroids) || !aligned16(pooled) || !aligned16(lse))
        return fail(ABX_ERR_INVALID_ARGUMENT, "IBCS LSE buffers must be 16-byte aligned");
    return check_cuda(abx::launch_lse(static_cast<const abx::bf16*>(scaled_centroids),
                                      static_cast<const abx::bf16*>(pooled), bh, qb, fine_blocks,
                                      fine_blocks, reinterpret_cast<half*>(lse), lse_max, lse_den, stream),
                      "lse launch");
}

int abx_ibcs_mix(const uint16_t* lse, const float* populations, const float* lse_max, const float* lse_den,
                 int64_t rows, int64_t fine_blocks, float* scores, abx_stream_t stream) {
    if (rows <= 0 || fine_blocks <= 0) return fail(ABX_ERR_INVALID_ARGUMENT, "bad IBCS mix shape");
    if (!lse || !populations || !lse_max || !lse_den || !scores)
        return fail(ABX_ERR_INVALID_ARGUMENT, "IBCS mix buffers must be non-null");
    return check_cuda(abx::launch_mix(reinterpret_cast<const half*>(lse), fine_blocks, populations, lse_max,
                                      lse_den, rows, fine_blocks, scores, stream),
                      "mix launch");
}

int abx_ibcs_workspace_size(int64_t bh, int64_t seq, size_t* bytes) {
    if (bytes == nullptr) return fail(ABX_ERR_INVALID_ARGUMENT, "bytes is null");
    if (int st = check_qk_shape(bh, seq)) return st;
    *bytes = ibcs_layout(bh, seq).total;
    return ABX_OK;
}

static int run_ibcs_front(const void* q, const void* k, int64_t bh, int64_t seq, void* workspace,
                          size_t workspace_bytes, const IbcsLayout& l, cudaStream_t stream) {
    if (workspace == nullptr || (reinterpret_cast<uintptr_t>(workspace) % kAlign) != 0)
        return fail(ABX_ERR_WORKSPACE, "workspace must be non-null and 256-byte aligned");
    if (workspace_bytes < l.total)
        return fail(ABX_ERR_WORKSPACE, "workspace too small (%zu < %zu bytes)", workspace_bytes, l.total);
    if (!q || !k || !aligned16(q) || !aligned16(k))
        return fail(ABX_ERR_INVALID_ARGUMENT, "q and k must be non-null and 16-byte aligned");
    char* ws = static_cast<char*>(workspace);
    auto* scaled = reinterpret_cast<abx::bf16*>(ws + l.scaled);
    auto* pops = reinterpret_cast<float*>(ws + l.populations);
    auto* pooled = reinterpret_cast<abx::bf16*>(ws + l.pooled);
    auto* lse = reinterpret_cast<half*>(ws + l.lse);
    auto* mx = reinterpret_cast<float*>(ws + l.lse_max);
    auto* den = reinterpret_cast<float*>(ws + l.lse_den);
    // clustering and key pooling in one launch
    if (int st = check_cuda(abx::launch_cluster(static_cast<const abx::bf16*>(q), bh, seq, nullptr, scaled,
                                                pops, nullptr, stream, static_cast<const abx::bf16*>(k), pooled),
                            "cluster launch"))
        return st;
    return check_cuda(abx::launch_lse(scaled, pooled, bh, l.qb, l.fine, l.ld, lse, mx, den, stream), "lse launch");
}

int abx_ibcs_scores(const void* q, const void* k, int64_t bh, int64_t seq, float* scores, void* workspace,
                    size_t workspace_bytes, abx_stream_t stream) {
    if (int st = check_qk_shape(bh, seq)) return st;
    if (scores == nullptr) return fail(ABX_ERR_INVALID_ARGUMENT, "scores is null");
    const IbcsLayout l = ibcs_layout(bh, seq);
    if (int st = run_ibcs_front(q, k, bh, seq, workspace, workspace_bytes, l, stream)) return st;
    char* ws = static_cast<char*>(workspace);
    return check_cuda(abx::launch_mix(reinterpret_cast<const half*>(ws + l.lse), l.ld,
                                      reinterpret_cast<const float*>(ws + l.populations),
                                      reinterpret_cast<const float*>(ws + l.lse_max),
                                      reinterpret_cast<const float*>(ws + l.lse_den), l.rows, l.fine, scores,
                                      stream),
                      "mix launch");
}

int abx_sip(const float* scores, const float* offsets, int64_t rows, int64_t population, int32_t* ids,
            float* log_weights, int64_t samples, abx_stream_t stream) {
    if (int st = check_sip_shape(rows, population, samples)) return st;
    if (!scores || !offsets || !ids || !log_weights)
        return fail(ABX_ERR_INVALID_ARGUMENT, "SIP buffers must be non-null");
    return check_cuda(abx::launch_sip(scores, offsets, rows, population, ids, log_weights, samples, stream),
                      "sip launch");
}

int abx_build_plan(const void* q, const void* k, int64_t bh, int64_t seq, const float* offsets, int64_t samples,
                   int32_t* ids, float* log_weights, void* workspace, size_t workspace_bytes,
                   abx_stream_t stream) {
    if (int st = check_qk_shape(bh, seq)) return st;
    const IbcsLayout l = ibcs_layout(bh, seq);
    if (int st = check_sip_shape(l.rows, l.fine, samples)) return st;
    if (!offsets || !ids || !log_weights) return fail(ABX_ERR_INVALID_ARGUMENT, "plan buffers must be non-null");
    if (int st = run_ibcs_front(q, k, bh, seq, workspace, workspace_bytes, l, stream)) return st;
    // SIP evaluates the mixture scores from the LSE rows itself (no score array).
    char* ws = static_cast<char*>(workspace);
    return check_cuda(abx::launch_sip_mixed(reinterpret_cast<const half*>(ws + l.lse), l.ld,
                                            reinterpret_cast<const float*>(ws + l.populations),
                                            reinterpret_cast<const float*>(ws + l.lse_max),
                                            reinterpret_cast<const float*>(ws + l.lse_den), offsets, l.rows, l.fine,
                                            ids, log_weights, samples, stream),
                      "sip launch");
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free build_plan: the IBCS scratch lives in a fixed device array.
//
// Some callers cannot call cudaMalloc: a host process whose device memory is
// owned by another allocator (a framework's caching pool, or a serving runtime
// that reserves all memory up front), a plugin host that forbids allocation
// after start-up, or a latency-critical path that cannot afford cudaMalloc's
// implicit device synchronisation. abx_build_plan_static serves them: it needs
// no workspace argument and allocates nothing, using the 256 MiB array below,
// which every GPU that loads libabx holds until the process exits.
// ---------------------------------------------------------------------------
namespace {

constexpr size_t kStaticScratchBytes = size_t(256) << 20;
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

using PfnCtxGetCurrent = CUresult (*)(CUcontext*);
using PfnCtxGetId = CUresult (*)(CUcontext, unsigned long long*);

// The array's device address per CUDA context, keyed by the context's unique
// id (cuCtxGetId never reuses an id within a process). A host that creates its
// own context on a device, or that resets the device, gets a fresh lookup
// instead of an address that belongs to another or a destroyed context.
struct ScratchSlot {
    unsigned long long context_id;
    void* ptr;
};
constexpr int kScratchSlots = 64;
std::mutex g_static_scratch_mutex;
ScratchSlot g_static_scratch_slots[kScratchSlots] = {};
int g_static_scratch_next = 0;

// Device address of g_static_scratch in the calling thread's current context.
// In host code the array's name is only a host-side stand-in, so the address
// is looked up with cudaGetSymbolAddress (with that device current) once per
// context and cached.
int static_scratch(void** out) {
    static const PfnCtxGetCurrent ctx_get_current = driver_entry<PfnCtxGetCurrent>("cuCtxGetCurrent");
    static const PfnCtxGetId ctx_get_id = driver_entry<PfnCtxGetId>("cuCtxGetId");
    if (ctx_get_current == nullptr || ctx_get_id == nullptr)
        return fail(ABX_ERR_CUDA, "cuCtxGetCurrent / cuCtxGetId unavailable in this driver");
    CUcontext ctx = nullptr;
    if (ctx_get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) {
        // No context is bound to this thread yet: the symbol lookup initialises
        // the current device's primary context and makes it current.
        void* ptr = nullptr;
        if (int st = check_cuda(cudaGetSymbolAddress(&ptr, g_static_scratch), "cudaGetSymbolAddress(static scratch)"))
            return st;
        if (ctx_get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr)
            return fail(ABX_ERR_CUDA, "no current CUDA context after the symbol lookup");
    }
    unsigned long long id = 0;
    if (ctx_get_id(ctx, &id) != CUDA_SUCCESS) return fail(ABX_ERR_CUDA, "cuCtxGetId failed");
    std::lock_guard<std::mutex> lock(g_static_scratch_mutex);
    for (const ScratchSlot& slot : g_static_scratch_slots) {
        if (slot.ptr != nullptr && slot.context_id == id) {
            *out = slot.ptr;
            return ABX_OK;
        }
    }
    void* ptr = nullptr;
    if (int st = check_cuda(cudaGetSymbolAddress(&ptr, g_static_scratch), "cudaGetSymbolAddress(static scratch)"))
        return st;
    g_static_scratch_slots[g_static_scratch_next] = ScratchSlot{id, ptr};
    g_static_scratch_next = (g_static_scratch_next + 1) % kScratchSlots;
    *out = ptr;
    return ABX_OK;
}

}  // namespace

extern "C" {

size_t abx_static_scratch_bytes(void) { return kStaticScratchBytes; }

int abx_build_plan_static(const void* q, const void* k, int64_t bh, int64_t seq, const float* offsets,
                          int64_t samples, int32_t* ids, float* log_weights, abx_stream_t stream) {
    if (int st = check_qk_shape(bh, seq)) return st;
    const IbcsLayout one = ibcs_layout(1, seq);
    if (one.total > kStaticScratchBytes)
        return fail(ABX_ERR_WORKSPACE,
                    "abx_build_plan_static: one head of %lld tokens needs %zu bytes of scratch, more than the "
                    "fixed %zu-byte array; use abx_build_plan with a caller workspace",
                    (long long)seq, one.total, kStaticScratchBytes);
    if (int st = check_sip_shape(one.rows, one.fine, samples)) return st;
    if (!q || !k || !offsets || !ids || !log_weights)
        return fail(ABX_ERR_INVALID_ARGUMENT, "q, k, offsets, ids and log_weights must be non-null");
    void* scratch = nullptr;
    if (int st = static_scratch(&scratch)) return st;
    // Heads per pass: as many as the array holds; passes run in stream order.
    int64_t per_pass = 1;
    while (per_pass < bh && ibcs_layout(per_pass + 1, seq).total <= kStaticScratchBytes) ++per_pass;
    const int64_t head_elems = seq * abx::kHeadDim;
    for (int64_t start = 0; start < bh; start += per_pass) {
        const int64_t heads = (bh - start) < per_pass ? (bh - start) : per_pass;
        const int64_t row0 = start * one.qb;
        const int st = abx_build_plan(static_cast<const abx::bf16*>(q) + start * head_elems,
                                      static_cast<const abx::bf16*>(k) + start * head_elems, heads, seq,
                                      offsets + row0, samples, ids + row0 * samples, log_weights + row0 * samples,
                                      scratch, kStaticScratchBytes, stream);
        if (st) return st;
    }
    return ABX_OK;
}

int abx_sparse_prefill(const void* q, const void* k, const void* v, int64_t bh, int64_t seq, const int32_t* ids,
                       const float* log_weights, int64_t samples, const void* text_k, const void* text_v,
                       int64_t text_tokens, void* o, float* lse, abx_stream_t stream) {
    if (int st = check_qk_shape(bh, seq)) return st;
    if (!q || !k || !v || !o) return fail(ABX_ERR_INVALID_ARGUMENT, "q, k, v and o must be non-null");
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o))
        return fail(ABX_ERR_INVALID_ARGUMENT, "q, k, v and o must be 16-byte aligned");
    if (samples < 0 || samples > seq / abx::kKv4)
        return fail(ABX_ERR_INVALID_ARGUMENT, "samples must be in [0, seq/4] (got %lld)", (long long)samples);
    if (samples > 0 && (ids == nullptr || log_weights == nullptr))
        return fail(ABX_ERR_INVALID_ARGUMENT, "ids and log_weights must be non-null");
    if (text_tokens < 0) return fail(ABX_ERR_INVALID_ARGUMENT, "negative text token count");
    if (text_tokens > 0 && (!text_k || !text_v || !aligned16(text_k) || !aligned16(text_v)))
        return fail(ABX_ERR_INVALID_ARGUMENT, "text_k/text_v must be non-null and 16-byte aligned");
    if (samples + (text_tokens + abx::kKv4 - 1) / abx::kKv4 <= 0)
        return fail(ABX_ERR_INVALID_ARGUMENT, "every row needs at least one key block");
    return check_cuda(abx::launch_prefill(static_cast<const abx::bf16*>(q), seq, static_cast<const abx::bf16*>(k),
                                          static_cast<const abx::bf16*>(v), bh, seq, ids, log_weights, samples,
                                          static_cast<const abx::bf16*>(text_k),
                                          static_cast<const abx::bf16*>(text_v), text_tokens,
                                          static_cast<abx::bf16*>(o), lse, stream),
                      "prefill launch");
}

int abx_prefill_workspace_size(int64_t bh, int64_t seq, int64_t samples, int64_t text_tokens, size_t* bytes) {
    if (bytes == nullptr) return fail(ABX_ERR_INVALID_ARGUMENT, "bytes must be non-null");
    if (int st = check_qk_shape(bh, seq)) return st;
    if (samples < 0 || text_tokens < 0) return fail(ABX_ERR_INVALID_ARGUMENT, "negative sample or text count");
    *bytes = abx::pair_supported(seq, samples, text_tokens) ? abx::pair_workspace_bytes(bh, seq, samples, text_tokens)
                                                             : 0;
    return ABX_OK;
}

}  // extern "C"

namespace {

// Arguments of the paired prefill once the shape is known to pair.
int check_paired(const void* q, const void* k, const void* v, int64_t bh, int64_t seq, const int32_t* ids,
                 const float* log_weights, int64_t samples, const void* text_k, const void* text_v,
                 int64_t text_tokens, const void* o, const void* workspace, size_t workspace_bytes) {
    if (int st = check_qk_shape(bh, seq)) return st;
    if (!q || !k || !v || !o) return fail(ABX_ERR_INVALID_ARGUMENT, "q, k, v and o must be non-null");
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o))
        return fail(ABX_ERR_INVALID_ARGUMENT, "q, k, v and o must be 16-byte aligned");
    if (samples > seq / abx::kKv4)
        return fail(ABX_ERR_INVALID_ARGUMENT, "samples must be in [0, seq/4] (got %lld)", (long long)samples);
    if (ids == nullptr || log_weights == nullptr)
        return fail(ABX_ERR_INVALID_ARGUMENT, "ids and log_weights must be non-null");
    if (text_tokens > 0 && (!text_k || !text_v || !aligned16(text_k) || !aligned16(text_v)))
        return fail(ABX_ERR_INVALID_ARGUMENT, "text_k/text_v must be non-null and 16-byte aligned");
    if (workspace == nullptr || workspace_bytes < abx::pair_workspace_bytes(bh, seq, samples, text_tokens))
        return fail(ABX_ERR_WORKSPACE, "workspace too small (%zu bytes, need %zu)", workspace_bytes,
                    abx::pair_workspace_bytes(bh, seq, samples, text_tokens));
    return ABX_OK;
}

}  // namespace

extern "C" {

int abx_sparse_prefill_paired(const void* q, const void* k, const void* v, int64_t bh, int64_t seq,
                              const int32_t* ids, const float* log_weights, int64_t samples, const void* text_k,
                              const void* text_v, int64_t text_tokens, void* o, float* lse, void* workspace,
                              size_t workspace_bytes, abx_stream_t stream) {
    if (samples < 0 || text_tokens < 0)
        return fail(ABX_ERR_INVALID_ARGUMENT, "negative sample or text token count");
    if (!abx::pair_supported(seq, samples, text_tokens) || ids == nullptr)
        return abx_sparse_prefill(q, k, v, bh, seq, ids, log_weights, samples, text_k, text_v, text_tokens, o, lse,
                                  stream);
    if (int st = check_paired(q, k, v, bh, seq, ids, log_weights, samples, text_k, text_v, text_tokens, o, workspace,
                              workspace_bytes))
        return st;
    return check_cuda(abx::launch_prefill_pair(static_cast<const abx::bf16*>(q), static_cast<const abx::bf16*>(k),
                                               static_cast<const abx::bf16*>(v), bh, seq, ids, log_weights, samples,
                                               static_cast<const abx::bf16*>(text_k),
                                               static_cast<const abx::bf16*>(text_v), text_tokens,
                                               static_cast<abx::bf16*>(o), lse, workspace, workspace_bytes, stream),
                      "paired prefill launch");
}

int abx_ipc_handle(const void* ptr, void* handle, size_t* offset) {
    if (ptr == nullptr || handle == nullptr || offset == nullptr)
        return fail(ABX_ERR_INVALID_ARGUMENT, "ptr, handle and offset must be non-null");
    using PfnAddressRange = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
    static const PfnAddressRange address_range = driver_entry<PfnAddressRange>("cuMemGetAddressRange");
    if (address_range == nullptr) return fail(ABX_ERR_CUDA, "cuMemGetAddressRange unavailable in this driver");
    CUdeviceptr base = 0;
    size_t bytes = 0;
    if (address_range(&base, &bytes, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
        return fail(ABX_ERR_INVALID_ARGUMENT, "ptr is not device memory of this process");
    cudaIpcMemHandle_t h;
    if (int st = check_cuda(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)), "cudaIpcGetMemHandle")) return st;
    std::memcpy(handle, &h, sizeof(h));
    *offset = static_cast<size_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
    return ABX_OK;
}

int abx_ipc_open(const void* handle, void** base) {
    if (handle == nullptr || base == nullptr) return fail(ABX_ERR_INVALID_ARGUMENT, "handle and base must be non-null");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    return check_cuda(cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
}

int abx_ipc_close(void* base) {
    if (base == nullptr) return fail(ABX_ERR_INVALID_ARGUMENT, "base must be non-null");
    return check_cuda(cudaIpcCloseMemHandle(base), "cudaIpcCloseMemHandle");
}

int abx_peer_copy(void* dst, const void* src, size_t bytes, abx_stream_t stream) {
    if (dst == nullptr || src == nullptr) return fail(ABX_ERR_INVALID_ARGUMENT, "dst and src must be non-null");
    if (bytes == 0) return ABX_OK;
    return check_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, stream), "peer copy");
}

int abx_sparse_prefill_scatter(const void* q, const void* k, const void* v, int64_t bh, int64_t seq,
                               const int32_t* ids, const float* log_weights, int64_t samples, const void* text_k,
                               const void* text_v, int64_t text_tokens, void* const* outs, int num_outs,
                               int64_t out_head_base, int64_t out_heads, float* lse, void* workspace,
                               size_t workspace_bytes, abx_stream_t stream) {
    if (samples < 0 || text_tokens < 0)
        return fail(ABX_ERR_INVALID_ARGUMENT, "negative sample or text token count");
    if (outs == nullptr || num_outs < 1 || num_outs > abx::kMaxScatterOutputs)
        return fail(ABX_ERR_INVALID_ARGUMENT, "between 1 and %d output buffers are needed (got %d)",
                    abx::kMaxScatterOutputs, num_outs);
    abx::bf16* dsts[abx::kMaxScatterOutputs];
    for (int d = 0; d < num_outs; ++d) {
        if (outs[d] == nullptr || !aligned16(outs[d]))
            return fail(ABX_ERR_INVALID_ARGUMENT, "output buffer %d must be non-null and 16-byte aligned", d);
        dsts[d] = static_cast<abx::bf16*>(outs[d]);
    }
    if (out_head_base < 0 || out_heads < out_head_base + bh)
        return fail(ABX_ERR_INVALID_ARGUMENT, "heads [%lld, %lld) lie outside the %lld-head output",
                    (long long)out_head_base, (long long)(out_head_base + bh), (long long)out_heads);
    if (!abx::pair_supported(seq, samples, text_tokens))
        return fail(ABX_ERR_UNSUPPORTED, "this shape cannot be paired (abx_prefill_workspace_size reports 0)");
    if (int st = check_paired(q, k, v, bh, seq, ids, log_weights, samples, text_k, text_v, text_tokens, outs[0],
                              workspace, workspace_bytes))
        return st;
    if (int st = check_cuda(abx::launch_pair_plan(ids, bh, seq, samples, text_tokens, workspace, workspace_bytes,
                                                  stream),
                            "pair plan launch"))
        return st;
    return check_cuda(abx::launch_pair_prefill(static_cast<const abx::bf16*>(q), static_cast<const abx::bf16*>(k),
                                               static_cast<const abx::bf16*>(v), bh, seq, ids, log_weights, samples,
                                               static_cast<const abx::bf16*>(text_k),
                                               static_cast<const abx::bf16*>(text_v), text_tokens, nullptr, lse,
                                               workspace, workspace_bytes, stream, dsts, num_outs, out_head_base),
                      "scatter prefill launch");
}

int abx_pair_plan(const int32_t* ids, int64_t bh, int64_t seq, int64_t samples, int64_t text_tokens, void* workspace,
                  size_t workspace_bytes, abx_stream_t stream) {
    if (int st = check_qk_shape(bh, seq)) return st;
    if (samples < 0 || text_tokens < 0) return fail(ABX_ERR_INVALID_ARGUMENT, "negative sample or text token count");
    if (!abx::pair_supported(seq, samples, text_tokens))
        return fail(ABX_ERR_UNSUPPORTED, "this shape cannot be paired (abx_prefill_workspace_size reports 0)");
    if (ids == nullptr) return fail(ABX_ERR_INVALID_ARGUMENT, "ids must be non-null");
    if (workspace == nullptr || workspace_bytes < abx::pair_workspace_bytes(bh, seq, samples, text_tokens))
        return fail(ABX_ERR_WORKSPACE, "workspace too small (%zu bytes, need %zu)", workspace_bytes,
                    abx::pair_workspace_bytes(bh, seq, samples, text_tokens));
    return check_cuda(abx::launch_pair_plan(ids, bh, seq, samples, text_tokens, workspace, workspace_bytes, stream),
                      "pair plan launch");
}

int abx_sparse_prefill_paired_planned(const void* q, const void* k, const void* v, int64_t bh, int64_t seq,
                                      const int32_t* ids, const float* log_weights, int64_t samples,
                                      const void* text_k, const void* text_v, int64_t text_tokens, void* o,
                                      float* lse, void* workspace, size_t workspace_bytes, abx_stream_t stream) {
    if (samples < 0 || text_tokens < 0)
        return fail(ABX_ERR_INVALID_ARGUMENT, "negative sample or text token count");
    if (!abx::pair_supported(seq, samples, text_tokens))
        return fail(ABX_ERR_UNSUPPORTED, "this shape cannot be paired (abx_prefill_workspace_size reports 0)");
    if (int st = check_paired(q, k, v, bh, seq, ids, log_weights, samples, text_k, text_v, text_tokens, o, workspace,
                              workspace_bytes))
        return st;
    return check_cuda(abx::launch_pair_prefill(static_cast<const abx::bf16*>(q), static_cast<const abx::bf16*>(k),
                                               static_cast<const abx::bf16*>(v), bh, seq, ids, log_weights, samples,
                                               static_cast<const abx::bf16*>(text_k),
                                               static_cast<const abx::bf16*>(text_v), text_tokens,
                                               static_cast<abx::bf16*>(o), lse, workspace, workspace_bytes, stream),
                      "paired prefill launch");
}

int abx_dense_prefill(const void* q, const void* k, const void* v, int64_t bh, int64_t seq, void* o, float* lse,
                      abx_stream_t stream) {
    if (int st = check_qk_shape(bh, seq)) return st;
    if (!q || !k || !v || !o) return fail(ABX_ERR_INVALID_ARGUMENT, "q, k, v and o must be non-null");
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o))
        return fail(ABX_ERR_INVALID_ARGUMENT, "q, k, v and o must be 16-byte aligned");
    return check_cuda(abx::launch_prefill(static_cast<const abx::bf16*>(q), seq, static_cast<const abx::bf16*>(k),
                                          static_cast<const abx::bf16*>(v), bh, seq, nullptr, nullptr,
                                          seq / abx::kKv4, nullptr, nullptr, 0, static_cast<abx::bf16*>(o), lse,
                                          stream),
                      "prefill launch");
}

int abx_cross_prefill(const void* q, int64_t q_tokens, const void* k, const void* v, int64_t kv_tokens, int64_t bh,
                      const int32_t* ids, const float* log_weights, int64_t samples, const void* text_k,
                      const void* text_v, int64_t text_tokens, void* o, float* lse, abx_stream_t stream) {
    if (bh <= 0 || q_tokens <= 0) return fail(ABX_ERR_INVALID_ARGUMENT, "bad query shape");
    if (kv_tokens < 0 || kv_tokens % abx::kKv4 != 0)
        return fail(ABX_ERR_INVALID_ARGUMENT, "key token count must be a non-negative multiple of 4");
    if (kv_tokens / abx::kKv4 > abx::kMaxFineBlocks)
        return fail(ABX_ERR_UNSUPPORTED, "more than %d key blocks", abx::kMaxFineBlocks);
    if (!q || !o || !aligned16(q) || !aligned16(o))
        return fail(ABX_ERR_INVALID_ARGUMENT, "q and o must be non-null and 16-byte aligned");
    if (samples < 0 || samples > kv_tokens / abx::kKv4)
        return fail(ABX_ERR_INVALID_ARGUMENT, "samples must be in [0, kv_tokens/4] (got %lld)", (long long)samples);
    if (samples > 0 && (!k || !v || !aligned16(k) || !aligned16(v)))
        return fail(ABX_ERR_INVALID_ARGUMENT, "k and v must be non-null and 16-byte aligned");
    if ((ids == nullptr) != (log_weights == nullptr))
        return fail(ABX_ERR_INVALID_ARGUMENT, "ids and log_weights are given together (or neither: dense)");
    if (text_tokens < 0) return fail(ABX_ERR_INVALID_ARGUMENT, "negative text token count");
    if (text_tokens > 0 && (!text_k || !text_v || !aligned16(text_k) || !aligned16(text_v)))
        return fail(ABX_ERR_INVALID_ARGUMENT, "text_k/text_v must be non-null and 16-byte aligned");
    if (samples + (text_tokens + abx::kKv4 - 1) / abx::kKv4 <= 0)
        return fail(ABX_ERR_INVALID_ARGUMENT, "every row needs at least one key");
    return check_cuda(abx::launch_prefill(static_cast<const abx::bf16*>(q), q_tokens,
                                          static_cast<const abx::bf16*>(k), static_cast<const abx::bf16*>(v), bh,
                                          kv_tokens, ids, log_weights, samples,
                                          static_cast<const abx::bf16*>(text_k),
                                          static_cast<const abx::bf16*>(text_v), text_tokens,
                                          static_cast<abx::bf16*>(o), lse, stream),
                      "prefill launch");
}

int abx_selftest_wait_timeout(int64_t limit_cycles, abx_stream_t stream) {
    if (limit_cycles <= 0 || limit_cycles > 4000000000LL)
        return fail(ABX_ERR_INVALID_ARGUMENT, "limit must be in (0, 4e9] cycles");
    abx::wait_selftest_kernel<<<1, 64, 0, stream>>>(static_cast<uint64_t>(limit_cycles), abx::device_error_word());
    return check_cuda(cudaGetLastError(), "self-test launch");
}

}  // extern "C"
