/*
 * abx.h — C ABI of the B200 (sm_100a) AB-Attention sparse-attention hot path.
 *
 * The reference binds its kernels through a pybind11 module (`ab_attention._C`,
 * csrc/bindings.cpp:3-8, csrc/ops.h:5-8) and runs the sparse prefill through
 * FlashInfer (ab_attention/flashinfer_backend.py:164-242). This header is the
 * replacement boundary: plain pointers, sizes and a cudaStream_t, no torch types.
 *
 * Conventions shared by every entry point:
 *   - Tensors are dense, row-major, on the current CUDA device. `bh` is batch*heads,
 *     `seq` the token count; q/k/v are bf16 [bh, seq, 128] (head dim fixed at 128
 *     as in csrc/ibcs.cu:32 and flashinfer_backend.py:19).
 *   - qb = ceil(seq/128) query blocks, F = seq/4 KV4 blocks, rows = bh*qb.
 *   - Every call is asynchronous on `stream` and returns an abx_status; 0 is success.
 *     The caller owns every buffer, including workspaces sized by *_workspace_size.
 *   - bf16 / fp16 buffers are passed as `void*` / `uint16_t*` (raw 16-bit words).
 */
#ifndef ABX_H_
#define ABX_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* abx_stream_t; /* identical to cudaStream_t */

enum abx_status {
  ABX_OK = 0,
  ABX_ERR_INVALID_ARGUMENT = 1, /* null pointer, bad shape or size                      */
  ABX_ERR_UNSUPPORTED = 2,      /* shape outside a kernel limit (F > 32768, smem cap)  */
  ABX_ERR_WORKSPACE = 3,        /* workspace missing, too small or misaligned           */
  ABX_ERR_CUDA = 4,             /* a CUDA runtime call or kernel launch failed          */
  ABX_ERR_DEVICE_TIMEOUT = 5    /* a bounded device-side wait gave up (see abx_device_status) */
};

/* Library identification and error text. abx_last_error() is thread-local. */
int abx_version(void);
const char* abx_status_string(int status);
const char* abx_last_error(void);

/* Sticky device-side error word for the current device (0 = none): set by a
 * kernel whose bounded wait expired. Reading it synchronizes `stream`; pass
 * clear=1 to reset it. */
int abx_device_status(abx_stream_t stream, int clear, int* status_out);

/* Self-test of the device-side failure path (no counterpart in the reference):
 * two warps wait, bounded by limit_cycles SM clock cycles, on an mbarrier that
 * nothing arrives at, one with the polling and one with the suspending form of
 * the library's bounded wait; both give up, the kernel returns normally and the
 * device error word reads ABX_ERR_DEVICE_TIMEOUT. The context stays usable. */
int abx_selftest_wait_timeout(int64_t limit_cycles, abx_stream_t stream);

/* ---------------------------------------------------------------------------
 * IBCS stages (parity entry points). Each mirrors one reference kernel.
 * ------------------------------------------------------------------------- */

/* cluster_queries_kernel (csrc/ibcs.cu:106-238): farthest-first 8-way clustering
 * of each 128-query block. Outputs (any may be NULL except populations):
 *   centroids        bf16 [rows, 8, 128]   bf16_rn(mean of members), 0 if empty
 *   scaled_centroids bf16 [rows, 8, 128]   bf16_rn(centroid * 128^-0.5 * log2 e)
 *                                          (the MMA operand, csrc/ibcs.cu:293-295)
 *   populations      f32  [rows, 8]        member counts (the reference stores fp16)
 *   assignments      i32  [rows, 128]      centroid slot per query, -1 past the end */
int abx_ibcs_cluster(const void* q, int64_t bh, int64_t seq, void* centroids,
                     void* scaled_centroids, float* populations, int32_t* assignments,
                     abx_stream_t stream);

/* pool_keys_kernel (csrc/ibcs.cu:244-266): two representatives per KV4 block,
 * bf16_rn(0.5*(k[4j+2t] + k[4j+2t+1])). pooled: bf16 [bh, F, 2, 128]. */
int abx_ibcs_pool(const void* k, int64_t bh, int64_t seq, void* pooled, abx_stream_t stream);

/* ibcs_lse_kernel (csrc/ibcs.cu:370-489): per (row, centroid, KV4 block) the fp16
 * pair log2-sum-exp of the two scaled centroid.key scores, plus each (row,
 * centroid)'s running normalizer. lse: fp16 [rows, 8, F]; lse_max/lse_den: f32 [rows, 8]. */
int abx_ibcs_lse(const void* scaled_centroids, const void* pooled, int64_t bh, int64_t qb,
                 int64_t fine_blocks, uint16_t* lse, float* lse_max, float* lse_den,
                 abx_stream_t stream);

/* ibcs_scores_kernel (csrc/ibcs.cu:495-538): population-weighted mixture of the
 * eight centroid distributions. scores: f32 [rows, F]. */
int abx_ibcs_mix(const uint16_t* lse, const float* populations, const float* lse_max,
                 const float* lse_den, int64_t rows, int64_t fine_blocks, float* scores,
                 abx_stream_t stream);

/* ---------------------------------------------------------------------------
 * Replacements for the reference native ops.
 * ------------------------------------------------------------------------- */

/* Workspace for abx_ibcs_scores and abx_build_plan (bytes, 256-byte aligned base). */
int abx_ibcs_workspace_size(int64_t bh, int64_t seq, size_t* bytes);

/* `_C.ibcs(q, k) -> scores` (csrc/ibcs.cu:549-617): all four IBCS stages.
 * scores: f32 [rows, F]. */
int abx_ibcs_scores(const void* q, const void* k, int64_t bh, int64_t seq, float* scores,
                    void* workspace, size_t workspace_bytes, abx_stream_t stream);

/* `_C.sip(scores, offsets, ids, logs)` (csrc/sip.cu:170-199): iterative pi=1
 * certainty then systematic sampling without replacement. scores f32 [rows,
 * population], offsets f32 [rows] in [0,1), ids i32 [rows, samples] and
 * log_weights f32 [rows, samples] written in place. 0 < samples < population. */
int abx_sip(const float* scores, const float* offsets, int64_t rows, int64_t population,
            int32_t* ids, float* log_weights, int64_t samples, abx_stream_t stream);

/* build_plan's device work (ab_attention/attention.py:27-82) in one call:
 * IBCS with the mixture fused into SIP, so the per-block scores never reach HBM.
 * ids/log_weights: [rows, samples]. Same results as abx_ibcs_scores + abx_sip. */
int abx_build_plan(const void* q, const void* k, int64_t bh, int64_t seq,
                   const float* offsets, int64_t samples, int32_t* ids, float* log_weights,
                   void* workspace, size_t workspace_bytes, abx_stream_t stream);

/* abx_build_plan without a workspace argument, for callers that cannot call
 * cudaMalloc (device memory owned by another allocator or reserved up front, or
 * a path where cudaMalloc's implicit synchronisation is not acceptable). No
 * counterpart in the reference. It allocates nothing: its scratch is a fixed
 * file-scope device array of abx_static_scratch_bytes() (256 MiB) that every GPU
 * loading libabx holds until exit, so one head of the input must fit in it
 * (about 90k tokens); larger inputs are rejected with ABX_ERR_WORKSPACE. Heads
 * are processed in passes that fit the array. The first call on a device looks
 * up the array's device address (make it before any stream capture). All calls
 * share the array: calls that overlap on the GPU (different streams, or
 * different host threads) race, so serialise them. Results equal abx_build_plan's. */
size_t abx_static_scratch_bytes(void);
int abx_build_plan_static(const void* q, const void* k, int64_t bh, int64_t seq,
                          const float* offsets, int64_t samples, int32_t* ids,
                          float* log_weights, abx_stream_t stream);

/* ---------------------------------------------------------------------------
 * Sparse prefill: replaces flashinfer_backend.paged_attention
 * (ab_attention/flashinfer_backend.py:164-242) and its ABSipAttention variant (:30-58).
 * For each row (bh, query block) the keys are the KV4 blocks ids[row, 0..samples)
 * (local to the head), each with logit shift log_weights[row, slot] in log2 units,
 * followed by `text_tokens` always-included keys from text_k/text_v
 * ([bh, text_tokens, 128], shift 0; NULL when text_tokens == 0).
 *   o   bf16 [bh, seq, 128]
 *   lse f32  [bh, seq] base-2 log-sum-exp of the scaled logits (NULL to skip)
 * ------------------------------------------------------------------------- */
int abx_sparse_prefill(const void* q, const void* k, const void* v, int64_t bh, int64_t seq,
                       const int32_t* ids, const float* log_weights, int64_t samples,
                       const void* text_k, const void* text_v, int64_t text_tokens,
                       void* o, float* lse, abx_stream_t stream);

/* abx_sparse_prefill with two adjacent query blocks of a head per CTA, fed from
 * one gather of the union of their samples (same results up to the order of
 * the floating-point sums). `workspace` (device memory, any alignment) holds the
 * per-pair union lists; abx_prefill_workspace_size() gives its size, 0 when the
 * shape cannot be paired (more than 65,534 slots, or a map of seq/4 slots
 * larger than shared memory), in which case this call is abx_sparse_prefill and
 * ignores the workspace. Same replaced interface as abx_sparse_prefill. */
int abx_prefill_workspace_size(int64_t bh, int64_t seq, int64_t samples, int64_t text_tokens, size_t* bytes);
int abx_sparse_prefill_paired(const void* q, const void* k, const void* v, int64_t bh, int64_t seq,
                              const int32_t* ids, const float* log_weights, int64_t samples,
                              const void* text_k, const void* text_v, int64_t text_tokens,
                              void* o, float* lse, void* workspace, size_t workspace_bytes,
                              abx_stream_t stream);

/* The two launches of abx_sparse_prefill_paired as separate calls (no
 * counterpart in the reference). abx_pair_plan writes each pair's union list
 * for `ids` into the workspace; abx_sparse_prefill_paired_planned runs the
 * prefill from those lists, which must have been written by abx_pair_plan for
 * the same ids, shape and text count (the kernel range-checks every list entry,
 * so stale lists give wrong results and ABX_ERR_INVALID_ARGUMENT, never an
 * out-of-bounds read). A plan reused over several calls (the video schedule
 * keeps a plan for four denoising steps) builds its lists once. Both return
 * ABX_ERR_UNSUPPORTED for a shape abx_prefill_workspace_size reports as 0. */
int abx_pair_plan(const int32_t* ids, int64_t bh, int64_t seq, int64_t samples, int64_t text_tokens,
                  void* workspace, size_t workspace_bytes, abx_stream_t stream);
int abx_sparse_prefill_paired_planned(const void* q, const void* k, const void* v, int64_t bh, int64_t seq,
                                      const int32_t* ids, const float* log_weights, int64_t samples,
                                      const void* text_k, const void* text_v, int64_t text_tokens, void* o,
                                      float* lse, void* workspace, size_t workspace_bytes, abx_stream_t stream);

/* CUDA IPC of an output buffer between the processes of one node (no
 * counterpart in the reference): abx_ipc_handle gives the 64-byte handle of the
 * allocation holding `ptr` and ptr's byte offset in it; another process opens
 * it with abx_ipc_open (the mapping is made for the caller's current device,
 * with peer access enabled to the owner's device) and adds the offset, then
 * closes it with abx_ipc_close. */
int abx_ipc_handle(const void* ptr, void* handle, size_t* offset);
int abx_ipc_open(const void* handle, void** base);
int abx_ipc_close(void* base);

/* Asynchronous copy of `bytes` on `stream`, either address possibly another
 * GPU's (a mapping opened by abx_ipc_open): between GPUs it runs on a copy
 * engine over NVLink and uses no SMs. No counterpart in the reference. */
int abx_peer_copy(void* dst, const void* src, size_t bytes, abx_stream_t stream);

/* The paired prefill (pair plan included) with its output rows written straight
 * into `num_outs` (1..8) copies of the whole layer's output, each [out_heads,
 * seq, 128] bf16, at heads [out_head_base, out_head_base + bh): on several GPUs,
 * one copy per rank, the other ranks' reached through their mapped (CUDA IPC)
 * addresses, so a head-sharded layer needs no all-gather afterwards. No
 * counterpart in the reference (it has no multi-GPU path); it replaces the NCCL
 * all-gather of the sharded outputs. The stores are plain peer stores over
 * NVLink, made visible system-wide before the kernel ends; the caller orders a
 * reader on another GPU after this call with any collective (an all-reduce of
 * one element) issued on `stream` after it. lse (optional) is this call's heads
 * only, [bh, seq]. ABX_ERR_UNSUPPORTED for a shape that cannot be paired. */
int abx_sparse_prefill_scatter(const void* q, const void* k, const void* v, int64_t bh, int64_t seq,
                               const int32_t* ids, const float* log_weights, int64_t samples,
                               const void* text_k, const void* text_v, int64_t text_tokens,
                               void* const* outs, int num_outs, int64_t out_head_base, int64_t out_heads,
                               float* lse, void* workspace, size_t workspace_bytes, abx_stream_t stream);

/* Dense attention through the same prefill kernel (every KV4 block, shift 0):
 * the dense comparator. o / lse as above. */
int abx_dense_prefill(const void* q, const void* k, const void* v, int64_t bh, int64_t seq,
                      void* o, float* lse, abx_stream_t stream);

/* Queries attending to keys of another length: q [bh, q_tokens, 128] against
 * the KV4 granules named by ids ([bh * ceil(q_tokens/128), samples]; NULL ids
 * and log_weights = the first `samples` granules of k/v in order, weight 0)
 * of k, v [bh, kv_tokens, 128], followed by the text keys text_k, text_v
 * [bh, text_tokens, 128] (any count; keys past text_tokens in the last
 * granule are masked). o [bh, q_tokens, 128], lse [bh, q_tokens] (base 2) or
 * NULL. No counterpart entry point in the reference: it covers the
 * HunyuanVideo partitions its video.py:129-151 runs through FlashInfer (text
 * queries over all video + text keys, and the padding partition with
 * samples = 0 and the padding tokens as text keys). */
int abx_cross_prefill(const void* q, int64_t q_tokens, const void* k, const void* v, int64_t kv_tokens, int64_t bh,
                      const int32_t* ids, const float* log_weights, int64_t samples, const void* text_k,
                      const void* text_v, int64_t text_tokens, void* o, float* lse, abx_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* ABX_H_ */
