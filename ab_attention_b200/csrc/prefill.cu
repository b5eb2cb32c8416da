// Paged sparse prefill with Horvitz-Thompson weights (replaces FlashInfer's
// fa3 batch prefill + the ABSipAttention variant,
// ab_attention/flashinfer_backend.py:30-58,164-242).
//
// For row = (head, query block), the keys are the KV4 granules named by
// ids[row, :] (4 consecutive tokens each) followed by the always-included text
// granules. Logits are in log2 units: l = (q.k) * 128^-0.5 * log2(e) + w_slot,
// where w_slot = log2(1/pi) is the SIP weight of the granule's slot; output
// o = sum 2^(l-max) v / sum 2^(l-max), lse = max + log2(sum). This is the HT
// ratio estimator of softmax attention.
//
// This is the portable warp-level (mma.sync) kernel: one CTA per row, 8 warps x
// 16 queries, 64-key tiles gathered granule by granule with cp.async into a
// swizzled double buffer, online softmax in registers.
#include "common.cuh"
#include "ibcs.cuh"

#include <cfloat>

namespace abx {
namespace {

constexpr int kPfWarps = 8;
constexpr int kPfThreads = kPfWarps * 32;
constexpr int kPfTileKeys = 64;
constexpr int kPfTileGranules = kPfTileKeys / kKv4;
constexpr int kPfStageChunks = kPfTileKeys * 16;  // 16 KB per operand per stage

struct PrefillArgs {
    const bf16* q;
    const bf16* k;
    const bf16* v;
    const int32_t* ids;   // null: dense (granule id = slot)
    const float* logw;    // null: all weights 0
    const bf16* text_k;
    const bf16* text_v;
    bf16* o;
    float* lse;
    int64_t seq;
    int64_t qb;
    int64_t text_tokens;
    int samples;
    int granules;         // samples + text_tokens / 4
    int fine_blocks;      // seq / 4: valid ids are [0, fine_blocks)
    float kappa;          // 128^-0.5 * log2(e)
    int* error;           // device error word (out-of-range ids)
};

__device__ __forceinline__ int swz(int row, int c) { return row * 16 + (c ^ (row & 7)); }

__global__ __launch_bounds__(kPfThreads) void prefill_kernel(const PrefillArgs args) {
    extern __shared__ __align__(128) uint4 smem[];
    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int g = lane >> 2;
    const int t = lane & 3;
    const int64_t row = blockIdx.x;
    const int64_t head = row / args.qb;
    const int64_t token0 = (row - head * args.qb) * kQueryBlock;
    const int n = static_cast<int>(min(static_cast<int64_t>(kQueryBlock), args.seq - token0));
    const int G = args.granules;
    const int tiles = (G + kPfTileGranules - 1) / kPfTileGranules;
    const int32_t* row_ids = args.ids ? args.ids + row * args.samples : nullptr;
    const float* row_w = args.logw ? args.logw + row * args.samples : nullptr;
    const bf16* k_head = args.k + head * args.seq * kHeadDim;
    const bf16* v_head = args.v + head * args.seq * kHeadDim;
    const bf16* tk_head = args.text_k ? args.text_k + head * args.text_tokens * kHeadDim : nullptr;
    const bf16* tv_head = args.text_v ? args.text_v + head * args.text_tokens * kHeadDim : nullptr;

    auto load_tile = [&](int tile, int stage) {
        uint4* ks = smem + stage * kPfStageChunks;
        uint4* vs = smem + (2 + stage) * kPfStageChunks;
#pragma unroll
        for (int it = 0; it < kPfStageChunks / kPfThreads; ++it) {
            const int idx = it * kPfThreads + tid;
            const int key = idx >> 4;
            const int c = idx & 15;
            const int slot = tile * kPfTileGranules + (key >> 2);
            if (slot < G) {
                const bf16* ksrc;
                const bf16* vsrc;
                if (slot < args.samples) {
                    int64_t id = row_ids ? __ldg(row_ids + slot) : slot;
                    if (id < 0 || id >= args.fine_blocks) {  // never read outside the head
                        raise_device_error(args.error, ABX_ERR_INVALID_ARGUMENT);
                        id = 0;
                    }
                    const int64_t off = (id * kKv4 + (key & 3)) * kHeadDim + c * 8;
                    ksrc = k_head + off;
                    vsrc = v_head + off;
                } else {
                    const int64_t off = (static_cast<int64_t>(slot - args.samples) * kKv4 + (key & 3)) * kHeadDim + c * 8;
                    ksrc = tk_head + off;
                    vsrc = tv_head + off;
                }
                cp_async_16(ks + swz(key, c), ksrc);
                cp_async_16(vs + swz(key, c), vsrc);
            } else {
                ks[swz(key, c)] = make_uint4(0u, 0u, 0u, 0u);
                vs[swz(key, c)] = make_uint4(0u, 0u, 0u, 0u);
            }
        }
    };

    load_tile(0, 0);
    cp_async_commit();

    // Q fragments for this warp's 16 queries (zero past the end of the block).
    uint32_t qa[8][4];
    {
        const int r_lo = warp * 16 + g;
        const int r_hi = r_lo + 8;
        const bf16* qrow_lo = args.q + (head * args.seq + token0 + r_lo) * kHeadDim;
        const bf16* qrow_hi = args.q + (head * args.seq + token0 + r_hi) * kHeadDim;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
            const int col = 16 * kk + 2 * t;
            qa[kk][0] = r_lo < n ? *reinterpret_cast<const uint32_t*>(qrow_lo + col) : 0u;
            qa[kk][1] = r_hi < n ? *reinterpret_cast<const uint32_t*>(qrow_hi + col) : 0u;
            qa[kk][2] = r_lo < n ? *reinterpret_cast<const uint32_t*>(qrow_lo + col + 8) : 0u;
            qa[kk][3] = r_hi < n ? *reinterpret_cast<const uint32_t*>(qrow_hi + col + 8) : 0u;
        }
    }

    float o[16][4];
#pragma unroll
    for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m_run[2] = {-FLT_MAX, -FLT_MAX};
    float l_run[2] = {0.f, 0.f};

    for (int tile = 0; tile < tiles; ++tile) {
        const int stage = tile & 1;
        cp_async_wait<0>();
        __syncthreads();
        if (tile + 1 < tiles) {
            load_tile(tile + 1, stage ^ 1);
            cp_async_commit();
        }
        const uint32_t kbase = smem_addr(smem + stage * kPfStageChunks);
        const uint32_t vbase = smem_addr(smem + (2 + stage) * kPfStageChunks);

        // S = Q K^T for 16 queries x 64 keys.
        float s[8][4];
#pragma unroll
        for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
            for (int np = 0; np < 4; ++np) {
                const int key = np * 16 + (lane >> 4) * 8 + (lane & 7);
                const int c = 2 * kk + ((lane >> 3) & 1);
                uint32_t b[4];
                ldmatrix_x4(b, kbase + swz(key, c) * 16);
                mma_bf16_16816(s[2 * np], qa[kk], b[0], b[1]);
                mma_bf16_16816(s[2 * np + 1], qa[kk], b[2], b[3]);
            }
        }

        // Logits with the per-granule HT shift; padding keys are masked.
        float tile_max[2] = {-FLT_MAX, -FLT_MAX};
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
            const int slot = tile * kPfTileGranules + 2 * nt + (t >> 1);
            const bool live = slot < G;
            const float w = (live && slot < args.samples && row_w) ? __ldg(row_w + slot) : 0.f;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                s[nt][e] = live ? fmaf(s[nt][e], args.kappa, w) : -INFINITY;
            }
            tile_max[0] = fmaxf(tile_max[0], fmaxf(s[nt][0], s[nt][1]));
            tile_max[1] = fmaxf(tile_max[1], fmaxf(s[nt][2], s[nt][3]));
        }
        float rescale[2];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            tile_max[r] = fmaxf(tile_max[r], __shfl_xor_sync(0xffffffffu, tile_max[r], 1));
            tile_max[r] = fmaxf(tile_max[r], __shfl_xor_sync(0xffffffffu, tile_max[r], 2));
            const float m_new = fmaxf(m_run[r], tile_max[r]);
            rescale[r] = exp2f(m_run[r] - m_new);
            m_run[r] = m_new;
            l_run[r] *= rescale[r];
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            o[i][0] *= rescale[0];
            o[i][1] *= rescale[0];
            o[i][2] *= rescale[1];
            o[i][3] *= rescale[1];
        }
        uint32_t pa[4][4];
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
            const float p0 = exp2f(s[nt][0] - m_run[0]);
            const float p1 = exp2f(s[nt][1] - m_run[0]);
            const float p2 = exp2f(s[nt][2] - m_run[1]);
            const float p3 = exp2f(s[nt][3] - m_run[1]);
            l_run[0] += p0 + p1;
            l_run[1] += p2 + p3;
            __nv_bfloat162 lo = __floats2bfloat162_rn(p0, p1);
            __nv_bfloat162 hi = __floats2bfloat162_rn(p2, p3);
            pa[nt >> 1][(nt & 1) * 2 + 0] = *reinterpret_cast<uint32_t*>(&lo);
            pa[nt >> 1][(nt & 1) * 2 + 1] = *reinterpret_cast<uint32_t*>(&hi);
        }

        // O += P V : 16 queries x 128 dims over 64 keys.
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
            for (int dp = 0; dp < 8; ++dp) {
                const int key = kk * 16 + (lane & 15);
                const int c = dp * 2 + (lane >> 4);
                uint32_t b[4];
                ldmatrix_x4_trans(b, vbase + swz(key, c) * 16);
                mma_bf16_16816(o[2 * dp], pa[kk], b[0], b[1]);
                mma_bf16_16816(o[2 * dp + 1], pa[kk], b[2], b[3]);
            }
        }
    }

    // Finalise: quad-reduce the row sums, normalise, store o (bf16) and lse.
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 1);
        l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 2);
    }
    const float inv0 = 1.f / l_run[0];
    const float inv1 = 1.f / l_run[1];
    const int r_lo = warp * 16 + g;
    const int r_hi = r_lo + 8;
    bf16* o_lo = args.o + (head * args.seq + token0 + r_lo) * kHeadDim;
    bf16* o_hi = args.o + (head * args.seq + token0 + r_hi) * kHeadDim;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const int col = i * 8 + 2 * t;
        if (r_lo < n) {
            __nv_bfloat162 v2 = __floats2bfloat162_rn(o[i][0] * inv0, o[i][1] * inv0);
            *reinterpret_cast<__nv_bfloat162*>(o_lo + col) = v2;
        }
        if (r_hi < n) {
            __nv_bfloat162 v2 = __floats2bfloat162_rn(o[i][2] * inv1, o[i][3] * inv1);
            *reinterpret_cast<__nv_bfloat162*>(o_hi + col) = v2;
        }
    }
    if (args.lse != nullptr && t == 0) {
        if (r_lo < n) args.lse[head * args.seq + token0 + r_lo] = m_run[0] + log2f(l_run[0]);
        if (r_hi < n) args.lse[head * args.seq + token0 + r_hi] = m_run[1] + log2f(l_run[1]);
    }
}

}  // namespace

cudaError_t launch_prefill(const bf16* q, const bf16* k, const bf16* v, int64_t bh, int64_t seq,
                           const int32_t* ids, const float* log_weights, int64_t samples,
                           const bf16* text_k, const bf16* text_v, int64_t text_tokens, bf16* o,
                           float* lse, cudaStream_t stream) {
    PrefillArgs args{};
    args.q = q;
    args.k = k;
    args.v = v;
    args.ids = ids;
    args.logw = log_weights;
    args.text_k = text_k;
    args.text_v = text_v;
    args.o = o;
    args.lse = lse;
    args.seq = seq;
    args.qb = ceil_div(seq, kQueryBlock);
    args.text_tokens = text_tokens;
    args.samples = static_cast<int>(samples);
    args.granules = static_cast<int>(samples + text_tokens / kKv4);
    args.fine_blocks = static_cast<int>(seq / kKv4);
    args.kappa = qk_scale_log2();
    args.error = device_error_word();
    const size_t smem = 4 * kPfStageChunks * sizeof(uint4);
    cudaError_t err = cudaFuncSetAttribute(prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem));
    if (err != cudaSuccess) return err;
    const int64_t rows = bh * args.qb;
    prefill_kernel<<<static_cast<unsigned>(rows), kPfThreads, smem, stream>>>(args);
    return cudaGetLastError();
}

}  // namespace abx
