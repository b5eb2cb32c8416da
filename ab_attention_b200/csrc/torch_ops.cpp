// torch.ops.ab_attention: the PyTorch operator layer over the libabx C ABI.
//
// Replaces the reference's pybind module `ab_attention._C` (csrc/bindings.cpp:3-8,
// csrc/ops.h:5-8: `ibcs(q, k) -> scores`, `sip(scores, offsets, ids, logs)`) and
// the sparse prefill its FlashInfer adapter runs (ab_attention/flashinfer_backend.py:
// 164-242), as TORCH_LIBRARY operators callable from Python, C++ and TorchScript.
// Each operator checks its tensors (device, dtype, shape, contiguity) the way the
// reference's TORCH_CHECKs do, allocates outputs and workspaces with the caching
// allocator, and calls the extern "C" entry points of include/abx.h on the current
// CUDA stream; a nonzero status becomes a RuntimeError with libabx's message.
// Only CUDA kernels are registered: a CPU tensor finds no kernel and raises, so
// there is no silent fallback. Meta kernels give the output shapes to tracers.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <cstdint>
#include <tuple>

#include "abx.h"

namespace {

constexpr int64_t kHeadDim = 128;
constexpr int64_t kQueryBlock = 128;

void check_status(int status, const char* what) {
    TORCH_CHECK(status == ABX_OK, what, " failed: ", abx_status_string(status), ": ", abx_last_error());
}

abx_stream_t stream_of(const at::Tensor& t) {
    return reinterpret_cast<abx_stream_t>(c10::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

void expect(const at::Tensor& t, const char* name, at::IntArrayRef shape, at::ScalarType dtype,
            const at::Tensor& like) {
    TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
    TORCH_CHECK(t.device() == like.device(), name, " must be on ", like.device());
    TORCH_CHECK(t.scalar_type() == dtype, name, " must be ", dtype, " (got ", t.scalar_type(), ")");
    TORCH_CHECK(t.sizes() == shape, name, " must have shape ", shape, " (got ", t.sizes(), ")");
    TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}

// [B, H, S, 128] or [BH, S, 128] -> (BH, S)
std::pair<int64_t, int64_t> heads_tokens(const at::Tensor& x, const char* name) {
    TORCH_CHECK(x.dim() == 3 || x.dim() == 4, name, " must be [B, H, S, 128] or [BH, S, 128]");
    TORCH_CHECK(x.size(-1) == kHeadDim, name, " must have head_dim 128");
    const int64_t bh = x.dim() == 4 ? x.size(0) * x.size(1) : x.size(0);
    return {bh, x.size(-2)};
}

int64_t rows_of(int64_t bh, int64_t seq) { return bh * ((seq + kQueryBlock - 1) / kQueryBlock); }

at::Tensor workspace(int64_t bytes, const at::Tensor& like) {
    // 256 bytes of slack: the caching allocator's blocks are 512-byte aligned, the
    // slack keeps a later alignment change from starving the layout
    return at::empty({bytes + 256}, like.options().dtype(at::kByte));
}

void* aligned256(const at::Tensor& ws) {
    const auto p = reinterpret_cast<uintptr_t>(ws.data_ptr());
    return reinterpret_cast<void*>((p + 255) & ~static_cast<uintptr_t>(255));
}

// `_C.ibcs(q, k) -> scores` (csrc/ibcs.cu:549-617): f32 [BH * ceil(S/128), S/4].
at::Tensor ibcs_cuda(const at::Tensor& q, const at::Tensor& k) {
    const auto [bh, seq] = heads_tokens(q, "q");
    expect(q, "q", q.sizes(), at::kBFloat16, q);
    expect(k, "k", q.sizes(), at::kBFloat16, q);
    c10::cuda::CUDAGuard guard(q.device());
    size_t bytes = 0;
    check_status(abx_ibcs_workspace_size(bh, seq, &bytes), "abx_ibcs_workspace_size");
    auto ws = workspace(static_cast<int64_t>(bytes), q);
    auto scores = at::empty({rows_of(bh, seq), seq / 4}, q.options().dtype(at::kFloat));
    check_status(abx_ibcs_scores(q.data_ptr(), k.data_ptr(), bh, seq, scores.data_ptr<float>(), aligned256(ws),
                                 bytes, stream_of(q)),
                 "abx_ibcs_scores");
    return scores;
}

// `_C.sip(scores, offsets, ids, logs)` (csrc/sip.cu:170-199): ids/logs written in place.
void sip_cuda(const at::Tensor& scores, const at::Tensor& offsets, at::Tensor ids, at::Tensor logs) {
    TORCH_CHECK(scores.dim() == 2 && ids.dim() == 2, "expected scores [rows, N] and ids/logs [rows, samples]");
    const int64_t rows = scores.size(0), population = scores.size(1), samples = ids.size(1);
    expect(scores, "scores", {rows, population}, at::kFloat, scores);
    expect(offsets, "offsets", {rows}, at::kFloat, scores);
    expect(ids, "ids", {rows, samples}, at::kInt, scores);
    expect(logs, "logs", {rows, samples}, at::kFloat, scores);
    c10::cuda::CUDAGuard guard(scores.device());
    check_status(abx_sip(scores.data_ptr<float>(), offsets.data_ptr<float>(), rows, population,
                         ids.data_ptr<int32_t>(), logs.data_ptr<float>(), samples, stream_of(scores)),
                 "abx_sip");
}

// build_plan's device work (ab_attention/attention.py:27-82) for given uniforms:
// (ids int32, log_weights f32) [rows, samples].
std::tuple<at::Tensor, at::Tensor> build_plan_cuda(const at::Tensor& q, const at::Tensor& k,
                                                   const at::Tensor& offsets, int64_t samples) {
    const auto [bh, seq] = heads_tokens(q, "q");
    const int64_t rows = rows_of(bh, seq);
    expect(q, "q", q.sizes(), at::kBFloat16, q);
    expect(k, "k", q.sizes(), at::kBFloat16, q);
    expect(offsets, "offsets", {rows}, at::kFloat, q);
    c10::cuda::CUDAGuard guard(q.device());
    size_t bytes = 0;
    check_status(abx_ibcs_workspace_size(bh, seq, &bytes), "abx_ibcs_workspace_size");
    auto ws = workspace(static_cast<int64_t>(bytes), q);
    auto ids = at::empty({rows, samples}, q.options().dtype(at::kInt));
    auto logw = at::empty({rows, samples}, q.options().dtype(at::kFloat));
    check_status(abx_build_plan(q.data_ptr(), k.data_ptr(), bh, seq, offsets.data_ptr<float>(), samples,
                                ids.data_ptr<int32_t>(), logw.data_ptr<float>(), aligned256(ws), bytes, stream_of(q)),
                 "abx_build_plan");
    return {ids, logw};
}

// The HT-weighted sparse prefill (flashinfer_backend.py:164-242 with the
// ABSipAttention shift, :30-58) over [BH, S, 128] q/k/v and a plan [rows,
// samples]: (o bf16 [BH, S, 128], base-2 lse f32 [BH, S]). Two adjacent query
// blocks per CTA when the shape pairs, one otherwise.
std::tuple<at::Tensor, at::Tensor> sparse_prefill_cuda(const at::Tensor& q, const at::Tensor& k,
                                                       const at::Tensor& v, const at::Tensor& ids,
                                                       const at::Tensor& log_weights) {
    TORCH_CHECK(q.dim() == 3, "q must be [batch*heads, tokens, 128]");
    const int64_t bh = q.size(0), seq = q.size(1);
    TORCH_CHECK(ids.dim() == 2, "ids must be [rows, samples]");
    const int64_t samples = ids.size(1), rows = rows_of(bh, seq);
    expect(q, "q", {bh, seq, kHeadDim}, at::kBFloat16, q);
    expect(k, "k", {bh, seq, kHeadDim}, at::kBFloat16, q);
    expect(v, "v", {bh, seq, kHeadDim}, at::kBFloat16, q);
    expect(ids, "ids", {rows, samples}, at::kInt, q);
    expect(log_weights, "log_weights", {rows, samples}, at::kFloat, q);
    c10::cuda::CUDAGuard guard(q.device());
    auto o = at::empty_like(q);
    auto lse = at::empty({bh, seq}, q.options().dtype(at::kFloat));
    size_t bytes = 0;
    check_status(abx_prefill_workspace_size(bh, seq, samples, 0, &bytes), "abx_prefill_workspace_size");
    if (bytes > 0) {
        auto ws = workspace(static_cast<int64_t>(bytes), q);
        check_status(abx_sparse_prefill_paired(q.data_ptr(), k.data_ptr(), v.data_ptr(), bh, seq,
                                               ids.data_ptr<int32_t>(), log_weights.data_ptr<float>(), samples,
                                               nullptr, nullptr, 0, o.data_ptr(), lse.data_ptr<float>(),
                                               aligned256(ws), bytes, stream_of(q)),
                     "abx_sparse_prefill_paired");
    } else {
        check_status(abx_sparse_prefill(q.data_ptr(), k.data_ptr(), v.data_ptr(), bh, seq, ids.data_ptr<int32_t>(),
                                        log_weights.data_ptr<float>(), samples, nullptr, nullptr, 0, o.data_ptr(),
                                        lse.data_ptr<float>(), stream_of(q)),
                     "abx_sparse_prefill");
    }
    return {o, lse};
}

// ---- shapes for tracers (no data, no kernels) ----------------------------------------

at::Tensor ibcs_meta(const at::Tensor& q, const at::Tensor& k) {
    const auto [bh, seq] = heads_tokens(q, "q");
    return at::empty({rows_of(bh, seq), seq / 4}, q.options().dtype(at::kFloat));
}

void sip_meta(const at::Tensor&, const at::Tensor&, at::Tensor, at::Tensor) {}

std::tuple<at::Tensor, at::Tensor> build_plan_meta(const at::Tensor& q, const at::Tensor&, const at::Tensor&,
                                                   int64_t samples) {
    const auto [bh, seq] = heads_tokens(q, "q");
    const int64_t rows = rows_of(bh, seq);
    return {at::empty({rows, samples}, q.options().dtype(at::kInt)),
            at::empty({rows, samples}, q.options().dtype(at::kFloat))};
}

std::tuple<at::Tensor, at::Tensor> sparse_prefill_meta(const at::Tensor& q, const at::Tensor&, const at::Tensor&,
                                                       const at::Tensor&, const at::Tensor&) {
    return {at::empty_like(q), at::empty({q.size(0), q.size(1)}, q.options().dtype(at::kFloat))};
}

}  // namespace

TORCH_LIBRARY(ab_attention, m) {
    m.def("ibcs(Tensor q, Tensor k) -> Tensor");
    m.def("sip(Tensor scores, Tensor offsets, Tensor(a!) ids, Tensor(b!) logs) -> ()");
    m.def("build_plan(Tensor q, Tensor k, Tensor offsets, int samples) -> (Tensor, Tensor)");
    m.def("sparse_prefill(Tensor q, Tensor k, Tensor v, Tensor ids, Tensor log_weights) -> (Tensor, Tensor)");
}

TORCH_LIBRARY_IMPL(ab_attention, CUDA, m) {
    m.impl("ibcs", &ibcs_cuda);
    m.impl("sip", &sip_cuda);
    m.impl("build_plan", &build_plan_cuda);
    m.impl("sparse_prefill", &sparse_prefill_cuda);
}

TORCH_LIBRARY_IMPL(ab_attention, Meta, m) {
    m.impl("ibcs", &ibcs_meta);
    m.impl("sip", &sip_meta);
    m.impl("build_plan", &build_plan_meta);
    m.impl("sparse_prefill", &sparse_prefill_meta);
}
