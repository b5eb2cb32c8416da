// Python bindings for the test-only reference harness (see ref_ibcs_harness.cu).
// ORACLE INFRASTRUCTURE: never linked into the shipped library.
#include <torch/extension.h>

#include <tuple>

torch::Tensor ibcs_cuda(torch::Tensor q, torch::Tensor k);
void sip_cuda(torch::Tensor scores, torch::Tensor offsets, torch::Tensor ids, torch::Tensor logs);

namespace abx_ref {
std::tuple<torch::Tensor, torch::Tensor> cluster(torch::Tensor q);
std::tuple<torch::Tensor, torch::Tensor, torch::Tensor> cluster_assignments(torch::Tensor q);
torch::Tensor pool(torch::Tensor k);
std::tuple<torch::Tensor, torch::Tensor, torch::Tensor> lse(torch::Tensor packed_q, torch::Tensor packed_k);
torch::Tensor scores(torch::Tensor lse, torch::Tensor pops, torch::Tensor mx, torch::Tensor den);
}  // namespace abx_ref

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
    m.def("ibcs", &ibcs_cuda, "reference ibcs_cuda (csrc/ibcs.cu:549)");
    m.def("sip", &sip_cuda, "reference sip_cuda (csrc/sip.cu:170)");
    m.def("cluster", &abx_ref::cluster, "reference cluster_queries_kernel (csrc/ibcs.cu:106)");
    m.def("cluster_assignments", &abx_ref::cluster_assignments,
          "reference cluster_queries_kernel with its shared-memory assignments read out (test hook)");
    m.def("pool", &abx_ref::pool, "reference pool_keys_kernel (csrc/ibcs.cu:244)");
    m.def("lse", &abx_ref::lse, "reference ibcs_lse_kernel (csrc/ibcs.cu:370)");
    m.def("scores", &abx_ref::scores, "reference ibcs_scores_kernel (csrc/ibcs.cu:495)");
}
