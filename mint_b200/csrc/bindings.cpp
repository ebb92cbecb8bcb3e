// Python bindings of the mint_b200 sm_100a extension (module mint_b200._C).
#include <torch/extension.h>

#include "host_common.h"

namespace mint {
void gemm_bf16(const at::Tensor& A, const at::Tensor& B, at::Tensor& C, const c10::optional<at::Tensor>& D,
               bool a_kmajor, bool b_kmajor, double alpha, double beta, const c10::optional<at::Tensor>& alpha_t,
               bool accumulate);
std::vector<at::Tensor> rmsnorm_fwd(const at::Tensor& x, const at::Tensor& scale, double eps, int64_t out_code);
std::vector<at::Tensor> rmsnorm_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& rstd,
                                    const at::Tensor& scale, int64_t dx_code);
std::vector<at::Tensor> add_rmsnorm_fwd(const at::Tensor& res, const at::Tensor& a, const at::Tensor& post,
                                        const c10::optional<at::Tensor>& pre, double eps, int64_t y_code);
std::vector<at::Tensor> add_rmsnorm_bwd(const c10::optional<at::Tensor>& dh, const c10::optional<at::Tensor>& dy,
                                        const at::Tensor& a, const at::Tensor& h, const at::Tensor& rstd_a,
                                        const at::Tensor& rstd_h, const at::Tensor& post,
                                        const c10::optional<at::Tensor>& pre);
std::vector<at::Tensor> qk_norm_rope_fwd(const at::Tensor& qkv, int64_t n_q, int64_t n_kv, int64_t Dh,
                                         const at::Tensor& qs, const at::Tensor& ks, const at::Tensor& cos_t,
                                         const at::Tensor& sin_t, int64_t start, double eps, bool use_rope);
std::vector<at::Tensor> qk_norm_rope_bwd(const at::Tensor& dq, const at::Tensor& dk, const at::Tensor& dv,
                                         const at::Tensor& qkv, const at::Tensor& rq, const at::Tensor& rk,
                                         const at::Tensor& qs, const at::Tensor& ks, const at::Tensor& cos_t,
                                         const at::Tensor& sin_t, int64_t n_q, int64_t n_kv, int64_t Dh,
                                         int64_t start, bool use_rope);
at::Tensor geglu_fwd(const at::Tensor& ab);
at::Tensor geglu_bwd(const at::Tensor& dh, const at::Tensor& ab);
at::Tensor embedding_fwd(const at::Tensor& ids, const at::Tensor& w, int64_t start);
at::Tensor embedding_bwd(const at::Tensor& dout, const at::Tensor& ids, int64_t rows, int64_t start);
at::Tensor ce_fused_fwd_bwd(at::Tensor& logits, const at::Tensor& targets, const at::Tensor& mask,
                            const at::Tensor& denom, int64_t valid, int64_t vstart);
std::vector<at::Tensor> ce_row_stats(const at::Tensor& logits, const at::Tensor& targets, int64_t valid,
                                     int64_t vstart);
void ce_grad_inplace(at::Tensor& logits, const at::Tensor& targets, const at::Tensor& mask, const at::Tensor& lse,
                     const at::Tensor& denom, int64_t valid, int64_t vstart);
void adamw_step(at::Tensor& p, const at::Tensor& g, at::Tensor& m, at::Tensor& v, double lr, double b1, double b2,
                double eps, double wd, int64_t step);
std::vector<at::Tensor> flash_attn_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                       const c10::optional<at::Tensor>& doc, bool causal, int64_t window,
                                       double scale, const c10::optional<at::Tensor>& dbounds);
std::vector<at::Tensor> flash_attn_bwd(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k,
                                       const at::Tensor& v, const at::Tensor& o, const at::Tensor& lse,
                                       const c10::optional<at::Tensor>& doc, bool causal, int64_t window,
                                       double scale, const c10::optional<at::Tensor>& dbounds);
at::Tensor doc_bounds(const at::Tensor& doc);
void zero_reduce_scatter(const std::vector<int64_t>& bucket_ptrs, at::Tensor& shard, double scale,
                         const c10::optional<at::Tensor>& sumsq, const std::vector<int64_t>& flag_ptrs,
                         const at::Tensor& flags_local, int64_t rank, int64_t world, int64_t seq);
void zero_all_gather(const at::Tensor& shard, const std::vector<int64_t>& bucket_ptrs, int64_t rank, int64_t world);
void zero_barrier(const std::vector<int64_t>& flag_ptrs, const at::Tensor& flags_local, int64_t rank, int64_t world,
                  int64_t seq);
void gemm_ag(const at::Tensor& A, const at::Tensor& B, at::Tensor& C, bool b_kmajor, const std::vector<int64_t>& src_ptrs,
             const at::Tensor& arrive, const std::vector<int64_t>& arrive_peers, at::Tensor& rowflag, at::Tensor& claim,
             int64_t rank, int64_t world, int64_t seg, int64_t seq);
void gemm_rs(const at::Tensor& A, const at::Tensor& B, at::Tensor& out, bool b_kmajor,
             const std::vector<int64_t>& push_ptrs, const at::Tensor& recv, const std::vector<int64_t>& flag_ptrs,
             const at::Tensor& flags, const at::Tensor& arrive, const std::vector<int64_t>& arrive_peers, int64_t rank,
             int64_t world, int64_t seg, int64_t seq);
}  // namespace mint

static int64_t read_status(bool reset) {
  int dev = 0;
  MINT_CUDA_CHECK(cudaGetDevice(&dev));
  return static_cast<int64_t>(mint::read_status_word(dev, reset));
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "mint_b200 sm_100a kernels";
  m.def("read_status", &read_status, "read (and optionally clear) this device's kernel status word",
        py::arg("reset") = false);
  m.def("gemm", &mint::gemm_bf16, "C = alpha * op(A) @ op(B) + beta * D (tcgen05)", py::arg("A"), py::arg("B"),
        py::arg("C"), py::arg("D"), py::arg("a_kmajor"), py::arg("b_kmajor"), py::arg("alpha") = 1.0,
        py::arg("beta") = 0.0, py::arg("alpha_t") = py::none(), py::arg("accumulate") = false);
  m.def("launch_count", &mint::launch_count, "kernels launched by this extension so far");
  m.def("rmsnorm_fwd", &mint::rmsnorm_fwd);
  m.def("rmsnorm_bwd", &mint::rmsnorm_bwd);
  m.def("add_rmsnorm_fwd", &mint::add_rmsnorm_fwd);
  m.def("add_rmsnorm_bwd", &mint::add_rmsnorm_bwd);
  m.def("qk_norm_rope_fwd", &mint::qk_norm_rope_fwd);
  m.def("qk_norm_rope_bwd", &mint::qk_norm_rope_bwd);
  m.def("geglu_fwd", &mint::geglu_fwd);
  m.def("geglu_bwd", &mint::geglu_bwd);
  m.def("embedding_fwd", &mint::embedding_fwd);
  m.def("embedding_bwd", &mint::embedding_bwd);
  m.def("ce_fused_fwd_bwd", &mint::ce_fused_fwd_bwd);
  m.def("ce_row_stats", &mint::ce_row_stats);
  m.def("ce_grad_inplace", &mint::ce_grad_inplace);
  m.def("adamw_step", &mint::adamw_step);
  m.def("flash_attn_fwd", &mint::flash_attn_fwd, "tcgen05 FlashAttention forward -> (o, lse)", py::arg("q"),
        py::arg("k"), py::arg("v"), py::arg("doc"), py::arg("causal"), py::arg("window"), py::arg("scale"),
        py::arg("dbounds") = py::none());
  m.def("flash_attn_bwd", &mint::flash_attn_bwd, "tcgen05 FlashAttention backward -> (dq, dk, dv)",
        py::arg("dout"), py::arg("q"), py::arg("k"), py::arg("v"), py::arg("o"), py::arg("lse"), py::arg("doc"),
        py::arg("causal"), py::arg("window"), py::arg("scale"), py::arg("dbounds") = py::none());
  m.def("gemm_ag", &mint::gemm_ag, "tensor-parallel all-gather of A's rows fused into a CTA-pair tcgen05 GEMM");
  m.def("gemm_rs", &mint::gemm_rs, "CTA-pair tcgen05 GEMM with the reduce-scatter of its output rows fused in");
  m.def("zero_reduce_scatter", &mint::zero_reduce_scatter,
        "ZeRO gradient reduce-scatter over NVLink peer memory, 1/dp scale and squared norm fused");
  m.def("zero_all_gather", &mint::zero_all_gather, "ZeRO parameter all-gather: push this rank's shard to every peer");
  m.def("zero_barrier", &mint::zero_barrier, "stream-ordered barrier of a ZeRO group over NVLink peer flags");
  m.def("doc_bounds", &mint::doc_bounds, "[B, T, 2] int32 document run [start, end) of every token");
}
