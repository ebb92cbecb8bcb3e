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
                double eps, double wd, int64_t step, const c10::optional<at::Tensor>& gscale);
void normuon_prep(const at::Tensor& gptrs, at::Tensor& mb, at::Tensor& sumsq, int64_t per, double mu,
                  const c10::optional<at::Tensor>& gscale);
void normuon_cast(const at::Tensor& gptrs, const at::Tensor& sumsq, at::Tensor& X);
at::Tensor normuon_stats(const at::Tensor& X, bool tall);
void normuon_scale(const at::Tensor& partial, at::Tensor& v2, at::Tensor& scale, int64_t red, double beta2);
void normuon_apply(const at::Tensor& X, const at::Tensor& scale, const at::Tensor& pptrs, int64_t r0, int64_t c0,
                   int64_t rs, int64_t cs, bool tall, double lr, double wd, const c10::optional<at::Tensor>& peer_ptrs,
                   int64_t rank, int64_t world);
void gemm_geglu_fwd(const at::Tensor& X, const at::Tensor& W12, at::Tensor& AB, at::Tensor& H);
void gemm_geglu_bwd(const at::Tensor& DY, const at::Tensor& W3, const at::Tensor& AB, at::Tensor& DAB);
void zero_adamw_push(at::Tensor& p, const at::Tensor& g, at::Tensor& m, at::Tensor& v, double lr, double b1,
                     double b2, double eps, double wd, int64_t step, const c10::optional<at::Tensor>& gscale,
                     const std::vector<int64_t>& bucket_ptrs, int64_t rank, int64_t world);
void sumsq_multi(const at::Tensor& ptrs, const at::Tensor& sizes, at::Tensor& out, int64_t max_len);
void clip_coef(const at::Tensor& sumsq, double max_norm, at::Tensor& coef, at::Tensor& norm);
void cast_multi(const at::Tensor& src, const at::Tensor& dst, const at::Tensor& sizes, int64_t max_len);
at::Tensor exp2_poly_eval(const at::Tensor& x);
std::vector<at::Tensor> flash_attn_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                       const c10::optional<at::Tensor>& doc, bool causal, int64_t window,
                                       double scale, const c10::optional<at::Tensor>& dbounds);
std::vector<at::Tensor> flash_attn_bwd(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k,
                                       const at::Tensor& v, const at::Tensor& o, const at::Tensor& lse,
                                       const c10::optional<at::Tensor>& doc, bool causal, int64_t window,
                                       double scale, const c10::optional<at::Tensor>& dbounds);
at::Tensor doc_bounds(const at::Tensor& doc);
at::Tensor decode_attention(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, bool causal,
                            int64_t window, double scale);
at::Tensor flash_attn_fwd_trace();
at::Tensor flash_attn_bwd_trace();
void zero_reduce_scatter(const std::vector<int64_t>& bucket_ptrs, at::Tensor& shard, double scale,
                         const c10::optional<at::Tensor>& sumsq, const std::vector<int64_t>& flag_ptrs,
                         const at::Tensor& flags_local, int64_t rank, int64_t world, int64_t seq);
void zero_all_gather(const at::Tensor& shard, const std::vector<int64_t>& bucket_ptrs, int64_t rank, int64_t world);
void zero_gather_pull(const std::vector<int64_t>& shard_ptrs, at::Tensor& full, int64_t rank, int64_t world);
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

static void set_wait_limit(int64_t ns) {
  int dev = 0;
  MINT_CUDA_CHECK(cudaGetDevice(&dev));
  mint::set_wait_limit_ns(dev, static_cast<uint64_t>(ns));
}

static int64_t get_wait_limit() {
  int dev = 0;
  MINT_CUDA_CHECK(cudaGetDevice(&dev));
  return static_cast<int64_t>(mint::wait_limit_ns(dev));
}

// The current device's status word as a 1-element int32 CUDA tensor (no copy; the block lives
// until the process exits), so the host can snapshot it with an asynchronous copy each step.
static at::Tensor status_tensor() {
  int dev = 0;
  MINT_CUDA_CHECK(cudaGetDevice(&dev));
  uint32_t* p = mint::status_ptr(dev);
  return at::from_blob(p, {1}, at::TensorOptions().dtype(at::kInt).device(at::kCUDA, dev));
}

// Copy `height` rows of `width` bytes from src (row pitch spitch bytes) to dst (pitch dpitch) on the
// current stream: the sequence shard of a tensor-parallel rank into its slots of the gathered
// buffer (one strided 2-D copy instead of an elementwise kernel).
static void copy_rows_2d(const at::Tensor& dst, int64_t dst_offset_bytes, int64_t dpitch, const at::Tensor& src,
                         int64_t spitch, int64_t width, int64_t height) {
  MINT_CHECK(dst.is_cuda() && src.is_cuda(), "copy_rows_2d needs CUDA tensors");
  MINT_CHECK(width <= dpitch && width <= spitch && height >= 0, "copy_rows_2d: bad geometry");
  MINT_CHECK(dst_offset_bytes + (height - 1) * dpitch + width <= dst.numel() * dst.element_size(),
             "copy_rows_2d: destination too small");
  MINT_CHECK((height - 1) * spitch + width <= src.numel() * src.element_size(), "copy_rows_2d: source too small");
  if (height == 0 || width == 0) return;
  c10::cuda::CUDAGuard g(dst.device());
  char* d = static_cast<char*>(dst.data_ptr()) + dst_offset_bytes;
  MINT_CUDA_CHECK(cudaMemcpy2DAsync(d, dpitch, src.data_ptr(), spitch, width, height, cudaMemcpyDeviceToDevice,
                                    at::cuda::getCurrentCUDAStream()));
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "mint_b200 sm_100a kernels";
  m.def("read_status", &read_status, "read (and optionally clear) this device's kernel status word",
        py::arg("reset") = false);
  m.def("set_wait_limit_ns", &set_wait_limit, "bound (ns) of every spin-wait in this device's kernels");
  m.def("wait_limit_ns", &get_wait_limit, "current spin-wait bound (ns) of this device's kernels");
  m.def("status_tensor", &status_tensor, "this device's kernel status word as a 1-element int32 tensor");
  m.def("copy_rows_2d", &copy_rows_2d, "strided 2-D device copy of rows (cudaMemcpy2DAsync)");
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
  m.def("adamw_step", &mint::adamw_step, "fused AdamW over a flat fp32 shard", py::arg("p"), py::arg("g"),
        py::arg("m"), py::arg("v"), py::arg("lr"), py::arg("b1"), py::arg("b2"), py::arg("eps"), py::arg("wd"),
        py::arg("step"), py::arg("gscale") = py::none());
  m.def("normuon_prep", &mint::normuon_prep, "NorMuon momentum + Nesterov + per-matrix squared norm (in place)");
  m.def("normuon_cast", &mint::normuon_cast, "NorMuon Frobenius normalization to the bf16 Polar-Express input");
  m.def("normuon_stats", &mint::normuon_stats, "row (tall) or column sums of squares of the orthogonalized stack");
  m.def("normuon_scale", &mint::normuon_scale, "NorMuon second moment update and per-row/column step scale");
  m.def("normuon_apply", &mint::normuon_apply,
        "NorMuon update with cautious weight decay through a pointer table; with peer_ptrs the new values are "
        "also stored into every data-parallel peer's copy (ZeRO-2 all-gather fused)",
        py::arg("X"), py::arg("scale"), py::arg("pptrs"), py::arg("r0"), py::arg("c0"), py::arg("rs"), py::arg("cs"),
        py::arg("tall"), py::arg("lr"), py::arg("wd"), py::arg("peer_ptrs") = py::none(), py::arg("rank") = 0,
        py::arg("world") = 1);
  m.def("zero_adamw_push", &mint::zero_adamw_push,
        "ZeRO-2 sharded AdamW with the parameter all-gather fused in (peer stores of the new values)");
  m.def("sumsq_multi", &mint::sumsq_multi, "sum of squares over a table of fp32 segments (accumulated)");
  m.def("clip_coef", &mint::clip_coef, "gradient-norm clip coefficient on the device");
  m.def("cast_multi", &mint::cast_multi, "fp32 -> bf16 copies of a table of segments in one launch");
  m.def("exp2_poly_eval", &mint::exp2_poly_eval, "elementwise 2^x with attention's FMA-pipe polynomial (tests)");
  m.def("flash_attn_fwd", &mint::flash_attn_fwd, "tcgen05 FlashAttention forward -> (o, lse)", py::arg("q"),
        py::arg("k"), py::arg("v"), py::arg("doc"), py::arg("causal"), py::arg("window"), py::arg("scale"),
        py::arg("dbounds") = py::none());
  m.def("flash_attn_bwd", &mint::flash_attn_bwd, "tcgen05 FlashAttention backward -> (dq, dk, dv)",
        py::arg("dout"), py::arg("q"), py::arg("k"), py::arg("v"), py::arg("o"), py::arg("lse"), py::arg("doc"),
        py::arg("causal"), py::arg("window"), py::arg("scale"), py::arg("dbounds") = py::none());
  m.def("gemm_ag", &mint::gemm_ag, "tensor-parallel all-gather of A's rows fused into a CTA-pair tcgen05 GEMM");
  m.def("gemm_geglu_fwd", &mint::gemm_geglu_fwd,
        "fc1||fc2 GEMM with GeGLU in the epilogue: X @ [W1;W2]^T -> ab (kept) and h = gelu_tanh(a) * b");
  m.def("gemm_geglu_bwd", &mint::gemm_geglu_bwd,
        "fc3 input-gradient GEMM with the GeGLU backward in the epilogue: dab from dy @ W3 and the saved ab");
  m.def("gemm_rs", &mint::gemm_rs, "CTA-pair tcgen05 GEMM with the reduce-scatter of its output rows fused in");
  m.def("zero_reduce_scatter", &mint::zero_reduce_scatter,
        "ZeRO gradient reduce-scatter over NVLink peer memory, 1/dp scale and squared norm fused");
  m.def("zero_all_gather", &mint::zero_all_gather, "ZeRO parameter all-gather: push this rank's shard to every peer");
  m.def("zero_gather_pull", &mint::zero_gather_pull, "ZeRO-3 parameter gather: pull every rank's shard over NVLink");
  m.def("zero_barrier", &mint::zero_barrier, "stream-ordered barrier of a ZeRO group over NVLink peer flags");
  m.def("flash_attn_fwd_trace", &mint::flash_attn_fwd_trace,
        "MINT_FA_TRACE=1 diagnostics: clock64 stamps of the last forward's longest query tile");
  m.def("flash_attn_bwd_trace", &mint::flash_attn_bwd_trace,
        "MINT_FA_TRACE=1 diagnostics: clock64 stamps of the last backward's key tile 0");
  m.def("decode_attention", &mint::decode_attention,
        "split-KV attention of a few query rows against a KV cache prefix (bottom-right causal, window)");
  m.def("doc_bounds", &mint::doc_bounds, "[B, T, 2] int32 document run [start, end) of every token");
}
