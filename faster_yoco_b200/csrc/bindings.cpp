// Python bindings of the sm_100a extension (faster_yoco_b200._C).
#include <torch/extension.h>

#include <mutex>
#include <unordered_map>

#include "common/host.h"

namespace fyb {

void gemm(const at::Tensor& A, const at::Tensor& B, at::Tensor& C, bool a_mn, bool b_mn,
          const c10::optional<at::Tensor>& R);
void gemm_pair(const at::Tensor& A, const at::Tensor& B, at::Tensor& C, bool a_mn, bool b_mn,
               const c10::optional<at::Tensor>& R, int64_t bn, int64_t splits);
int64_t gemm_sq(const at::Tensor& A, const at::Tensor& B, at::Tensor& C, bool accumulate, at::Tensor& sq_part);
int64_t gemm_sq_slots(int64_t M, int64_t N, int64_t K);
std::vector<int64_t> gemm_route(int64_t M, int64_t N, int64_t K);
void gemm_rope(const at::Tensor& A, const at::Tensor& B, at::Tensor& C, const at::Tensor& cos_t,
               const at::Tensor& sin_t, int64_t L, int64_t rot_cols, int64_t bn);
std::vector<at::Tensor> gemm_swiglu(const at::Tensor& A, const at::Tensor& B);
void gemm_swiglu_bwd(const at::Tensor& G, const at::Tensor& W, bool w_mn, const at::Tensor& U, at::Tensor& dU);
void gemm_gather(const at::Tensor& A, const at::Tensor& B, at::Tensor& C, const at::Tensor& flat,
                 const at::Tensor& peers, int64_t seg, int64_t chunk, int64_t rank, int64_t bn,
                 const c10::optional<at::Tensor>& cos_t, const c10::optional<at::Tensor>& sin_t, int64_t L,
                 int64_t rot_cols, const c10::optional<at::Tensor>& residual);
std::vector<at::Tensor> gemm_gather_swiglu(const at::Tensor& A, const at::Tensor& B, const at::Tensor& flat,
                                           const at::Tensor& peers, int64_t seg, int64_t chunk, int64_t rank);
void gemm_scatter(const at::Tensor& A, const at::Tensor& B, at::Tensor& C, bool accumulate, const at::Tensor& grad_flat,
                  const at::Tensor& bases, int64_t seg, int64_t rank, int64_t chunk);
std::vector<at::Tensor> rms_norm_fwd(const at::Tensor& x, const c10::optional<at::Tensor>& w, double eps);
std::vector<at::Tensor> rms_norm_bwd(const at::Tensor& dy, const at::Tensor& x, const c10::optional<at::Tensor>& w,
                                     const at::Tensor& rstd, const c10::optional<at::Tensor>& dres);
std::vector<at::Tensor> subln_swiglu_fwd(const at::Tensor& o, const at::Tensor& g, double eps, int64_t D);
std::vector<at::Tensor> subln_swiglu_bwd(const at::Tensor& dout, const at::Tensor& o, const at::Tensor& g,
                                         const at::Tensor& rstd, int64_t D, const c10::optional<at::Tensor>& dg_out);
at::Tensor swiglu_fwd(const at::Tensor& x, const at::Tensor& y);
std::vector<at::Tensor> swiglu_bwd(const at::Tensor& x, const at::Tensor& y, const at::Tensor& g,
                                   const c10::optional<at::Tensor>& dx_out, const c10::optional<at::Tensor>& dy_out);
at::Tensor gate_cumsum_fwd(const at::Tensor& y, int64_t B, int64_t L, double normalizer, bool chunk_local);
void gate_cumsum_bwd(const at::Tensor& dg, const at::Tensor& y, at::Tensor& dy, double normalizer);
at::Tensor rope_fwd(const at::Tensor& x, const at::Tensor& cos_t, const at::Tensor& sin_t, bool conj, bool neox);
at::Tensor embedding_fwd(const at::Tensor& tok, const at::Tensor& w, double scale);
at::Tensor embedding_bwd(const at::Tensor& tok, const at::Tensor& dy, int64_t V, double scale,
                         const c10::optional<at::Tensor>& out);
std::vector<at::Tensor> ce_fwd(const at::Tensor& logits, const at::Tensor& target, int64_t ignore);
at::Tensor ce_bwd(const at::Tensor& logits, const at::Tensor& target, const at::Tensor& lse, const at::Tensor& grad,
                  int64_t ignore, const c10::optional<at::Tensor>& out);
void adam_step(at::Tensor& p32, const at::Tensor& g16, at::Tensor& m, at::Tensor& v, at::Tensor& p16,
               const at::Tensor& hyper, const at::Tensor& factor, double b1, double b2, double eps, double wd,
               bool adamw, int64_t chunk, int64_t world, int64_t rank);
void adam_push(at::Tensor& p32, const at::Tensor& g16, at::Tensor& m, at::Tensor& v, at::Tensor& p16,
               const at::Tensor& hyper, const at::Tensor& factor, double b1, double b2, double eps, double wd,
               bool adamw, const std::vector<int64_t>& peer_params, int64_t peer_off, int64_t rank, int64_t chunk);
at::Tensor sq_norm(const at::Tensor& x);
at::Tensor sq_norm_ranges(const at::Tensor& x, const at::Tensor& chunks);
std::vector<at::Tensor> attention_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, bool causal,
                                      int64_t window, double scale);
std::vector<at::Tensor> attention_bwd(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k,
                                      const at::Tensor& v, const at::Tensor& o, const at::Tensor& lse, bool causal,
                                      int64_t window, double scale, const c10::optional<at::Tensor>& dq_out,
                                      const c10::optional<at::Tensor>& dk_out, const c10::optional<at::Tensor>& dv_out,
                                      const c10::optional<at::Tensor>& rope_cos,
                                      const c10::optional<at::Tensor>& rope_sin, bool rope_q, bool rope_k);
at::Tensor retention_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& gcum);
at::Tensor retention_chunk_cumsum(const at::Tensor& g);
std::vector<at::Tensor> retention_chunk_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                            const at::Tensor& gloc, const c10::optional<at::Tensor>& state_in,
                                            bool want_state);
at::Tensor retention_chunk_state(const at::Tensor& k, const at::Tensor& v, const at::Tensor& gloc,
                                 const c10::optional<at::Tensor>& state_in);
std::vector<at::Tensor> retention_chunk_bwd(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k,
                                            const at::Tensor& v, const at::Tensor& gloc, const at::Tensor& states,
                                            const c10::optional<at::Tensor>& dstate_out, bool want_dstate_in,
                                            bool has_state_in, const c10::optional<at::Tensor>& dq_out,
                                            const c10::optional<at::Tensor>& dk_out,
                                            const c10::optional<at::Tensor>& dv_out,
                                            const c10::optional<at::Tensor>& rope_cos,
                                            const c10::optional<at::Tensor>& rope_sin, bool want_dgate);
at::Tensor retention_decode(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& g,
                            at::Tensor& state);
std::vector<at::Tensor> retention_bwd(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k,
                                      const at::Tensor& v, const at::Tensor& gcum, const at::Tensor& o,
                                      const c10::optional<at::Tensor>& dq_out, const c10::optional<at::Tensor>& dk_out,
                                      const c10::optional<at::Tensor>& dv_out,
                                      const c10::optional<at::Tensor>& rope_cos,
                                      const c10::optional<at::Tensor>& rope_sin);
std::vector<at::Tensor> ipc_alloc(int64_t nbytes);
int64_t ipc_open(const at::Tensor& handle_bytes);
void ipc_close(int64_t ptr);
void flag_barrier(const std::vector<int64_t>& peer_flags, const at::Tensor& my_flags, const at::Tensor& counters,
                  int64_t rank, int64_t slot);
void reduce_owner(const std::vector<int64_t>& peer_grads, at::Tensor& out, int64_t base, int64_t n, at::Tensor& part,
                  at::Tensor& sq, int64_t chunk, int64_t rank);
void gather_segments(const std::vector<int64_t>& peer_params, at::Tensor& dst, const at::Tensor& segs, int64_t rank,
                     int64_t ctas);
void sum_partials(const at::Tensor& part, at::Tensor& out);
void push_bucket(const at::Tensor& src, const std::vector<int64_t>& peer_dst, const std::vector<int64_t>& peer_arrive,
                 const at::Tensor& ranges, int64_t bucket, int64_t rank, int64_t ctas);
void wait_arrivals(const at::Tensor& arrive, at::Tensor& expected, int64_t bucket, int64_t increment);
void peer_copy(int64_t dst, int64_t src, int64_t nbytes);
void signal_peer(int64_t counter_base, int64_t index);
void push_grads(const at::Tensor& grad, const std::vector<int64_t>& peer_staging,
                const std::vector<int64_t>& peer_arrive, const at::Tensor& pieces, int64_t bucket, int64_t rank,
                int64_t seg, int64_t ctas, int64_t chunk);
void reduce_staged(at::Tensor& grad, const at::Tensor& staging, const at::Tensor& ranges, int64_t world, int64_t rank,
                   int64_t seg, at::Tensor& part, int64_t ctas, int64_t chunk);
void reduce_compact(at::Tensor& grad, const at::Tensor& staging, int64_t n, int64_t world, int64_t rank, int64_t seg,
                    int64_t chunk, at::Tensor& part, int64_t ctas);
void zero_staged(at::Tensor& staging, const at::Tensor& ranges, int64_t world, int64_t rank, int64_t seg,
                 int64_t ctas);
void embedding_bwd_scatter(const at::Tensor& tok, const at::Tensor& dy, double scale, at::Tensor& slot,
                           const at::Tensor& grad_flat, const at::Tensor& bases, int64_t seg, int64_t rank,
                           int64_t chunk);
void push_range(const at::Tensor& src, const std::vector<int64_t>& peer_dst, int64_t off, int64_t n, int64_t rank,
                int64_t ctas, int64_t chunk);
void mailbox_put(const std::vector<int64_t>& peer_boxes, const at::Tensor& vals, int64_t rank,
                 const at::Tensor& counter);
void mailbox_sum(const at::Tensor& box, at::Tensor& out, int64_t world, at::Tensor& counter);

// one status word per device, allocated once (zero = ok)
int* status_ptr() {
  static std::mutex mu;
  static std::unordered_map<int, int*> ptrs;
  int dev;
  FYB_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(mu);
  auto it = ptrs.find(dev);
  if (it != ptrs.end()) return it->second;
  int* p = nullptr;
  FYB_CUDA(cudaMalloc(&p, 4 * sizeof(int)));
  FYB_CUDA(cudaMemset(p, 0, 4 * sizeof(int)));
  bind_bounds_gemm(p);
  bind_bounds_elementwise(p);
  bind_bounds_comm(p);
  ptrs[dev] = p;
  return p;
}

at::Tensor status_tensor() {
  int dev;
  FYB_CUDA(cudaGetDevice(&dev));
  auto opts = at::TensorOptions().dtype(at::kInt).device(at::kCUDA, dev);
  return at::from_blob(status_ptr(), {4}, opts);
}

}  // namespace fyb

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "faster_yoco_b200 sm_100a kernels";
  m.def("gemm", &fyb::gemm, "C = A @ B^T on tcgen05 (operands K-major or MN-major)", py::arg("A"), py::arg("B"),
        py::arg("C"), py::arg("a_mn_major"), py::arg("b_mn_major"), py::arg("residual") = py::none());
  m.def("gemm_pair", &fyb::gemm_pair, "C = A @ B^T on CTA pairs (tcgen05.mma.cta_group::2, 256 x bn tiles)",
        py::arg("A"), py::arg("B"), py::arg("C"), py::arg("a_mn_major"), py::arg("b_mn_major"),
        py::arg("residual") = py::none(), py::arg("bn") = 256, py::arg("splits") = 1);
  m.def("gemm_rope", &fyb::gemm_rope,
        "C = A @ B^T with the interleaved rotary embedding of the leading rot_cols columns in the epilogue",
        py::arg("A"), py::arg("B"), py::arg("C"), py::arg("cos"), py::arg("sin"), py::arg("L"), py::arg("rot_cols"),
        py::arg("bn") = 256);
  m.def("gemm_swiglu", &fyb::gemm_swiglu,
        "{u, h}: u = A @ [fc1; gate]^T and h = silu(u[:, :f]) * u[:, f:] from one GEMM (SwiGLU epilogue)");
  m.def("gemm_swiglu_bwd", &fyb::gemm_swiglu_bwd,
        "du = SwiGLU backward of (G @ W) against the saved u, computed in the GEMM epilogue", py::arg("G"),
        py::arg("W"), py::arg("w_mn"), py::arg("u"), py::arg("du"));
  m.def("gemm_gather", &fyb::gemm_gather,
        "C = A @ B^T with the ZeRO all-gather of the weight B fused in: the GEMM's gather warps pull B's rows owned by "
        "other ranks from their replicas (peer loads) ahead of the tiles that read them",
        py::arg("A"), py::arg("B"), py::arg("C"), py::arg("flat"), py::arg("peers"), py::arg("seg"),
        py::arg("chunk"), py::arg("rank"), py::arg("bn") = 256, py::arg("cos") = py::none(),
        py::arg("sin") = py::none(), py::arg("L") = 0, py::arg("rot_cols") = 0, py::arg("residual") = py::none());
  m.def("gemm_gather_swiglu", &fyb::gemm_gather_swiglu,
        "{u, h} of the fc1 | gate projection with the weight's all-gather fused in and SwiGLU in the epilogue",
        py::arg("A"), py::arg("B"), py::arg("flat"), py::arg("peers"), py::arg("seg"), py::arg("chunk"),
        py::arg("rank"));
  m.def("gemm_route", &fyb::gemm_route, "kernel choice {0 one-CTA / 1 CTA pair, tile width, splits} for an M x N x K GEMM");
  m.def("gemm_sq", &fyb::gemm_sq,
        "weight gradient dW = A^T B (bf16, optionally accumulated) with fp32 sum-of-squares partials of the stored "
        "values; returns the number of partials", py::arg("A"), py::arg("B"), py::arg("C"), py::arg("accumulate"),
        py::arg("sq_part"));
  m.def("gemm_sq_slots", &fyb::gemm_sq_slots, "partials a gemm_sq call of this shape writes");
  m.def("gemm_scatter", &fyb::gemm_scatter,
        "weight gradient dW = A^T B stored straight into each element's ZeRO owner (own slot or peer staging)",
        py::arg("A"), py::arg("B"), py::arg("C"), py::arg("accumulate"), py::arg("grad_flat"), py::arg("bases"),
        py::arg("seg"), py::arg("rank"), py::arg("chunk") = 0);
  m.def("rms_norm_fwd", &fyb::rms_norm_fwd);
  m.def("rms_norm_bwd", &fyb::rms_norm_bwd, py::arg("dy"), py::arg("x"), py::arg("w"), py::arg("rstd"),
        py::arg("dres") = py::none());
  m.def("subln_swiglu_fwd", &fyb::subln_swiglu_fwd);
  m.def("subln_swiglu_bwd", &fyb::subln_swiglu_bwd, py::arg("dout"), py::arg("o"), py::arg("g"), py::arg("rstd"),
        py::arg("D"), py::arg("dg_out") = py::none());
  m.def("swiglu_fwd", &fyb::swiglu_fwd);
  m.def("swiglu_bwd", &fyb::swiglu_bwd, py::arg("x"), py::arg("y"), py::arg("g"), py::arg("dx_out") = py::none(),
        py::arg("dy_out") = py::none());
  m.def("gate_cumsum_fwd", &fyb::gate_cumsum_fwd, py::arg("y"), py::arg("B"), py::arg("L"), py::arg("normalizer"),
        py::arg("chunk_local") = false);
  m.def("gate_cumsum_bwd", &fyb::gate_cumsum_bwd);
  m.def("rope_fwd", &fyb::rope_fwd, py::arg("x"), py::arg("cos"), py::arg("sin"), py::arg("conj") = false,
        py::arg("neox") = false);
  m.def("embedding_fwd", &fyb::embedding_fwd);
  m.def("embedding_bwd", &fyb::embedding_bwd, py::arg("tok"), py::arg("dy"), py::arg("V"), py::arg("scale"),
        py::arg("out") = py::none());
  m.def("ce_fwd", &fyb::ce_fwd);
  m.def("ce_bwd", &fyb::ce_bwd, py::arg("logits"), py::arg("target"), py::arg("lse"), py::arg("grad"),
        py::arg("ignore"), py::arg("out") = py::none());
  m.def("adam_step", &fyb::adam_step, "Adam (apex expression) on this owner's state + the bf16 parameter copy",
        py::arg("p32"), py::arg("g16"), py::arg("m"), py::arg("v"), py::arg("p16"), py::arg("hyper"),
        py::arg("factor"), py::arg("b1"), py::arg("b2"), py::arg("eps"), py::arg("wd"), py::arg("adamw"),
        py::arg("chunk") = 0, py::arg("world") = 1, py::arg("rank") = 0);
  m.def("adam_push", &fyb::adam_push, "Adam on this owner's segment fused with its all-gather push to every peer",
        py::arg("p32"), py::arg("g16"), py::arg("m"), py::arg("v"), py::arg("p16"), py::arg("hyper"),
        py::arg("factor"), py::arg("b1"), py::arg("b2"), py::arg("eps"), py::arg("wd"), py::arg("adamw"),
        py::arg("peer_params"), py::arg("peer_off"), py::arg("rank"), py::arg("chunk") = 0);
  m.def("sq_norm_ranges", &fyb::sq_norm_ranges, "sum of squares over chunks [n, 2] (start, len <= 65536) of a bf16 buffer");
  m.def("sq_norm", &fyb::sq_norm);
  m.def("attention_fwd", &fyb::attention_fwd);
  m.def("attention_bwd", &fyb::attention_bwd, py::arg("dout"), py::arg("q"), py::arg("k"), py::arg("v"),
        py::arg("o"), py::arg("lse"), py::arg("causal"), py::arg("window"), py::arg("scale"),
        py::arg("dq_out") = py::none(), py::arg("dk_out") = py::none(), py::arg("dv_out") = py::none(),
        py::arg("rope_cos") = py::none(), py::arg("rope_sin") = py::none(), py::arg("rope_q") = false,
        py::arg("rope_k") = false);
  m.def("retention_fwd", &fyb::retention_fwd);
  m.def("retention_chunk_cumsum", &fyb::retention_chunk_cumsum);
  m.def("retention_chunk_fwd", &fyb::retention_chunk_fwd, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("gloc"),
        py::arg("state_in") = py::none(), py::arg("want_state") = false);
  m.def("retention_chunk_state", &fyb::retention_chunk_state, py::arg("k"), py::arg("v"), py::arg("gloc"),
        py::arg("state_in") = py::none());
  m.def("retention_chunk_bwd", &fyb::retention_chunk_bwd, py::arg("dout"), py::arg("q"), py::arg("k"), py::arg("v"),
        py::arg("gloc"), py::arg("states"), py::arg("dstate_out") = py::none(), py::arg("want_dstate_in") = false,
        py::arg("has_state_in") = false, py::arg("dq") = py::none(), py::arg("dk") = py::none(),
        py::arg("dv") = py::none(), py::arg("rope_cos") = py::none(), py::arg("rope_sin") = py::none(),
        py::arg("want_dgate") = false);
  m.def("retention_decode", &fyb::retention_decode);
  m.def("retention_bwd", &fyb::retention_bwd, py::arg("dout"), py::arg("q"), py::arg("k"), py::arg("v"),
        py::arg("gcum"), py::arg("o"), py::arg("dq_out") = py::none(), py::arg("dk_out") = py::none(),
        py::arg("dv_out") = py::none(), py::arg("rope_cos") = py::none(), py::arg("rope_sin") = py::none());
  m.def("ipc_alloc", &fyb::ipc_alloc, "cudaMalloc'd byte buffer + its CUDA IPC handle");
  m.def("ipc_open", &fyb::ipc_open);
  m.def("ipc_close", &fyb::ipc_close);
  m.def("flag_barrier", &fyb::flag_barrier);
  m.def("reduce_owner", &fyb::reduce_owner, py::arg("peer_grads"), py::arg("out"), py::arg("base"), py::arg("n"),
        py::arg("part"), py::arg("sq"), py::arg("chunk") = 0, py::arg("rank") = 0);
  m.def("gather_segments", &fyb::gather_segments);
  m.def("sum_partials", &fyb::sum_partials);
  m.def("push_range", &fyb::push_range, py::arg("src"), py::arg("peer_dst"), py::arg("off"), py::arg("n"),
        py::arg("rank"), py::arg("ctas"), py::arg("chunk") = 0);
  m.def("push_bucket", &fyb::push_bucket);
  m.def("wait_arrivals", &fyb::wait_arrivals);
  m.def("peer_copy", &fyb::peer_copy, "cudaMemcpyAsync of nbytes between (peer) device addresses on the current stream");
  m.def("signal_peer", &fyb::signal_peer, "release-add 1 to counter_base[index] (a peer's counter) on the current stream");
  m.def("push_grads", &fyb::push_grads, py::arg("grad"), py::arg("peer_staging"), py::arg("peer_arrive"),
        py::arg("pieces"), py::arg("bucket"), py::arg("rank"), py::arg("seg"), py::arg("ctas"), py::arg("chunk") = 0);
  m.def("reduce_staged", &fyb::reduce_staged, py::arg("grad"), py::arg("staging"), py::arg("ranges"), py::arg("world"),
        py::arg("rank"), py::arg("seg"), py::arg("part"), py::arg("ctas"), py::arg("chunk") = 0);
  m.def("reduce_compact", &fyb::reduce_compact,
        "owner's segment summed from its gradient buffer and the staging slots (GEMM-fused reduce-scatter)",
        py::arg("grad"), py::arg("staging"), py::arg("n"), py::arg("world"), py::arg("rank"), py::arg("seg"),
        py::arg("chunk"), py::arg("part"), py::arg("ctas"));
  m.def("zero_staged", &fyb::zero_staged, "clear other ranks' staging slots over local ranges [n, 2]",
        py::arg("staging"), py::arg("ranges"), py::arg("world"), py::arg("rank"), py::arg("seg"), py::arg("ctas"));
  m.def("embedding_bwd_scatter", &fyb::embedding_bwd_scatter,
        "embedding weight gradient, touched rows stored at their ZeRO owners", py::arg("tok"), py::arg("dy"),
        py::arg("scale"), py::arg("slot"), py::arg("grad_flat"), py::arg("bases"), py::arg("seg"), py::arg("rank"),
        py::arg("chunk") = 0);
  m.def("mailbox_put", &fyb::mailbox_put);
  m.def("mailbox_sum", &fyb::mailbox_sum);
  m.def("status", &fyb::status_tensor, "device status word of the kernels with bounded waits");
}
