// Python bindings of the native extension.
#include <torch/extension.h>

int64_t gemm_tma_epilogue(int64_t level);
void gemm_entry(torch::Tensor A, torch::Tensor B, torch::Tensor D, bool a_mn, bool b_mn, int64_t epi,
                c10::optional<torch::Tensor> R, c10::optional<torch::Tensor> alpha,
                c10::optional<torch::Tensor> cos_t, c10::optional<torch::Tensor> sin_t,
                c10::optional<torch::Tensor> D2, int64_t p0, int64_t p1);
std::vector<torch::Tensor> rmsnorm_fwd(torch::Tensor x, torch::Tensor w, double eps);
torch::Tensor rmsnorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor rstd, torch::Tensor dw_acc);
void rope_bwd(torch::Tensor d, torch::Tensor c, torch::Tensor s, int64_t rc, int64_t hd, int64_t sl);
void rope_fwd(torch::Tensor d, torch::Tensor c, torch::Tensor s, int64_t rc, int64_t hd, int64_t sl);
void swiglu_bwd(torch::Tensor da, torch::Tensor gu, torch::Tensor dgu);
torch::Tensor embedding_fwd(torch::Tensor tok, torch::Tensor w, c10::ScalarType out_dtype);
void embedding_bwd(torch::Tensor tok, torch::Tensor dout, torch::Tensor acc);
std::vector<torch::Tensor> cross_entropy_fwd(torch::Tensor logits, torch::Tensor labels, int64_t ignore);
void adamw(torch::Tensor p, torch::Tensor g, torch::Tensor m, torch::Tensor v, torch::Tensor out,
           c10::optional<torch::Tensor> clip, double lr, double b1, double b2, double eps, double wd, int64_t step);
torch::Tensor sumsq(torch::Tensor x);
torch::Tensor sum_small(torch::Tensor x);
std::vector<torch::Tensor> attn_fwd(torch::Tensor qkv, int64_t B, int64_t S, int64_t nq, int64_t nkv, int64_t hd,
                                    double scale, bool legacy);
torch::Tensor attn_bwd(torch::Tensor dO, torch::Tensor qkv, torch::Tensor o, torch::Tensor lse, int64_t B, int64_t S,
                       int64_t nq, int64_t nkv, int64_t hd, double scale, bool legacy);
int64_t device_error();
void gemm_peer_ar(torch::Tensor A, torch::Tensor B, torch::Tensor D, bool b_mn, c10::optional<torch::Tensor> R,
                  c10::optional<torch::Tensor> alpha, std::vector<int64_t> bases, int64_t rank, int64_t stage_off,
                  int64_t flag_off, int64_t epoch, double timeout_s, bool two_shot);
void gemm_peer_rs(torch::Tensor A, torch::Tensor B, torch::Tensor D, bool b_mn, c10::optional<torch::Tensor> R,
                  std::vector<int64_t> bases, int64_t rank, int64_t stage_off, int64_t flag_off, int64_t epoch,
                  double timeout_s, int64_t row0, int64_t rows);
torch::Tensor sym_malloc(int64_t nbytes);
torch::Tensor ipc_handle(torch::Tensor heap);
int64_t ipc_open(torch::Tensor handle);
void ipc_close(int64_t ptr);
void peer_barrier(std::vector<int64_t> bases, int64_t flag_off, int64_t rank, int64_t epoch, double timeout_s);
void peer_all_gather(std::vector<int64_t> bases, int64_t src_off, int64_t shard_bytes, torch::Tensor out);
void peer_all_gather_ce(std::vector<int64_t> bases, int64_t src_off, int64_t shard_bytes, torch::Tensor out,
                        int64_t src_stride, int64_t skip_rank);
int64_t reduce_scatter_blocks(int64_t n);
void peer_reduce_scatter(std::vector<int64_t> bases, int64_t grad_off, int64_t rank, double scale, torch::Tensor out,
                         c10::optional<torch::Tensor> part, int64_t split, double rep_w);
void peer_all_reduce_bf16(std::vector<int64_t> bases, int64_t src_off, c10::optional<torch::Tensor> residual,
                          torch::Tensor out);
void peer_reduce_rows_bf16(std::vector<int64_t> bases, int64_t src_off, int64_t row0, int64_t cols, torch::Tensor out);
void wait_flag_probe(torch::Tensor flag, int64_t target, double timeout_s);
int64_t gemm_ce_blocks(int64_t N);
torch::Tensor tmem_a_operand_check(torch::Tensor A, torch::Tensor B);
void gemm_ag(torch::Tensor A_gathered, torch::Tensor A_local, torch::Tensor B, torch::Tensor D, int64_t epi,
             c10::optional<torch::Tensor> cos_t, c10::optional<torch::Tensor> sin_t, c10::optional<torch::Tensor> D2,
             int64_t p0, int64_t p1, std::vector<int64_t> bases, int64_t rank, int64_t stage_off, int64_t staged_off,
             int64_t epoch, double timeout_s);
void peer_signal(std::vector<int64_t> bases, int64_t flag_off, int64_t rank, int64_t epoch);
void gemm_ce_stats(torch::Tensor h, torch::Tensor w, torch::Tensor labels, torch::Tensor stats, torch::Tensor tgt,
                   int64_t vocab_off, int64_t vocab_total, int64_t ignore);
void gemm_ce_grad(torch::Tensor h, torch::Tensor w, torch::Tensor labels, torch::Tensor lse, torch::Tensor dloss,
                  torch::Tensor inv_n, torch::Tensor out, int64_t vocab_off, int64_t vocab_total, int64_t ignore);
void ce_stats_reduce(torch::Tensor stats, torch::Tensor tgt, torch::Tensor labels, int64_t vocab_off, int64_t v_local,
                     int64_t vocab_total, int64_t ignore, torch::Tensor lse, torch::Tensor row_loss,
                     c10::optional<torch::Tensor> xchg);
void ce_peer_combine(std::vector<int64_t> bases, int64_t off, torch::Tensor labels, int64_t vocab_total, int64_t ignore,
                     torch::Tensor lse, torch::Tensor row_loss);
void ce_loss_finish(torch::Tensor row_loss, torch::Tensor labels, int64_t vocab_total, int64_t ignore,
                    torch::Tensor loss, torch::Tensor inv_n);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sm_100a kernels for B200-native 2-D parallel LLaMA training";
  m.def("gemm", &gemm_entry, "tcgen05 GEMM with fused epilogues");
  m.def("gemm_tma_epilogue", &gemm_tma_epilogue, "TMA-store GEMM epilogue level (0 none, 1 store/accumulate/residual, 2 also RoPE/SwiGLU); returns the previous level");
  m.def("rmsnorm_fwd", &rmsnorm_fwd);
  m.def("rmsnorm_bwd", &rmsnorm_bwd);
  m.def("rope_bwd", &rope_bwd);
  m.def("rope_fwd", &rope_fwd);
  m.def("swiglu_bwd", &swiglu_bwd);
  m.def("embedding_fwd", &embedding_fwd);
  m.def("embedding_bwd", &embedding_bwd);
  m.def("cross_entropy_fwd", &cross_entropy_fwd);
  m.def("adamw", &adamw);
  m.def("sumsq", &sumsq);
  m.def("sum_small", &sum_small, "fixed-order sum of a small fp32 buffer");
  m.def("attn_fwd", &attn_fwd, py::arg("qkv"), py::arg("B"), py::arg("S"), py::arg("nq"), py::arg("nkv"),
        py::arg("hd"), py::arg("scale"), py::arg("legacy") = false);
  m.def("attn_bwd", &attn_bwd, py::arg("dO"), py::arg("qkv"), py::arg("o"), py::arg("lse"), py::arg("B"),
        py::arg("S"), py::arg("nq"), py::arg("nkv"), py::arg("hd"), py::arg("scale"), py::arg("legacy") = false);
  m.def("device_error", &device_error, "read and clear the device error word");
  m.def("gemm_peer_ar", &gemm_peer_ar, "tcgen05 GEMM fused with an NVLink all-reduce over the peer group",
        py::arg("A"), py::arg("B"), py::arg("D"), py::arg("b_mn"), py::arg("R"), py::arg("alpha"), py::arg("bases"),
        py::arg("rank"), py::arg("stage_off"), py::arg("flag_off"), py::arg("epoch"), py::arg("timeout_s"),
        py::arg("two_shot") = false);
  m.def("gemm_peer_rs", &gemm_peer_rs, "tcgen05 GEMM fused with an NVLink reduce-scatter of rows over the peer group");
  m.def("sym_malloc", &sym_malloc, "raw device allocation for a symmetric heap");
  m.def("ipc_handle", &ipc_handle);
  m.def("ipc_open", &ipc_open);
  m.def("ipc_close", &ipc_close);
  m.def("peer_barrier", &peer_barrier);
  m.def("peer_all_gather", &peer_all_gather);
  m.def("peer_all_gather_ce", &peer_all_gather_ce, "all-gather with one copy-engine memcpy per rank",
        py::arg("bases"), py::arg("src_off"), py::arg("shard_bytes"), py::arg("out"), py::arg("src_stride") = 0,
        py::arg("skip_rank") = -1);
  m.def("peer_reduce_scatter", &peer_reduce_scatter, py::arg("bases"), py::arg("grad_off"), py::arg("rank"),
        py::arg("scale"), py::arg("out"), py::arg("part") = py::none(), py::arg("split") = 0, py::arg("rep_w") = 1.0);
  m.def("reduce_scatter_blocks", &reduce_scatter_blocks);
  m.def("peer_all_reduce_bf16", &peer_all_reduce_bf16);
  m.def("peer_reduce_rows_bf16", &peer_reduce_rows_bf16);
  m.def("wait_flag_probe", &wait_flag_probe, "bounded wait on a flag (tests the timeout path)");
  m.def("gemm_ce_blocks", &gemm_ce_blocks, "column blocks of the fused cross-entropy statistics");
  m.def("tmem_a_operand_check", &tmem_a_operand_check, "one tcgen05 MMA with its A operand in tensor memory");
  m.def("gemm_ag", &gemm_ag, "sequence-parallel all-gather fused in front of the tcgen05 GEMM");
  m.def("peer_signal", &peer_signal, "raise this rank's flag to `epoch` in every peer's heap");
  m.def("gemm_ce_stats", &gemm_ce_stats, "head GEMM -> per-block log-sum-exp statistics and target logits");
  m.def("gemm_ce_grad", &gemm_ce_grad, "head GEMM recomputed -> bf16 logit gradient");
  m.def("ce_stats_reduce", &ce_stats_reduce);
  m.def("ce_peer_combine", &ce_peer_combine, "vocabulary-parallel log-sum-exp over the TP group's heaps");
  m.def("ce_loss_finish", &ce_loss_finish);
}
