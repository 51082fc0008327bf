// Python bindings for every sm_100a kernel and the device communicator.
#include <torch/extension.h>

namespace mnb {
// gemm.cu
void gemm(torch::Tensor a, torch::Tensor b, torch::Tensor out, bool a_mn, bool b_mn,
          c10::optional<torch::Tensor> bias, c10::optional<torch::Tensor> aux, c10::optional<torch::Tensor> resid,
          int64_t epi, int64_t splits, c10::optional<torch::Tensor> workspace, torch::Tensor status);
// elementwise.cu
void layernorm_fwd(torch::Tensor x, torch::Tensor w, torch::Tensor b, torch::Tensor y, torch::Tensor mean,
                   torch::Tensor rstd, double eps);
void layernorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor mean, torch::Tensor rstd,
                   torch::Tensor dx, torch::Tensor dw, torch::Tensor db, torch::Tensor partials, bool accumulate);
void layernorm_bwd_add(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor mean, torch::Tensor rstd,
                       torch::Tensor add, torch::Tensor dx, torch::Tensor dw, torch::Tensor db, torch::Tensor partials,
                       bool accumulate);
int ln_bwd_blocks(int rows);
int colsum_row_blocks(int rows);
void bias_grad(torch::Tensor g, torch::Tensor out, torch::Tensor partials, bool accumulate);
void gelu_fwd(torch::Tensor x, torch::Tensor y);
void gelu_bwd(torch::Tensor x, torch::Tensor dy, torch::Tensor dx);
void embed_fwd(torch::Tensor idx, torch::Tensor wte, torch::Tensor wpe, torch::Tensor y);
void embed_bwd(torch::Tensor idx, torch::Tensor dy, torch::Tensor dwte, torch::Tensor dwpe, bool accumulate_pos);
void xent_fwd_bwd(torch::Tensor logits, torch::Tensor targets, torch::Tensor loss, double grad_scale,
                  int64_t ignore_index);
void adamw_step(torch::Tensor table, torch::Tensor chunks, bool param_bf16, bool grad_bf16, double lr, double beta1,
                double beta2, double eps, double wd, double bc1, double bc2, double grad_scale);
void stamp(torch::Tensor out, int64_t idx);
// attention.cu
void flash_attn_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o, torch::Tensor lse,
                    int64_t n_head, double scale);
void flash_attn_bwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o, torch::Tensor dout,
                    torch::Tensor lse, torch::Tensor dq, torch::Tensor dk, torch::Tensor dv, torch::Tensor dq_acc,
                    torch::Tensor delta, int64_t n_head, double scale);
// attention_tc.cu
void flash_attn_fwd_tc(torch::Tensor qkv, torch::Tensor o, torch::Tensor lse, int64_t n_head, double scale,
                       torch::Tensor status);
void flash_attn_bwd_tc(torch::Tensor qkv, torch::Tensor o, torch::Tensor dout, torch::Tensor lse, torch::Tensor dqkv,
                       torch::Tensor dq_acc, torch::Tensor delta, int64_t n_head, double scale, torch::Tensor status);
void exp2_poly_eval(torch::Tensor x, torch::Tensor y);
// comm.cu
void register_comm(pybind11::module_& m);
}  // namespace mnb

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "mini_nccl_b200 sm_100a kernels";
  m.def("gemm", &mnb::gemm, "tcgen05 GEMM with fused epilogues");
  m.def("layernorm_fwd", &mnb::layernorm_fwd);
  m.def("layernorm_bwd", &mnb::layernorm_bwd);
  m.def("layernorm_bwd_add", &mnb::layernorm_bwd_add);
  m.def("ln_bwd_blocks", &mnb::ln_bwd_blocks);
  m.def("colsum_row_blocks", &mnb::colsum_row_blocks);
  m.def("bias_grad", &mnb::bias_grad);
  m.def("gelu_fwd", &mnb::gelu_fwd);
  m.def("gelu_bwd", &mnb::gelu_bwd);
  m.def("embed_fwd", &mnb::embed_fwd);
  m.def("embed_bwd", &mnb::embed_bwd);
  m.def("xent_fwd_bwd", &mnb::xent_fwd_bwd);
  m.def("adamw_step", &mnb::adamw_step);
  m.def("stamp", &mnb::stamp, "write %globaltimer into out[idx] in stream order");
  m.def("flash_attn_fwd", &mnb::flash_attn_fwd);
  m.def("flash_attn_bwd", &mnb::flash_attn_bwd);
  m.def("flash_attn_fwd_tc", &mnb::flash_attn_fwd_tc, "tcgen05 flash attention forward");
  m.def("flash_attn_bwd_tc", &mnb::flash_attn_bwd_tc, "tcgen05 flash attention backward");
  m.def("exp2_poly_eval", &mnb::exp2_poly_eval, "the attention softmax's FMA-pipe exp2, over a tensor");
  mnb::register_comm(m);
}
