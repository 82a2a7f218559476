// Python bindings for the sm_100a kernels of libra_b200 (module libra_b200._C).
#include <torch/extension.h>

namespace libra {
void gemm_allreduce(torch::Tensor a, torch::Tensor b, bool b_mn, c10::optional<torch::Tensor> residual, torch::Tensor y,
                    std::vector<int64_t> recv, std::vector<int64_t> gath, std::vector<int64_t> flags, int64_t me,
                    int64_t parity, int64_t max_rows, int64_t rs_rows, torch::Tensor err);
void gemm_allgather(torch::Tensor a, torch::Tensor b, bool b_mn, torch::Tensor y, std::vector<int64_t> shards,
                    std::vector<int64_t> ready, torch::Tensor gath, torch::Tensor counter, int64_t me, int64_t call,
                    torch::Tensor err);
void gemm_bf16(torch::Tensor a, torch::Tensor b, torch::Tensor c, bool a_mn, bool b_mn, int64_t epi,
               c10::optional<torch::Tensor> residual, torch::Tensor err, bool streamk);
std::vector<torch::Tensor> rmsnorm_fwd(torch::Tensor x, torch::Tensor w, double eps);
torch::Tensor rmsnorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor rstd, torch::Tensor dw,
                          bool accumulate_dw, c10::optional<torch::Tensor> dx_accum);
std::vector<torch::Tensor> qk_norm_rope_fwd(torch::Tensor qkv, torch::Tensor qw, torch::Tensor kw, torch::Tensor pos,
                                            torch::Tensor cos_t, torch::Tensor sin_t, int64_t nq, int64_t nkv,
                                            double eps);
torch::Tensor qk_norm_rope_bwd(torch::Tensor qkv, torch::Tensor qw, torch::Tensor kw, torch::Tensor pos,
                               torch::Tensor cos_t, torch::Tensor sin_t, torch::Tensor rstd, torch::Tensor dq,
                               torch::Tensor dk, torch::Tensor dv, torch::Tensor dqw, torch::Tensor dkw, int64_t nq,
                               int64_t nkv);
torch::Tensor swiglu_fwd(torch::Tensor gu);
torch::Tensor swiglu_bwd(torch::Tensor gu, torch::Tensor dh);
std::vector<torch::Tensor> logprob_fwd(torch::Tensor logits, torch::Tensor targets, int64_t vocab_start,
                                       double temperature, bool with_entropy);
void logprob_bwd_(torch::Tensor logits, torch::Tensor targets, int64_t vocab_start, double temperature,
                  torch::Tensor lse, torch::Tensor grad);
void grad_sq_norm(torch::Tensor grad, torch::Tensor out);
void adamw_step(torch::Tensor master, torch::Tensor grad, torch::Tensor m, torch::Tensor v, torch::Tensor param,
                double lr, double beta1, double beta2, double eps, double wd, int64_t step,
                c10::optional<torch::Tensor> sq_norm, double max_norm, double grad_scale);
void adamw_step_allgather(torch::Tensor master, torch::Tensor grad, torch::Tensor m, torch::Tensor v, double lr,
                          double beta1, double beta2, double eps, double wd, int64_t step,
                          c10::optional<torch::Tensor> sq_norm, double max_norm, double grad_scale,
                          std::vector<int64_t> param_peers, std::vector<int64_t> flag_peers, int64_t me, int64_t epoch,
                          torch::Tensor err, int64_t grid_ctas);
std::vector<torch::Tensor> vocab_stats_exchange(std::vector<int64_t> data_ptrs, std::vector<int64_t> flag_ptrs,
                                                int64_t me, int64_t max_rows, torch::Tensor m, torch::Tensor s,
                                                torch::Tensor zt, int64_t epoch, torch::Tensor err);
void grad_reduce_scatter_peer(torch::Tensor out, double scale, c10::optional<torch::Tensor> sq_out,
                              std::vector<int64_t> src_peers, std::vector<int64_t> flag_peers, int64_t me,
                              int64_t epoch, torch::Tensor err, int64_t grid_ctas);
torch::Tensor paged_decode_attention(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                                     torch::Tensor block_tables, torch::Tensor seq_lens, int64_t max_len,
                                     double scale);
void gemm_swiglu(torch::Tensor x, torch::Tensor w, torch::Tensor a, c10::optional<torch::Tensor> gu,
                 torch::Tensor err);
void grouped_gemm(torch::Tensor a, torch::Tensor b, torch::Tensor c, torch::Tensor offs, int64_t mode, bool b_mn,
                  int64_t epi, c10::optional<torch::Tensor> c2, torch::Tensor err);
void grouped_gemm_wgrad(torch::Tensor dy, torch::Tensor x, torch::Tensor c, torch::Tensor offs, bool accumulate,
                        torch::Tensor err);
namespace rollout {
void paged_decode_v2(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor block_tables,
                     torch::Tensor seq_lens, torch::Tensor out, torch::Tensor part_out, torch::Tensor part_ml,
                     int64_t split_len, double scale);
void sample_tokens(torch::Tensor logits, torch::Tensor temperature, torch::Tensor seeds, torch::Tensor positions,
                   torch::Tensor out_tok, torch::Tensor out_lp, c10::optional<torch::Tensor> next_tok, bool pdl);
void sample_tokens_filtered(torch::Tensor logits, torch::Tensor temperature, torch::Tensor top_p, torch::Tensor top_k,
                            torch::Tensor seeds, torch::Tensor positions, torch::Tensor out_tok, torch::Tensor out_lp);
}  // namespace rollout
namespace reshard {
void weight_reshard(torch::Tensor items, int64_t grid);
}  // namespace reshard
namespace attn {
std::vector<torch::Tensor> flash_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor cu_seqlens,
                                     torch::Tensor tiles, double scale, bool causal, torch::Tensor err,
                                     c10::optional<torch::Tensor> cu_k);
std::vector<torch::Tensor> flash_bwd(torch::Tensor dout, torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                     torch::Tensor out, torch::Tensor lse, torch::Tensor cu_seqlens,
                                     torch::Tensor q_tiles, torch::Tensor kv_tiles, double scale, bool causal,
                                     torch::Tensor err);
}  // namespace attn
namespace ipc {
std::tuple<py::bytes, int64_t> ipc_export(torch::Tensor t);
int64_t ipc_open(py::bytes handle);
void ipc_close(int64_t ptr);
}  // namespace ipc
namespace tp {
std::vector<torch::Tensor> allreduce_add_rmsnorm(std::vector<int64_t> data_ptrs, std::vector<int64_t> flag_ptrs,
                                                 int64_t me, int64_t slot_offset_bytes, torch::Tensor residual,
                                                 torch::Tensor w, double eps, int64_t epoch, int64_t grid,
                                                 torch::Tensor err);
}  // namespace tp
namespace ep {
void ep_push(std::vector<int64_t> rx, std::vector<int64_t> flags, int64_t me, int64_t slot_off, torch::Tensor x,
             c10::optional<torch::Tensor> scale, torch::Tensor dst_rank, torch::Tensor dst_row, int64_t k,
             int64_t max_rows, int64_t epoch, int64_t grid, torch::Tensor err);
void ep_pull(std::vector<int64_t> tx, std::vector<int64_t> flags, int64_t me, int64_t slot_off,
             c10::optional<torch::Tensor> weight, c10::optional<torch::Tensor> residual, torch::Tensor src_rank,
             torch::Tensor src_row, int64_t k, int64_t max_rows, torch::Tensor out, c10::optional<torch::Tensor> gath,
             int64_t epoch, int64_t grid, torch::Tensor err);
}  // namespace ep
void decode_attention(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor block_tables,
                      torch::Tensor seq_lens, torch::Tensor out, torch::Tensor part_o, torch::Tensor part_ml,
                      torch::Tensor counters, torch::Tensor err, double scale, bool pdl);
void decode_qkv_post(torch::Tensor acc, torch::Tensor qw, torch::Tensor kw, torch::Tensor pos, torch::Tensor cos_t,
                     torch::Tensor sin_t, torch::Tensor slot, torch::Tensor q_out, torch::Tensor k_cache,
                     torch::Tensor v_cache, double eps, bool pdl);
void decode_residual_norm(torch::Tensor x, torch::Tensor acc, torch::Tensor w, torch::Tensor h_out, double eps,
                          bool pdl);
void decode_swiglu(torch::Tensor acc, torch::Tensor a, bool pdl);
void gemm_decode(torch::Tensor x, torch::Tensor w, torch::Tensor acc, torch::Tensor err, bool pdl);
}  // namespace libra

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("decode_attention", &libra::decode_attention,
        "paged decode attention, stream-K over KV blocks with an in-kernel merge (no allocation)", py::arg("q"),
        py::arg("k_cache"), py::arg("v_cache"), py::arg("block_tables"), py::arg("seq_lens"), py::arg("out"),
        py::arg("part_o"), py::arg("part_ml"), py::arg("counters"), py::arg("err"), py::arg("scale"),
        py::arg("pdl") = false);
  m.def("decode_qkv_post", &libra::decode_qkv_post,
        "fused decode: qkv accumulator -> q/k RMSNorm + RoPE -> q and the paged KV cache (zeroes the accumulator)",
        py::arg("acc"), py::arg("qw"), py::arg("kw"), py::arg("pos"), py::arg("cos"), py::arg("sin"), py::arg("slot"),
        py::arg("q_out"), py::arg("k_cache"), py::arg("v_cache"), py::arg("eps"), py::arg("pdl") = false);
  m.def("decode_residual_norm", &libra::decode_residual_norm,
        "fused decode: x += acc (bf16), h = RMSNorm(x) * w (zeroes the accumulator)", py::arg("x"), py::arg("acc"),
        py::arg("w"), py::arg("h_out"), py::arg("eps"), py::arg("pdl") = false);
  m.def("decode_swiglu", &libra::decode_swiglu, "fused decode: SwiGLU of the gate/up accumulator (zeroes it)",
        py::arg("acc"), py::arg("a"), py::arg("pdl") = false);
  m.def("gemm_decode", &libra::gemm_decode,
        "decode-step skinny GEMM acc += x w^T on tcgen05 (weights as the 128-row MMA operand, stream-K over all SMs)",
        py::arg("x"), py::arg("w"), py::arg("acc"), py::arg("err"), py::arg("pdl") = false);
  m.doc() = "libra_b200 sm_100a kernels";
  m.def("gemm_bf16", &libra::gemm_bf16, "tcgen05 bf16 GEMM", py::arg("a"), py::arg("b"), py::arg("c"),
        py::arg("a_mn"), py::arg("b_mn"), py::arg("epi"), py::arg("residual"), py::arg("err"),
        py::arg("streamk") = false);
  m.def("gemm_swiglu", &libra::gemm_swiglu, "tcgen05 gate/up GEMM with fused SwiGLU epilogue", py::arg("x"),
        py::arg("w"), py::arg("a"), py::arg("gu"), py::arg("err"));
  m.def("grouped_gemm", &libra::grouped_gemm,
        "per-expert tcgen05 GEMM over padded row groups whose offsets live in device memory");
  m.def("grouped_gemm_wgrad", &libra::grouped_gemm_wgrad,
        "per-expert weight gradient dW_g (+)= dy[rows of g]^T x[rows of g] over padded row groups");
  m.def("rmsnorm_fwd", &libra::rmsnorm_fwd);
  m.def("rmsnorm_bwd", &libra::rmsnorm_bwd);
  m.def("qk_norm_rope_fwd", &libra::qk_norm_rope_fwd);
  m.def("qk_norm_rope_bwd", &libra::qk_norm_rope_bwd);
  m.def("swiglu_fwd", &libra::swiglu_fwd);
  m.def("swiglu_bwd", &libra::swiglu_bwd);
  m.def("logprob_fwd", &libra::logprob_fwd);
  m.def("logprob_bwd_", &libra::logprob_bwd_);
  m.def("grad_sq_norm", &libra::grad_sq_norm);
  m.def("adamw_step", &libra::adamw_step);
  m.def("adamw_step_allgather", &libra::adamw_step_allgather,
        "AdamW on this rank's shard with the bf16 result stored into every rank's parameter buffer");
  m.def("vocab_stats_exchange", &libra::vocab_stats_exchange,
        "vocab-parallel log-softmax: per-row (max, sum-exp, target logit) exchange over peer memory -> (lse, target)");
  m.def("grad_reduce_scatter_peer", &libra::grad_reduce_scatter_peer,
        "distributed-optimizer gradient reduce-scatter over peer memory, fused with 1/dp scaling and the global "
        "sum of squares");
  m.def("paged_decode_attention", &libra::paged_decode_attention);
  m.def("weight_reshard", &libra::reshard::weight_reshard,
        "trainer -> rollout weight sync: planned 2-D copies (peer sources over NVLink, fp32/bf16 -> bf16)");
  m.def("paged_decode_v2", &libra::rollout::paged_decode_v2,
        "paged decode attention with caller-owned split workspace (graph-capturable)");
  m.def("sample_tokens", &libra::rollout::sample_tokens,
        "Gumbel-max temperature sampling with the sampled token's logprob", py::arg("logits"), py::arg("temperature"),
        py::arg("seeds"), py::arg("positions"), py::arg("out_tok"), py::arg("out_lp"), py::arg("next_tok") = py::none(),
        py::arg("pdl") = false);
  m.def("sample_tokens_filtered", &libra::rollout::sample_tokens_filtered,
        "top-k / top-p (nucleus) temperature sampling by radix-selected thresholds + Gumbel-max, with logprobs");
  m.def("flash_fwd", &libra::attn::flash_fwd, "tcgen05 varlen GQA attention forward", py::arg("q"), py::arg("k"),
        py::arg("v"), py::arg("cu_seqlens"), py::arg("tiles"), py::arg("scale"), py::arg("causal"), py::arg("err"),
        py::arg("cu_k") = py::none());
  m.def("gemm_allreduce", &libra::gemm_allreduce,
        "tensor-parallel GEMM fused with a peer-memory all-reduce or reduce-scatter (+ residual)");
  m.def("gemm_allgather", &libra::gemm_allgather,
        "sequence-parallel all-gather of the A rows fused into the tensor-parallel GEMM");
  m.def("flash_bwd", &libra::attn::flash_bwd, "tcgen05 varlen GQA attention backward (dq, dk, dv)");
  m.def("ipc_export", &libra::ipc::ipc_export, "CUDA IPC handle of the allocation holding a tensor + offset");
  m.def("ipc_open", &libra::ipc::ipc_open, "map a peer allocation into the current device's context");
  m.def("ipc_close", &libra::ipc::ipc_close);
  m.def("tp_allreduce_add_rmsnorm", &libra::tp::allreduce_add_rmsnorm,
        "peer-memory all-reduce of TP partials + residual + RMSNorm");
  m.def("ep_push", &libra::ep::ep_push, "MoE dispatch: rows stored straight into the expert owners' peer buffers");
  m.def("ep_pull", &libra::ep::ep_pull,
        "MoE combine: weighted sum of the expert outputs loaded from the owners' peer buffers (+ residual)");
}
