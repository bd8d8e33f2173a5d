// Python bindings of the sm_100a kernel library (module graspo_b200._C).
#include <torch/extension.h>

namespace gb {
bool& pdl_enabled();
void gemm_tc(torch::Tensor A, torch::Tensor B, c10::optional<torch::Tensor> A2,
             c10::optional<torch::Tensor> B2, torch::Tensor C, c10::optional<torch::Tensor> R,
             c10::optional<torch::Tensor> aux, c10::optional<torch::Tensor> targets,
             c10::optional<torch::Tensor> tgt_logit, c10::optional<torch::Tensor> row_lse,
             c10::optional<torch::Tensor> row_scale, int64_t epilogue, bool swap, int64_t bn,
             int64_t splits, torch::Tensor err, int64_t max_ctas, c10::optional<torch::Tensor> push_dst,
             c10::optional<torch::Tensor> push_flag, c10::optional<torch::Tensor> tile_ctr, int64_t layout,
             c10::optional<torch::Tensor> push_out, c10::optional<torch::Tensor> push_sig, int64_t push_self,
             int64_t push_rows, int64_t push_fence_once);
void tp_reduce(torch::Tensor srcs, int64_t counter, int64_t expected, c10::optional<torch::Tensor> residual,
               torch::Tensor out, int64_t ld_src, torch::Tensor err, int64_t spin_limit);
void paged_decode_attention_tc(torch::Tensor q, torch::Tensor k_pool, torch::Tensor v_pool,
                               torch::Tensor block_table, torch::Tensor start, torch::Tensor len,
                               torch::Tensor out, double scale, int64_t splits, torch::Tensor scratch,
                               int64_t prefix_len, int64_t group_rows, int64_t prefix_splits,
                               torch::Tensor err);
void peer_copy(int64_t dst, torch::Tensor src, int64_t src_offset_bytes, int64_t nbytes);
void signal_counters(torch::Tensor counters, int64_t count);
void dp_reduce(torch::Tensor grads, torch::Tensor srcs, int64_t counter, int64_t expected, double scale,
               torch::Tensor err, int64_t spin_limit);
void conv_silu_fwd(torch::Tensor x, c10::optional<torch::Tensor> prev, torch::Tensor w, torch::Tensor y);
void conv_silu_bwd(torch::Tensor x, c10::optional<torch::Tensor> prev, torch::Tensor w, torch::Tensor dy,
                   torch::Tensor dx);
void gated_rmsnorm_fwd(torch::Tensor x, torch::Tensor z, torch::Tensor w, torch::Tensor y, double eps);
void gated_rmsnorm_bwd(torch::Tensor x, torch::Tensor z, torch::Tensor w, torch::Tensor dy, torch::Tensor dx,
                       torch::Tensor dz, double eps);
void sigmoid_gate_fwd(torch::Tensor o, torch::Tensor g, torch::Tensor y);
void sigmoid_gate_bwd(torch::Tensor o, torch::Tensor g, torch::Tensor dy, torch::Tensor dout, torch::Tensor dg);
void lse_push(torch::Tensor partials, torch::Tensor tgt, torch::Tensor dst, torch::Tensor sig, int64_t self);
void lse_merge(torch::Tensor srcs, int64_t counter, int64_t expected, torch::Tensor lse, torch::Tensor logp,
               torch::Tensor err, int64_t spin_limit);
std::vector<torch::Tensor> symm_alloc(int64_t nbytes, int64_t device);
int64_t symm_open(torch::Tensor handle, int64_t device);
void symm_close(int64_t ptr, int64_t device);
bool enable_peer_access(int64_t device, int64_t peer);
void add_rmsnorm(torch::Tensor h, c10::optional<torch::Tensor> delta, c10::optional<torch::Tensor> h_out,
                 torch::Tensor w, torch::Tensor y, c10::optional<torch::Tensor> rstd,
                 c10::optional<torch::Tensor> lora_a, c10::optional<torch::Tensor> lora_u, double scale,
                 double eps, c10::optional<torch::Tensor> delta_lora_b, int64_t delta_lora_r,
                 c10::optional<torch::Tensor> peer_src, c10::optional<torch::Tensor> peer_sync,
                 int64_t peer_expected, c10::optional<torch::Tensor> err,
                 c10::optional<torch::Tensor> zero_tail);
void rmsnorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> rstd,
                 c10::optional<torch::Tensor> dres, torch::Tensor dx, double eps);
void qk_norm_rope(torch::Tensor qkv, torch::Tensor q_w, torch::Tensor k_w, torch::Tensor inv_freq,
                  torch::Tensor pos, torch::Tensor q_out, torch::Tensor k_out, torch::Tensor v_out,
                  c10::optional<torch::Tensor> block_table, c10::optional<torch::Tensor> row_of_token,
                  c10::optional<torch::Tensor> slot, int64_t nq, int64_t nkv, int64_t page_size, double eps,
                  c10::optional<torch::Tensor> lora_b, int64_t lora_r, c10::optional<torch::Tensor> err);
void qk_norm_rope_bwd(torch::Tensor dq, torch::Tensor dk, torch::Tensor dv, torch::Tensor qkv,
                      torch::Tensor q_w, torch::Tensor k_w, torch::Tensor inv_freq, torch::Tensor pos,
                      torch::Tensor dqkv, int64_t nq, int64_t nkv, double eps);
void swiglu_bwd(torch::Tensor gu, torch::Tensor dh, torch::Tensor dgu);
void lora_down(torch::Tensor x, torch::Tensor A, torch::Tensor U, double scale);
void gated_delta_step(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor g, torch::Tensor beta,
                      torch::Tensor state, torch::Tensor out);
void embedding(torch::Tensor ids, torch::Tensor table, torch::Tensor out);
bool kernel_checks();
void flash_attn_fwd_tc(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor out, torch::Tensor lse,
                       torch::Tensor start, torch::Tensor end, int64_t B, int64_t S, double scale, torch::Tensor err);
void flash_attn_bwd_tc(torch::Tensor dout, torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor out,
                       torch::Tensor lse, torch::Tensor dq, torch::Tensor dk, torch::Tensor dv, torch::Tensor start,
                       torch::Tensor end, int64_t B, int64_t S, double scale, torch::Tensor err);
void paged_decode_attention(torch::Tensor q, torch::Tensor k_pool, torch::Tensor v_pool,
                            torch::Tensor block_table, torch::Tensor start, torch::Tensor len,
                            torch::Tensor out, double scale, int64_t splits,
                            c10::optional<torch::Tensor> scratch, int64_t prefix_len, int64_t group_rows,
                            int64_t prefix_splits, c10::optional<torch::Tensor> err);
void sample_append_split(torch::Tensor logits, double temperature, int64_t seed, torch::Tensor next_ids,
                         torch::Tensor slot, torch::Tensor pos, torch::Tensor kv_len, torch::Tensor finished,
                         torch::Tensor out_tokens, int64_t prompt_slots, int64_t eos_id, int64_t pad_id,
                         bool ignore_eos, int64_t vocab_start, torch::Tensor scratch, int64_t chunk,
                         torch::Tensor err, c10::optional<torch::Tensor> exch_dst,
                         c10::optional<torch::Tensor> exch_sig, int64_t exch_self, int64_t exch_slots,
                         int64_t exch_arrivals, int64_t spin_limit);
void sample_append(torch::Tensor logits, double temperature, double top_p, int64_t seed,
                   torch::Tensor next_ids, torch::Tensor slot, torch::Tensor pos, torch::Tensor kv_len,
                   torch::Tensor finished, torch::Tensor out_tokens, int64_t prompt_slots,
                   int64_t eos_id, int64_t pad_id, bool ignore_eos, c10::optional<torch::Tensor> active);
void lse_combine(torch::Tensor partials, torch::Tensor tgt, torch::Tensor lse, torch::Tensor logp);
void grpo_loss(torch::Tensor logp, torch::Tensor old_logp, torch::Tensor adv, torch::Tensor mask,
               double clip_eps, double grad_scale, torch::Tensor loss, torch::Tensor dlogp,
               c10::optional<torch::Tensor> stats);
void dropout(torch::Tensor x, torch::Tensor y, double p, int64_t seed, int64_t stream_id,
             c10::optional<torch::Tensor> add);
void grad_sumsq(torch::Tensor g, torch::Tensor out);
void adamw(torch::Tensor p, torch::Tensor g, torch::Tensor m, torch::Tensor v, double lr, double b1,
           double b2, double eps, double wd, int64_t step, torch::Tensor sumsq, double max_norm,
           c10::optional<torch::Tensor> loss, c10::optional<torch::Tensor> skipped);
void transpose_bf16(torch::Tensor in, torch::Tensor out);
}  // namespace gb

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "graspo_b200 sm_100a kernels";
  m.def("gemm_tc", &gb::gemm_tc, "tcgen05 GEMM with fused epilogues", py::arg("A"), py::arg("B"), py::arg("A2"),
        py::arg("B2"), py::arg("C"), py::arg("R"), py::arg("aux"), py::arg("targets"), py::arg("tgt_logit"),
        py::arg("row_lse"), py::arg("row_scale"), py::arg("epilogue"), py::arg("swap"), py::arg("bn"),
        py::arg("splits"), py::arg("err"), py::arg("max_ctas"), py::arg("push_dst") = py::none(),
        py::arg("push_flag") = py::none(), py::arg("tile_ctr") = py::none(), py::arg("layout") = 0,
        py::arg("push_out") = py::none(), py::arg("push_sig") = py::none(), py::arg("push_self") = 0,
        py::arg("push_rows") = 0, py::arg("push_fence_once") = 0);
  m.def("tp_reduce", &gb::tp_reduce,
        "sum of the tensor-parallel receive slots (rank order) + optional residual, after a bounded wait "
        "on the arrival counter",
        py::arg("srcs"), py::arg("counter"), py::arg("expected"), py::arg("residual"), py::arg("out"),
        py::arg("ld_src"), py::arg("err"), py::arg("spin_limit") = 0);
  m.def("paged_decode_attention_tc", &gb::paged_decode_attention_tc,
        "paged decode attention on tcgen05 / TMA: prompt keys once per group, per-row keys split, merged "
        "by the last arriving CTA");
  m.def("peer_copy", &gb::peer_copy, "copy-engine copy of a local byte range to a (peer) device address");
  m.def("signal_counters", &gb::signal_counters, "add a count to peers' 64-bit arrival counters (release)");
  m.def("dp_reduce", &gb::dp_reduce,
        "data-parallel gradient sum in rank order times a scale, after a bounded wait on the arrival counter",
        py::arg("grads"), py::arg("srcs"), py::arg("counter"), py::arg("expected"), py::arg("scale"), py::arg("err"),
        py::arg("spin_limit") = 0);
  m.def("conv_silu_fwd", &gb::conv_silu_fwd, "causal depthwise conv1d + SiLU, channels-last");
  m.def("conv_silu_bwd", &gb::conv_silu_bwd, "input gradient of the causal conv1d + SiLU (frozen weight)");
  m.def("gated_rmsnorm_fwd", &gb::gated_rmsnorm_fwd, "w * rmsnorm(x) * silu(z)");
  m.def("gated_rmsnorm_bwd", &gb::gated_rmsnorm_bwd, "gradients of the gated RMSNorm for x and z");
  m.def("sigmoid_gate_fwd", &gb::sigmoid_gate_fwd, "o * sigmoid(g)");
  m.def("sigmoid_gate_bwd", &gb::sigmoid_gate_bwd, "gradients of o * sigmoid(g)");
  m.def("lse_push", &gb::lse_push,
        "vocab-parallel log-prob: this shard's (log-sum-exp, target logit) per token into every rank's slot");
  m.def("lse_merge", &gb::lse_merge,
        "vocab-parallel log-prob: bounded wait, then merge every shard's pair into lse and log-prob",
        py::arg("srcs"), py::arg("counter"), py::arg("expected"), py::arg("lse"), py::arg("logp"), py::arg("err"),
        py::arg("spin_limit") = 0);
  m.def("symm_alloc", &gb::symm_alloc, "zeroed device buffer + its CUDA IPC handle");
  m.def("symm_open", &gb::symm_open, "map a peer's buffer from its IPC handle; returns the device address");
  m.def("symm_close", &gb::symm_close);
  m.def("enable_peer_access", &gb::enable_peer_access, "direct access from one GPU to another's memory");
  m.def("set_pdl", [](bool on) { gb::pdl_enabled() = on; },
        "launch the decode-chain kernels with programmatic dependent launch (default on)");
  m.def("pdl_enabled", []() { return gb::pdl_enabled(); });
  m.def("add_rmsnorm", &gb::add_rmsnorm, py::arg("h"), py::arg("delta"), py::arg("h_out"), py::arg("w"),
        py::arg("y"), py::arg("rstd"), py::arg("lora_a"), py::arg("lora_u"), py::arg("scale"), py::arg("eps"),
        py::arg("delta_lora_b") = py::none(), py::arg("delta_lora_r") = 0, py::arg("peer_src") = py::none(),
        py::arg("peer_sync") = py::none(), py::arg("peer_expected") = 0, py::arg("err") = py::none(),
        py::arg("zero_tail") = py::none());
  m.def("rmsnorm_bwd", &gb::rmsnorm_bwd);
  m.def("qk_norm_rope", &gb::qk_norm_rope, py::arg("qkv"), py::arg("q_w"), py::arg("k_w"), py::arg("inv_freq"),
        py::arg("pos"), py::arg("q_out"), py::arg("k_out"), py::arg("v_out"), py::arg("block_table"),
        py::arg("row_of_token"), py::arg("slot"), py::arg("nq"), py::arg("nkv"), py::arg("page_size"),
        py::arg("eps"), py::arg("lora_b") = py::none(), py::arg("lora_r") = 0, py::arg("err") = py::none());
  m.def("qk_norm_rope_bwd", &gb::qk_norm_rope_bwd);
  m.def("swiglu_bwd", &gb::swiglu_bwd);
  m.def("lora_down", &gb::lora_down);
  m.def("gated_delta_step", &gb::gated_delta_step, "one decoding step of the gated delta rule");
  m.def("embedding", &gb::embedding);
  m.def("kernel_checks", &gb::kernel_checks, "true when built with GRASPO_KERNEL_CHECKS (index checks)");
  m.def("paged_decode_attention", &gb::paged_decode_attention, py::arg("q"), py::arg("k_pool"), py::arg("v_pool"),
        py::arg("block_table"), py::arg("start"), py::arg("len"), py::arg("out"), py::arg("scale"),
        py::arg("splits"), py::arg("scratch"), py::arg("prefix_len") = 0, py::arg("group_rows") = 1,
        py::arg("prefix_splits") = 1, py::arg("err") = py::none());
  m.def("flash_attn_fwd_tc", &gb::flash_attn_fwd_tc, "causal flash attention forward on tcgen05 / TMEM");
  m.def("flash_attn_bwd_tc", &gb::flash_attn_bwd_tc, "causal flash attention backward on tcgen05 / TMEM");
  m.def("sample_append", &gb::sample_append);
  m.def("sample_append_split", &gb::sample_append_split,
        "Gumbel-max sampling over vocabulary chunks on every SM (top-p 1), optionally vocab-parallel with the "
        "shards' winners exchanged through peer memory",
        py::arg("logits"), py::arg("temperature"), py::arg("seed"), py::arg("next_ids"), py::arg("slot"),
        py::arg("pos"), py::arg("kv_len"), py::arg("finished"), py::arg("out_tokens"), py::arg("prompt_slots"),
        py::arg("eos_id"), py::arg("pad_id"), py::arg("ignore_eos"), py::arg("vocab_start"), py::arg("scratch"),
        py::arg("chunk"), py::arg("err"), py::arg("exch_dst") = py::none(), py::arg("exch_sig") = py::none(),
        py::arg("exch_self") = 0, py::arg("exch_slots") = 0, py::arg("exch_arrivals") = 0,
        py::arg("spin_limit") = 0);
  m.def("lse_combine", &gb::lse_combine);
  m.def("grpo_loss", &gb::grpo_loss);
  m.def("dropout", &gb::dropout);
  m.def("grad_sumsq", &gb::grad_sumsq);
  m.def("adamw", &gb::adamw);
  m.def("transpose_bf16", &gb::transpose_bf16);
}
