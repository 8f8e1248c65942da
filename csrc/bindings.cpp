// Python bindings of the rl_b200 native extension (module rl_b200._C).
#include <torch/extension.h>

#include <atomic>
#include <map>
#include <string>
#include <vector>

// norm.cu
std::vector<at::Tensor> rmsnorm_fwd(at::Tensor x, at::Tensor w, double eps);
std::vector<at::Tensor> add_rmsnorm_fwd(at::Tensor x, at::Tensor delta, at::Tensor w, double eps);
std::vector<at::Tensor> rmsnorm_bwd(at::Tensor dy, at::Tensor x, at::Tensor w, at::Tensor rstd);
std::vector<at::Tensor> rmsnorm_bwd_add(at::Tensor dy, at::Tensor x, at::Tensor w, at::Tensor rstd,
                                        c10::optional<at::Tensor> ds);
// elementwise.cu
at::Tensor rope_qkv(at::Tensor qkv, at::Tensor positions, at::Tensor cache, int64_t nq, int64_t nkv, int64_t hd,
                    bool inverse);
at::Tensor swiglu_fwd(at::Tensor gu);
at::Tensor swiglu_bwd(at::Tensor dout, at::Tensor gu);
void write_kv_cache(at::Tensor k, at::Tensor v, at::Tensor k_cache, at::Tensor v_cache, at::Tensor slots,
                    double k_scale, double v_scale);
// logprob.cu
std::vector<at::Tensor> logprob_partials(at::Tensor logits, at::Tensor targets, double temperature);
void logprob_bwd(at::Tensor dlp, at::Tensor logits, at::Tensor targets, at::Tensor lse, double temperature,
                 at::Tensor out);
// sampling.cu
void sample(at::Tensor logits, double temperature, int64_t top_k, double top_p, int64_t seed, at::Tensor offset,
            at::Tensor out_tok, at::Tensor out_lp);
// optim.cu
void adamw_step(at::Tensor master, at::Tensor grad, at::Tensor exp_avg, at::Tensor exp_avg_sq,
                c10::optional<at::Tensor> param_out, double lr, double beta1, double beta2, double eps,
                double weight_decay, int64_t step, double grad_scale);
at::Tensor sum_sq(at::Tensor x);
// quant.cu
std::vector<at::Tensor> quant_fp8_block(at::Tensor w, int64_t blk, bool pow2, c10::optional<at::Tensor> out,
                                        c10::optional<at::Tensor> out_scale);
std::vector<at::Tensor> quant_fp8_group(at::Tensor x, int64_t group, bool pow2);
std::vector<at::Tensor> quant_fp8_group_t(at::Tensor x, int64_t group, bool pow2);
// attention.cu
std::vector<at::Tensor> flash_attn_fwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor cu_seqlens,
                                       int64_t max_seqlen, double scale, bool causal);
std::vector<at::Tensor> flash_attn_bwd(at::Tensor dout, at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor out,
                                       at::Tensor lse, at::Tensor cu_seqlens, int64_t max_seqlen, double scale,
                                       bool causal);
at::Tensor paged_decode_attn(at::Tensor q, at::Tensor k_cache, at::Tensor v_cache, at::Tensor block_tables,
                             at::Tensor seq_lens, double scale, int64_t max_seq_len, double k_scale, double v_scale);
// gemm_tcgen05.cu
at::Tensor gemm_nt(at::Tensor a, at::Tensor b);
int64_t gemm_error_flag(bool reset);
void gemm_rs(at::Tensor a, at::Tensor b, at::Tensor out, std::vector<int64_t> recv_ptrs,
             std::vector<int64_t> flag_ptrs, std::vector<int64_t> ack_ptrs, int64_t me, int64_t epoch);
// attention_sm100.cu
std::vector<at::Tensor> flash_attn_fwd_tc(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor cu_seqlens,
                                          int64_t max_seqlen, double scale, bool causal);
std::vector<at::Tensor> flash_attn_seg_fwd_tc(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor seg, int64_t max_q,
                                              double scale, c10::optional<at::Tensor> cp_flags, int64_t cp_epoch,
                                              int64_t cp_size);
std::vector<at::Tensor> flash_attn_bwd_tc(at::Tensor dout, at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor out,
                                          at::Tensor lse, at::Tensor cu_seqlens, int64_t max_seqlen, double scale,
                                          bool causal);
std::vector<at::Tensor> flash_attn_seg_bwd_tc(at::Tensor dout, at::Tensor q, at::Tensor k, at::Tensor v,
                                              at::Tensor out, at::Tensor lse, at::Tensor seg, int64_t max_k,
                                              double scale);
int64_t attn_tc_error_flag(bool reset);
// gemm_sm100.cu
void gemm_sm100(at::Tensor a, at::Tensor b, at::Tensor out, bool a_mn, bool b_mn, bool accumulate, int64_t tile);
int64_t gemm_sm100_error_flag(bool reset);
std::vector<at::Tensor> gemm_logprob_partials(at::Tensor h, at::Tensor w, at::Tensor targets, double temperature);
at::Tensor gemm_dlogits(at::Tensor h, at::Tensor w, at::Tensor targets, at::Tensor lse, at::Tensor dlp,
                        double temperature);
// gemm_grouped.cu
at::Tensor grouped_gemm_nt(at::Tensor x, at::Tensor w, at::Tensor offs);
int64_t grouped_gemm_error_flag(bool reset);
// gemm_fp8.cu
at::Tensor gemm_fp8(at::Tensor a, at::Tensor a_scale, at::Tensor b, at::Tensor b_scale, int64_t splits);
at::Tensor gemm_mxf8(at::Tensor a, at::Tensor a_scale, at::Tensor b, at::Tensor b_scale, int64_t splits);
int64_t gemm_fp8_error_flag(bool reset);
// symm.cu
std::tuple<int64_t, at::Tensor> symm_alloc(int64_t bytes);
int64_t symm_open(at::Tensor handle);
void symm_close(int64_t ptr);
at::Tensor symm_view(int64_t ptr, int64_t numel, int64_t dtype_code, int64_t device);
void refit_copy(at::Tensor tasks, at::Tensor dst);
at::Tensor gemm_decode(at::Tensor x, at::Tensor w);
at::Tensor gemm_decode_split(at::Tensor x, at::Tensor w, int64_t splits);
at::Tensor gemm_ag(at::Tensor a, at::Tensor b, at::Tensor shard_flags, int64_t n, int64_t me, int64_t epoch);
void stream_write_u32(int64_t ptr, int64_t value);
at::Tensor ar_add_rmsnorm(at::Tensor partial, at::Tensor resid, at::Tensor w, double eps, std::vector<int64_t> slots,
                          std::vector<int64_t> flags, int64_t me, int64_t cap, at::Tensor ctr, at::Tensor done);
int64_t decode_ar_error_flag(bool reset);
std::vector<at::Tensor> spec_verify(at::Tensor target_logits, at::Tensor draft_logits, at::Tensor draft_tokens,
                                    double temperature, int64_t seed, int64_t offset);
std::vector<at::Tensor> flash_attn_seg_fwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor seg, int64_t max_q,
                                           double scale, c10::optional<at::Tensor> cp_flags, int64_t cp_epoch,
                                           int64_t cp_size);
int64_t attn_error_flag(bool reset);
std::vector<at::Tensor> flash_attn_seg_bwd(at::Tensor dout, at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor out,
                                           at::Tensor lse, at::Tensor seg, int64_t max_k, double scale);
int64_t bounds_error_elementwise(bool reset);
int64_t bounds_error_attention(bool reset);
int64_t bounds_error_ep_comm(bool reset);
int64_t bounds_error_moe_router(bool reset);

// Error words of the bounds-checked debug build, per instrumented source file
// (0 everywhere in the release build).
std::map<std::string, int64_t> bounds_errors(bool reset) {
  return {{"elementwise", bounds_error_elementwise(reset)},
          {"attention", bounds_error_attention(reset)},
          {"ep_comm", bounds_error_ep_comm(reset)},
          {"moe_router", bounds_error_moe_router(reset)}};
}

bool debug_bounds_build() {
#ifdef RLB_DEBUG_BOUNDS
  return true;
#else
  return false;
#endif
}

// nvls.cu
void nvls_barrier(std::vector<int64_t> pad_ptrs, int64_t rank, int64_t epoch);
void nvls_all_reduce(int64_t mc_ptr, int64_t nbytes, bool f32, int64_t rank, int64_t world);
void nvls_reduce_shard(int64_t mc_ptr, int64_t lo, int64_t len, at::Tensor out, bool f32);
int64_t nvls_error_flag(bool reset);
std::vector<at::Tensor> moe_router_topk(at::Tensor logits, int64_t k);
void ep_scatter(at::Tensor src, c10::optional<at::Tensor> src_row, at::Tensor dst_rank, at::Tensor dst_row,
                c10::optional<at::Tensor> tags, int64_t cap, std::vector<int64_t> buf, std::vector<int64_t> tag,
                std::vector<int64_t> flags, std::vector<int64_t> acks, int64_t me, int64_t epoch, at::Tensor counter);
void ep_consume(at::Tensor out, c10::optional<at::Tensor> out_tag, int64_t cap, std::vector<int64_t> buf,
                std::vector<int64_t> tag, std::vector<int64_t> flags, std::vector<int64_t> acks, int64_t me,
                int64_t epoch, at::Tensor counter);
int64_t ep_error_flag(bool reset);
at::Tensor dp_reduce_shard(std::vector<int64_t> grad_ptrs, int64_t lo, int64_t len, at::Tensor out);
void dp_wait_ready(std::vector<int64_t> flag_ptrs, int64_t idx, int64_t epoch);
int64_t dp_error_flag(bool reset);
void dp_adam_allgather(std::vector<int64_t> param_ptrs, int64_t lo, at::Tensor master, at::Tensor grad,
                       at::Tensor exp_avg, at::Tensor exp_avg_sq, at::Tensor nodecay, double lr, double b1, double b2,
                       double eps, double wd, int64_t step, double gscale);
int64_t gemm_decode_error_flag(bool reset);
void refit_quant_fp8(at::Tensor tasks, at::Tensor q, at::Tensor scales, bool pow2);

namespace rlb {
namespace {
std::atomic<int64_t> g_peer_wait_cycles{4000000000LL};
}
int64_t peer_wait_cycles() { return g_peer_wait_cycles.load(std::memory_order_relaxed); }
void set_peer_wait_cycles(int64_t cycles) {
  TORCH_CHECK(cycles > 0, "rl_b200: the peer wait bound must be positive");
  g_peer_wait_cycles.store(cycles, std::memory_order_relaxed);
}
}  // namespace rlb

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "rl_b200 sm_100a kernels";
  m.def("rmsnorm_fwd", &rmsnorm_fwd);
  m.def("add_rmsnorm_fwd", &add_rmsnorm_fwd);
  m.def("rmsnorm_bwd", &rmsnorm_bwd);
  m.def("rmsnorm_bwd_add", &rmsnorm_bwd_add, py::arg("dy"), py::arg("x"), py::arg("w"), py::arg("rstd"),
        py::arg("ds") = py::none());
  m.def("rope_qkv", &rope_qkv);
  m.def("swiglu_fwd", &swiglu_fwd);
  m.def("swiglu_bwd", &swiglu_bwd);
  m.def("write_kv_cache", &write_kv_cache, py::arg("k"), py::arg("v"), py::arg("k_cache"), py::arg("v_cache"),
        py::arg("slots"), py::arg("k_scale") = 1.0, py::arg("v_scale") = 1.0);
  m.def("logprob_partials", &logprob_partials);
  m.def("logprob_bwd", &logprob_bwd);
  m.def("sample", &sample);
  m.def("adamw_step", &adamw_step);
  m.def("sum_sq", &sum_sq);
  m.def("quant_fp8_block", &quant_fp8_block, py::arg("w"), py::arg("blk"), py::arg("pow2"), py::arg("out") = py::none(),
        py::arg("out_scale") = py::none());
  m.def("quant_fp8_group", &quant_fp8_group);
  m.def("quant_fp8_group_t", &quant_fp8_group_t, "1 x group e4m3 quantisation with MN-major scales [K/group, Mp]");
  m.def("flash_attn_fwd", &flash_attn_fwd);
  m.def("flash_attn_bwd", &flash_attn_bwd);
  m.def("paged_decode_attn", &paged_decode_attn);
  m.def("gemm_nt", &gemm_nt);
  m.def("gemm_error_flag", &gemm_error_flag, py::arg("reset") = false);
  m.def("gemm_rs", &gemm_rs);
  m.def("gemm_sm100", &gemm_sm100, py::arg("a"), py::arg("b"), py::arg("out"), py::arg("a_mn") = false,
        py::arg("b_mn") = false, py::arg("accumulate") = false, py::arg("tile") = 0,
        "tcgen05 GEMM out = op(a) op(b)^T; a [M,K] or [K,M] (a_mn), b [N,K] or [K,N] (b_mn); bf16 or fp32 (+=) out");
  m.def("flash_attn_fwd_tc", &flash_attn_fwd_tc, "tcgen05 varlen flash-attention forward (head dim 128)");
  m.def("flash_attn_seg_fwd_tc", &flash_attn_seg_fwd_tc, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("seg"),
        py::arg("max_q"), py::arg("scale"), py::arg("cp_flags") = py::none(), py::arg("cp_epoch") = 0,
        py::arg("cp_size") = 0, "tcgen05 segment flash-attention forward (head dim 128)");
  m.def("flash_attn_bwd_tc", &flash_attn_bwd_tc, "tcgen05 varlen flash-attention backward (head dim 128)");
  m.def("flash_attn_seg_bwd_tc", &flash_attn_seg_bwd_tc, "tcgen05 segment flash-attention backward (head dim 128)");
  m.def("attn_tc_error_flag", &attn_tc_error_flag, py::arg("reset") = false);
  m.def("peer_wait_cycles", &rlb::peer_wait_cycles,
        "bound (SM cycles) of every in-kernel wait on a peer's or a copy engine's flag");
  m.def("set_peer_wait_cycles", &rlb::set_peer_wait_cycles, py::arg("cycles"));
  m.def("gemm_sm100_error_flag", &gemm_sm100_error_flag, py::arg("reset") = false);
  m.def("gemm_logprob_partials", &gemm_logprob_partials);
  m.def("gemm_dlogits", &gemm_dlogits);
  m.def("gemm_fp8", &gemm_fp8, py::arg("a"), py::arg("a_scale"), py::arg("b"), py::arg("b_scale"),
        py::arg("splits") = 0, "block-scaled e4m3 GEMM (1x128 activation, 128x128 weight fp32 scales) -> bf16");
  m.def("gemm_mxf8", &gemm_mxf8, py::arg("a"), py::arg("a_scale_t"), py::arg("b"), py::arg("b_scale_t"),
        py::arg("splits") = 0, "e4m3 GEMM with power-of-two block scales applied by the tensor cores -> bf16");
  m.def("gemm_fp8_error_flag", &gemm_fp8_error_flag, py::arg("reset") = false);
  m.def("grouped_gemm_nt", &grouped_gemm_nt, "per-expert bf16 GEMM, rows grouped by expert (tcgen05)");
  m.def("grouped_gemm_error_flag", &grouped_gemm_error_flag, py::arg("reset") = false);
  m.def("symm_alloc", &symm_alloc);
  m.def("symm_open", &symm_open);
  m.def("symm_close", &symm_close);
  m.def("symm_view", &symm_view);
  m.def("dp_reduce_shard", &dp_reduce_shard, "DP gradient reduce-scatter over NVLink peer loads (+ norm partials)");
  m.def("dp_wait_ready", &dp_wait_ready, "bounded wait until every DP rank published a gradient bucket's epoch");
  m.def("dp_error_flag", &dp_error_flag, "error word of the DP bucket-readiness waits (1000 + bucket on expiry)");
  m.def("dp_adam_allgather", &dp_adam_allgather, "sharded AdamW fused with the parameter all-gather (peer stores)");
  m.def("gemm_ag", &gemm_ag, "all-gather -> GEMM: waits per gathered shard (copy-engine transfers) on device flags");
  m.def("bounds_errors", &bounds_errors, "bounds-checked debug build: error word per instrumented file (site<<40|index)");
  m.def("debug_bounds_build", &debug_bounds_build, "whether this library is the bounds-checked debug build");
  m.def("nvls_barrier", &nvls_barrier, "bounded signal-word barrier over a multicast group's ranks");
  m.def("nvls_all_reduce", &nvls_all_reduce, "in-place sum through NVSwitch multicast (multimem.ld_reduce / st)");
  m.def("nvls_reduce_shard", &nvls_reduce_shard, "sum of a multicast range into a local tensor (multimem.ld_reduce)");
  m.def("nvls_error_flag", &nvls_error_flag, "error word of the NVLS barrier waits");
  m.def("moe_router_topk", &moe_router_topk, "MoE router: softmax, top-k and the expert-grouped permutation");
  m.def("ep_scatter", &ep_scatter, "MoE token rows -> peers' receive buffers at their final positions (P2P stores)");
  m.def("ep_consume", &ep_consume, "wait for every source's scatter, copy the received rows out, acknowledge");
  m.def("ep_error_flag", &ep_error_flag, py::arg("reset") = false);
  m.def("flash_attn_seg_fwd", &flash_attn_seg_fwd, "segment attention (query chunks vs key prefixes), forward",
        py::arg("q"), py::arg("k"), py::arg("v"), py::arg("seg"), py::arg("max_q"), py::arg("scale"),
        py::arg("cp_flags") = py::none(), py::arg("cp_epoch") = 0, py::arg("cp_size") = 0);
  m.def("attn_error_flag", &attn_error_flag, py::arg("reset") = false);
  m.def("flash_attn_seg_bwd", &flash_attn_seg_bwd, "segment attention backward (shared keys accumulate)");
  m.def("spec_verify", &spec_verify, "speculative decoding: rejection-sampling verification of draft tokens");
  m.def("ar_add_rmsnorm", &ar_add_rmsnorm, "TP all-reduce (peer loads) + residual add + RMSNorm, one kernel");
  m.def("decode_ar_error_flag", &decode_ar_error_flag, py::arg("reset") = false);
  m.def("stream_write_u32", &stream_write_u32, "stream memory write (no kernel) of a 32-bit word");
  m.def("gemm_decode", &gemm_decode, "decode-shaped (<= 256 rows) split-K tcgen05 GEMM: x @ w^T");
  m.def("gemm_decode_split", &gemm_decode_split, "gemm_decode with an explicit K split (1, 2, 4 or 8; 0 = choose)");
  m.def("gemm_decode_error_flag", &gemm_decode_error_flag, py::arg("reset") = false);
  m.def("refit_copy", &refit_copy, "train->rollout reshard (bf16) reading peer shards over NVLink");
  m.def("refit_quant_fp8", &refit_quant_fp8, "train->rollout reshard fused with 128x128 e4m3 block quantisation");
}
