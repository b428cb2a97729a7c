// Python bindings of the sm_100a kernel library (hrm_text_b200._C).
#include <torch/extension.h>

namespace hrm {
void gemm(const at::Tensor& a, bool a_mn, const at::Tensor& b, bool b_mn, int64_t M, int64_t N, int64_t K,
          int64_t epi, const at::Tensor& out, const c10::optional<at::Tensor>& out2,
          const c10::optional<at::Tensor>& residual, const c10::optional<at::Tensor>& aux,
          const c10::optional<at::Tensor>& positions, const c10::optional<at::Tensor>& cos_tab,
          const c10::optional<at::Tensor>& sin_tab, int64_t rope_begin, int64_t rope_end, int64_t pair_offset,
          const c10::optional<at::Tensor>& labels, const c10::optional<at::Tensor>& ce_max,
          const c10::optional<at::Tensor>& ce_sum, const c10::optional<at::Tensor>& ce_arg,
          const c10::optional<at::Tensor>& ce_tgt, bool stream_k, int64_t splitk,
          const c10::optional<at::Tensor>& jobs);
void copy_jobs(const at::Tensor& jobs, int64_t device);
int64_t gemm_balanced_split(int64_t s0, int64_t tiles, int64_t units, int64_t nk);
void shard_update(const at::Tensor& items, const at::Tensor& buf, const std::vector<int64_t>& offs,
                  const at::Tensor& full_grad, const at::Tensor& shard16, const at::Tensor& ran, int64_t world,
                  int64_t rank, const at::Tensor& hyper, double beta1, double beta2, double wd, double ema_decay);
int64_t attn_schedule_capacity(int64_t T, int64_t n_cu);
void attn_schedule(const at::Tensor& cu_seqlens, const at::Tensor& prefix_lens, bool causal, int64_t T,
                   const at::Tensor& sched);
void attn_fwd(const at::Tensor& qkv, int64_t H, const at::Tensor& sched, const at::Tensor& out, const at::Tensor& y,
              const at::Tensor& lse);
void attn_fwd_tc(const at::Tensor& qkv, int64_t H, const at::Tensor& sched, const at::Tensor& out,
                 const at::Tensor& y, const at::Tensor& lse);
at::Tensor wait_flag_probe(const at::Tensor& flag, int64_t expected, double timeout_s);
at::Tensor sample_tokens(const at::Tensor& logits, double temp, int64_t seed, int64_t offset);
at::Tensor decode_attention(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                            const at::Tensor& total);
at::Tensor decode_attention_gqkv(const at::Tensor& gqkv, int64_t H, const at::Tensor& k_cache,
                                 const at::Tensor& v_cache, const at::Tensor& lengths);
void decode_linear_finish(const at::Tensor& acc, int64_t epi, const at::Tensor& out,
                          const c10::optional<at::Tensor>& residual, const c10::optional<at::Tensor>& positions,
                          const c10::optional<at::Tensor>& cos_tab, const c10::optional<at::Tensor>& sin_tab,
                          int64_t rope_begin, int64_t rope_end, int64_t pair_offset);
void attn_bwd_set_profile(bool enabled);
at::Tensor attn_bwd_phase_counters(bool reset);
void attn_bwd_tc(const at::Tensor& qkv, int64_t H, const at::Tensor& sched, const at::Tensor& out,
                 const at::Tensor& lse, const at::Tensor& dy, const at::Tensor& positions, const at::Tensor& cos_tab,
                 const at::Tensor& sin_tab, const at::Tensor& d_out, const at::Tensor& dsum, const at::Tensor& dq_acc,
                 const at::Tensor& dqkv);
void attn_bwd(const at::Tensor& qkv, int64_t H, const at::Tensor& sched, const at::Tensor& out,
              const at::Tensor& lse, const at::Tensor& dy, const at::Tensor& positions, const at::Tensor& cos_tab,
              const at::Tensor& sin_tab, const at::Tensor& d_out, const at::Tensor& dsum, const at::Tensor& dq_acc,
              const at::Tensor& dqkv);
void rmsnorm_fwd(const at::Tensor& x, const c10::optional<at::Tensor>& inj, const c10::optional<at::Tensor>& s_out,
                 const at::Tensor& y, const at::Tensor& rstd, int64_t T, double eps);
void rmsnorm_bwd(const at::Tensor& dy, const at::Tensor& s, const at::Tensor& rstd,
                 const c10::optional<at::Tensor>& dres, const at::Tensor& dx, int64_t T);
void embedding_fwd(const at::Tensor& ids, const at::Tensor& w, const at::Tensor& out, double scale);
void embedding_bwd(const at::Tensor& ids, const at::Tensor& dout, const at::Tensor& gw, double scale);
void ce_finalize(const at::Tensor& pmax, const at::Tensor& psum, const at::Tensor& parg, const at::Tensor& tgt,
                 const at::Tensor& labels, const at::Tensor& lse, const at::Tensor& loss_rows,
                 const at::Tensor& correct);
void ce_dlogits(const at::Tensor& logits, const at::Tensor& lse, const at::Tensor& labels, const at::Tensor& grad);
void adam_atan2(const at::Tensor& p, const at::Tensor& g, const c10::optional<at::Tensor>& m, const at::Tensor& v,
                const c10::optional<at::Tensor>& ema, const c10::optional<at::Tensor>& out16, const at::Tensor& hyper,
                double beta1, double beta2, double wd, double ema_decay);
void cast_f32_bf16(const at::Tensor& src, const at::Tensor& dst);
at::Tensor device_error_word();
bool debug_bounds_build();
}  // namespace hrm

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "HRM-Text sm_100a kernels";
  m.def("gemm", &hrm::gemm, "tcgen05 GEMM with fused epilogues");
  m.def("gemm_balanced_split", &hrm::gemm_balanced_split,
        "split-K factor chosen for an fp32 weight gradient (L2-sized split s0, tiles, CTA pairs, k-blocks)");
  m.def("copy_jobs", &hrm::copy_jobs, "fused-collective copy jobs (gather / push) without a GEMM to ride on");
  m.def("shard_update", &hrm::shard_update, "step-end inbox reduction + AdamATan2 on this rank's shards");
  m.def("attn_schedule_capacity", &hrm::attn_schedule_capacity);
  m.def("attn_schedule", &hrm::attn_schedule);
  m.def("attn_fwd", &hrm::attn_fwd);
  m.def("attn_fwd_tc", &hrm::attn_fwd_tc, "tcgen05 PrefixLM attention forward");
  m.def("attn_bwd", &hrm::attn_bwd);
  m.def("attn_bwd_tc", &hrm::attn_bwd_tc, "tcgen05 PrefixLM attention backward");
  m.def("decode_attention", &hrm::decode_attention, "split-KV decode attention against a static KV cache");
  m.def("decode_linear_finish", &hrm::decode_linear_finish,
        "bf16 output of a split-K decode-step linear layer with the RoPE / SwiGLU / residual epilogues");
  m.def("decode_attention_gqkv", &hrm::decode_attention_gqkv,
        "decode step attention from the fused projection: KV append, split-KV attention, sigmoid gate");
  m.def("sample_tokens", &hrm::sample_tokens, "greedy / Gumbel-max token sampling (fused, one CTA per row)");
  m.def("wait_flag_probe", &hrm::wait_flag_probe, "bounded device wait on a flag (failure-detection probe)");
  m.def("attn_bwd_set_profile", &hrm::attn_bwd_set_profile, "enable per-phase clock tracing of attn_bwd_tc");
  m.def("attn_bwd_phase_counters", &hrm::attn_bwd_phase_counters, "read (and optionally reset) the phase counters");
  m.def("rmsnorm_fwd", &hrm::rmsnorm_fwd);
  m.def("rmsnorm_bwd", &hrm::rmsnorm_bwd);
  m.def("embedding_fwd", &hrm::embedding_fwd);
  m.def("embedding_bwd", &hrm::embedding_bwd);
  m.def("ce_finalize", &hrm::ce_finalize);
  m.def("ce_dlogits", &hrm::ce_dlogits);
  m.def("adam_atan2", &hrm::adam_atan2);
  m.def("cast_f32_bf16", &hrm::cast_f32_bf16);
  m.def("device_error_word", &hrm::device_error_word);
  m.def("debug_bounds_build", &hrm::debug_bounds_build, "built with HRM_DEBUG_BOUNDS (device bounds checks)");
}
