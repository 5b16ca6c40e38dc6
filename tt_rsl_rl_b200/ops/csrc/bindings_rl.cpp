// Python bindings of the RL kernels. Tensors are validated for device and dtype; descriptor tables ("plans") are
// built once on the host and copied to persistent device tensors so launches stay capturable in CUDA graphs.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <vector>

#include "kernels.cuh"
#include "env_kernels.cuh"
#include "rl_kernels.cuh"

namespace {

using torch::Tensor;
using OptT = c10::optional<Tensor>;

cudaStream_t cur() { return at::cuda::getCurrentCUDAStream(); }

void ok(cudaError_t e, const char* what) { TORCH_CHECK(e == cudaSuccess, what, " failed: ", cudaGetErrorString(e)); }

template <typename T>
T* P(const OptT& t) {
  return (t.has_value() && t->defined()) ? reinterpret_cast<T*>(t->data_ptr()) : nullptr;
}
template <typename T>
T* P(const Tensor& t) {
  return reinterpret_cast<T*>(t.data_ptr());
}

void check_f32(const Tensor& t, const char* n) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == torch::kFloat32, n, " must be a CUDA float32 tensor");
}
// Elements addressable from t's first element to the end of its storage (row-padded views may address past numel()).
int64_t avail(const Tensor& t) {
  return static_cast<int64_t>(t.storage().nbytes() / t.element_size()) - t.storage_offset();
}

void check_bf16(const Tensor& t, const char* n) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == torch::kBFloat16, n, " must be a CUDA bfloat16 tensor");
}

int flag_dtype(const Tensor& t) {
  if (t.scalar_type() == torch::kFloat32) return 0;
  if (t.scalar_type() == torch::kBool || t.scalar_type() == torch::kUInt8) return 1;
  if (t.scalar_type() == torch::kInt64) return 2;
  TORCH_CHECK(false, "flag tensors must be float32, bool, uint8 or int64");
  return 0;
}

// ---------------------------------------------------------------------------------------------------------------
void prep_obs(const std::vector<Tensor>& srcs, const OptT& store, int64_t ld_store, const Tensor& x, int64_t ld_x,
              const OptT& mean, const OptT& std, double eps) {
  TORCH_CHECK(!srcs.empty() && srcs.size() <= rlb::kMaxObsGroups, "prep_obs: 1..4 observation groups");
  check_bf16(x, "x");
  rlb::PrepObsArgs a{};
  a.groups = static_cast<int>(srcs.size());
  a.rows = static_cast<int>(srcs[0].size(0));
  int D = 0;
  for (size_t g = 0; g < srcs.size(); ++g) {
    check_f32(srcs[g], "observation group");
    TORCH_CHECK(srcs[g].dim() == 2 && srcs[g].size(0) == a.rows && srcs[g].stride(1) == 1, "bad observation group");
    a.src[g] = P<const float>(srcs[g]);
    a.src_ld[g] = static_cast<int>(srcs[g].stride(0));
    a.width[g] = static_cast<int>(srcs[g].size(1));
    D += a.width[g];
  }
  TORCH_CHECK(ld_x >= D && x.numel() >= (a.rows - 1) * ld_x + D, "prep_obs: x too small");
  a.store = P<float>(store);
  if (a.store) TORCH_CHECK(ld_store >= D && avail(*store) >= (a.rows - 1) * ld_store + D, "prep_obs: store too small");
  a.ld_store = static_cast<int>(ld_store);
  a.x = x.data_ptr();
  a.ld_x = static_cast<int>(ld_x);
  a.mean = P<const float>(mean);
  a.std = P<const float>(std);
  a.eps = static_cast<float>(eps);
  ok(rlb::prep_obs(a, cur()), "prep_obs");
}

void gaussian_sample(const Tensor& head, int64_t ld_head, int64_t rows, int64_t A, bool hetero, bool log_std,
                     const OptT& std_param, double std_lo, double std_hi, double log_lo, double log_hi, int64_t seed,
                     const Tensor& counter, const Tensor& ticket, const Tensor& actions, const Tensor& out_mean,
                     const Tensor& out_std, const Tensor& out_logp, const OptT& actions_copy) {
  check_f32(head, "head");
  TORCH_CHECK(counter.scalar_type() == torch::kInt64 && ticket.scalar_type() == torch::kInt32, "counter/ticket dtype");
  TORCH_CHECK(actions.numel() >= rows * A && out_mean.numel() >= rows * A && out_std.numel() >= rows * A &&
                  out_logp.numel() >= rows,
              "gaussian_sample: outputs too small");
  TORCH_CHECK(hetero || (std_param.has_value() && std_param->numel() >= A), "gaussian_sample: std_param required");
  rlb::SampleArgs a{};
  a.head = P<const float>(head);
  a.ld_head = static_cast<int>(ld_head);
  a.rows = static_cast<int>(rows);
  a.A = static_cast<int>(A);
  a.hetero = hetero;
  a.log_std = log_std;
  a.std_param = P<const float>(std_param);
  a.std_lo = static_cast<float>(std_lo);
  a.std_hi = static_cast<float>(std_hi);
  a.log_std_lo = static_cast<float>(log_lo);
  a.log_std_hi = static_cast<float>(log_hi);
  a.seed = static_cast<uint64_t>(seed);
  a.counter = reinterpret_cast<uint64_t*>(counter.data_ptr());
  a.ticket = reinterpret_cast<unsigned int*>(ticket.data_ptr());
  a.actions = P<float>(actions);
  a.out_mean = P<float>(out_mean);
  a.out_std = P<float>(out_std);
  a.out_logp = P<float>(out_logp);
  a.actions_copy = P<float>(actions_copy);
  ok(rlb::gaussian_sample(a, cur()), "gaussian_sample");
}

void process_step(const Tensor& rewards, const OptT& intrinsic, const Tensor& dones, const OptT& timeouts,
                  const Tensor& values_slot, double gamma, const Tensor& rewards_slot, const Tensor& dones_slot,
                  const OptT& nonfinite) {
  check_f32(rewards, "rewards");
  const int64_t n = rewards.numel();
  TORCH_CHECK(dones.numel() == n && rewards_slot.numel() >= n && dones_slot.numel() >= n, "process_step: sizes");
  rlb::ProcessArgs a{};
  a.rewards = P<const float>(rewards);
  a.intrinsic = P<const float>(intrinsic);
  a.dones = dones.data_ptr();
  a.dones_dtype = flag_dtype(dones);
  if (timeouts.has_value() && timeouts->defined()) {
    TORCH_CHECK(timeouts->numel() == n, "process_step: time_outs size");
    a.timeouts = timeouts->data_ptr();
    a.timeouts_dtype = flag_dtype(*timeouts);
  }
  a.values_slot = P<const float>(values_slot);
  a.gamma = static_cast<float>(gamma);
  a.rows = static_cast<int>(n);
  a.rewards_slot = P<float>(rewards_slot);
  a.dones_slot = P<float>(dones_slot);
  a.nonfinite_flag = P<unsigned int>(nonfinite);
  ok(rlb::process_step(a, cur()), "process_step");
}

int64_t gae_blocks(int64_t N) { return rlb::gae_blocks(static_cast<int>(N)); }

void gae(const Tensor& rewards, const Tensor& dones, const Tensor& values, const Tensor& last_values,
         const Tensor& returns, const Tensor& advantages, int64_t T, int64_t N, double gamma, double lam,
         const Tensor& partial) {
  for (const Tensor* t : {&rewards, &dones, &values, &returns, &advantages}) {
    check_f32(*t, "gae buffer");
    TORCH_CHECK(t->numel() >= T * N, "gae: buffer too small");
  }
  TORCH_CHECK(partial.scalar_type() == torch::kFloat64 && partial.numel() >= 2 * rlb::gae_blocks(N), "gae: partial");
  rlb::GaeArgs a{P<const float>(rewards), P<const float>(dones), P<const float>(values), P<const float>(last_values),
                 P<float>(returns),       P<float>(advantages),    static_cast<int>(T),   static_cast<int>(N),
                 static_cast<float>(gamma), static_cast<float>(lam), P<double>(partial)};
  ok(rlb::gae(a, cur()), "gae");
}

void adv_normalize(const Tensor& adv, const Tensor& partial, int64_t parts) {
  check_f32(adv, "adv");
  ok(rlb::adv_normalize(P<float>(adv), adv.numel(), P<const double>(partial), static_cast<int>(parts), cur()),
     "adv_normalize");
}

int64_t feistel_half_bits(int64_t total) { return rlb::feistel_half_bits(total); }
int64_t feistel_permute(int64_t i, int64_t n, int64_t half_bits, int64_t key) {
  return rlb::feistel_permute_host(static_cast<uint32_t>(i), static_cast<uint32_t>(n), static_cast<uint32_t>(half_bits),
                                   static_cast<uint32_t>(key));
}

void gather_minibatch(int64_t B, int64_t offset, int64_t total, const OptT& key, int64_t half_bits, const OptT& idx_in,
                      const Tensor& idx_out, const std::vector<Tensor>& obs, const std::vector<OptT>& means,
                      const std::vector<OptT>& stds, double eps, const std::vector<Tensor>& xs,
                      const std::vector<int64_t>& ld_xs, const OptT& status, int64_t copies,
                      const std::vector<int64_t>& rows, const std::vector<OptT>& perms,
                      const std::vector<OptT>& signs) {
  const size_t nm = obs.size();
  TORCH_CHECK(nm >= 1 && nm <= static_cast<size_t>(rlb::kGatherModels) && xs.size() == nm && ld_xs.size() == nm &&
                  means.size() == nm && stds.size() == nm && rows.size() == nm && perms.size() == nm &&
                  signs.size() == nm,
              "gather_minibatch: 1 to 3 models with one entry per model in every list");
  TORCH_CHECK(copies >= 1, "gather_minibatch: copies >= 1");
  TORCH_CHECK(idx_out.scalar_type() == torch::kInt32 && idx_out.numel() >= B, "gather_minibatch: idx_out");
  TORCH_CHECK(total < (1ll << 31), "gather_minibatch: rollout too large");
  rlb::GatherArgs a{};
  a.B = static_cast<int>(B);
  a.offset = offset;
  a.total = total;
  a.key_ptr = P<const uint32_t>(key);
  a.half_bits = static_cast<int>(half_bits);
  a.idx_in = P<const int>(idx_in);
  a.idx_out = P<int>(idx_out);
  a.copies = static_cast<int>(copies);
  a.models = static_cast<int>(nm);
  for (size_t m = 0; m < nm; ++m) {
    check_f32(obs[m], "obs");
    check_bf16(xs[m], "x");
    TORCH_CHECK(obs[m].dim() == 2 && obs[m].size(0) >= total, "gather_minibatch: obs must be [rows, dim]");
    a.obs[m] = P<const float>(obs[m]);
    a.obs_ld[m] = static_cast<int>(obs[m].stride(0));
    a.dim[m] = static_cast<int>(obs[m].size(1));
    a.rows[m] = static_cast<int>(rows[m]);
    TORCH_CHECK(rows[m] >= 1 && rows[m] <= copies * B, "gather_minibatch: rows per model in [1, copies * B]");
    a.mean[m] = P<const float>(means[m]);
    a.std[m] = P<const float>(stds[m]);
    a.x[m] = xs[m].data_ptr();
    a.ld_x[m] = static_cast<int>(ld_xs[m]);
    // bf16 rows are written in 4-column (8-byte) groups up to the next multiple of 4 columns
    TORCH_CHECK(ld_xs[m] % 4 == 0 && ld_xs[m] >= (a.dim[m] + 3) / 4 * 4 &&
                    (reinterpret_cast<uintptr_t>(xs[m].data_ptr()) % 8) == 0,
                "gather_minibatch: x pitch must be a multiple of 4 covering dim rounded up to 4, 8-byte aligned");
    TORCH_CHECK(xs[m].numel() >= (rows[m] - 1) * ld_xs[m] + (a.dim[m] + 3) / 4 * 4, "gather_minibatch: x too small");
    TORCH_CHECK(obs[m].stride(1) == 1, "gather_minibatch: obs rows must be contiguous");
    // 16-byte loads read whole 4-column groups: the last group of the last row must lie inside the storage
    a.vec4[m] = (a.obs_ld[m] % 4 == 0 && (reinterpret_cast<uintptr_t>(obs[m].data_ptr()) % 16) == 0 &&
                 avail(obs[m]) >= (total - 1) * a.obs_ld[m] + (a.dim[m] + 3) / 4 * 4)
                    ? 1
                    : 0;
    if (perms[m].has_value()) {
      TORCH_CHECK(signs[m].has_value(), "gather_minibatch: perm without sign");
      TORCH_CHECK(perms[m]->scalar_type() == torch::kInt32 && perms[m]->numel() >= copies * a.dim[m] &&
                      perms[m]->is_contiguous(),
                  "gather_minibatch: perm must be int32 [copies, dim]");
      check_f32(*signs[m], "sign");
      TORCH_CHECK(signs[m]->numel() >= copies * a.dim[m], "gather_minibatch: sign must be [copies, dim]");
      a.perm[m] = P<const int>(perms[m]);
      a.sign[m] = P<const float>(signs[m]);
    }
  }
  a.eps = static_cast<float>(eps);
  a.status = P<unsigned int>(status);
  ok(rlb::gather_minibatch(a, cur()), "gather_minibatch");
}

int64_t ppo_loss_blocks(int64_t B) { return rlb::ppo_loss_blocks(static_cast<int>(B)); }

void ppo_loss(int64_t B, int64_t A, bool hetero, bool log_std, const Tensor& head, int64_t ld_head, const Tensor& value,
              int64_t ld_value, const OptT& std_param, double std_lo, double std_hi, double log_lo, double log_hi,
              const Tensor& idx, const Tensor& st_actions, const Tensor& st_mean, const Tensor& st_std,
              const Tensor& st_logp, const Tensor& st_adv, const Tensor& st_ret, const Tensor& st_val,
              const OptT& adv_override, double clip, double value_coef, double entropy_coef, bool clipped_value,
              const Tensor& d_head, int64_t ld_dhead, const Tensor& d_value, int64_t ld_dvalue,
              const Tensor& stats_partial, const Tensor& dhead_colsum, const Tensor& dvalue_colsum,
              const OptT& dstd_partial, int64_t copies, bool aug, const OptT& act_perm, const OptT& act_sign,
              double mirror_coef, const OptT& status) {
  // B: original samples of the minibatch; the actor rows are copies * B (symmetry copies after the originals)
  check_f32(head, "head");
  check_f32(value, "value");
  check_bf16(d_head, "d_head");
  check_bf16(d_value, "d_value");
  TORCH_CHECK(copies >= 1, "ppo_loss: copies >= 1");
  const int64_t rows = copies * B;
  const int64_t value_rows = aug ? rows : B;
  TORCH_CHECK(idx.scalar_type() == torch::kInt32 && idx.numel() >= B, "ppo_loss: idx");
  const int64_t blocks = rlb::ppo_loss_blocks(static_cast<int>(rows));
  const int64_t head_cols = hetero ? 2 * A : A;
  TORCH_CHECK(ld_dhead >= head_cols && d_head.numel() >= rows * ld_dhead, "ppo_loss: d_head too small");
  TORCH_CHECK(head.numel() >= (rows - 1) * ld_head + head_cols, "ppo_loss: head too small");
  TORCH_CHECK(d_value.numel() >= value_rows * ld_dvalue && value.numel() >= (value_rows - 1) * ld_value + 1,
              "ppo_loss: value / d_value too small");
  TORCH_CHECK(stats_partial.numel() >= blocks * rlb::kLossStats && dhead_colsum.numel() >= blocks * head_cols &&
                  dvalue_colsum.numel() >= blocks,
              "ppo_loss: partial buffers too small");
  TORCH_CHECK(hetero || (std_param.has_value() && dstd_partial.has_value()), "ppo_loss: std_param/dstd_partial");
  TORCH_CHECK(copies == 1 || (act_perm.has_value() && act_sign.has_value() &&
                              act_perm->scalar_type() == torch::kInt32 && act_perm->numel() >= copies * A &&
                              act_sign->numel() >= copies * A),
              "ppo_loss: symmetry copies need int32 act_perm and act_sign [copies, A]");
  rlb::PpoLossArgs a{};
  a.B = static_cast<int>(rows);
  a.n0 = static_cast<int>(B);
  a.copies = static_cast<int>(copies);
  a.aug = aug ? 1 : 0;
  a.act_perm = copies > 1 ? P<const int>(act_perm) : nullptr;
  a.act_sign = copies > 1 ? P<const float>(act_sign) : nullptr;
  a.mirror_coef = static_cast<float>(mirror_coef);
  a.A = static_cast<int>(A);
  a.hetero = hetero;
  a.log_std = log_std;
  a.head = P<const float>(head);
  a.ld_head = static_cast<int>(ld_head);
  a.value = P<const float>(value);
  a.ld_value = static_cast<int>(ld_value);
  a.std_param = P<const float>(std_param);
  a.std_lo = static_cast<float>(std_lo);
  a.std_hi = static_cast<float>(std_hi);
  a.log_std_lo = static_cast<float>(log_lo);
  a.log_std_hi = static_cast<float>(log_hi);
  a.idx = P<const int>(idx);
  a.st_actions = P<const float>(st_actions);
  a.st_mean = P<const float>(st_mean);
  a.st_std = P<const float>(st_std);
  a.st_logp = P<const float>(st_logp);
  a.st_adv = P<const float>(st_adv);
  a.st_ret = P<const float>(st_ret);
  a.st_val = P<const float>(st_val);
  a.adv_override = P<const float>(adv_override);
  a.clip = static_cast<float>(clip);
  a.value_coef = static_cast<float>(value_coef);
  a.entropy_coef = static_cast<float>(entropy_coef);
  a.clipped_value = clipped_value;
  a.d_head = d_head.data_ptr();
  a.ld_dhead = static_cast<int>(ld_dhead);
  a.d_value = d_value.data_ptr();
  a.ld_dvalue = static_cast<int>(ld_dvalue);
  a.stats_partial = P<float>(stats_partial);
  a.dhead_colsum = P<float>(dhead_colsum);
  a.dvalue_colsum = P<float>(dvalue_colsum);
  a.dstd_partial = P<float>(dstd_partial);
  a.total = st_actions.size(0);
  a.status = P<unsigned int>(status);
  ok(rlb::ppo_loss(a, cur()), "ppo_loss");
}

// ---- reduction plan --------------------------------------------------------------------------------------------
// srcs[i]: partial buffer [parts_i, n_i]; dst_offsets[i]: offset into the flat gradient vector.
std::tuple<Tensor, int64_t, int64_t> make_reduce_plan(const std::vector<Tensor>& srcs, const std::vector<int64_t>& parts,
                                                      const std::vector<int64_t>& ns,
                                                      const std::vector<int64_t>& dst_offsets) {
  TORCH_CHECK(srcs.size() == parts.size() && parts.size() == ns.size() && ns.size() == dst_offsets.size() &&
                  !srcs.empty(),
              "make_reduce_plan: list sizes");
  std::vector<rlb::ReduceSegment> segs(srcs.size());
  int chunks = 0;
  for (size_t i = 0; i < srcs.size(); ++i) {
    check_f32(srcs[i], "partial");
    TORCH_CHECK(srcs[i].numel() >= parts[i] * ns[i], "make_reduce_plan: partial buffer too small");
    segs[i].src = P<const float>(srcs[i]);
    segs[i].dst_offset = dst_offsets[i];
    segs[i].n = ns[i];
    segs[i].parts = static_cast<int>(parts[i]);
    segs[i].first_chunk = chunks;
    chunks += static_cast<int>((ns[i] + rlb::kReduceChunk - 1) / rlb::kReduceChunk);
  }
  auto dev = torch::empty({static_cast<int64_t>(segs.size() * sizeof(rlb::ReduceSegment))},
                          torch::dtype(torch::kUInt8).device(srcs[0].device()));
  ok(cudaMemcpy(dev.data_ptr(), segs.data(), segs.size() * sizeof(rlb::ReduceSegment), cudaMemcpyHostToDevice),
     "make_reduce_plan copy");
  return {dev, static_cast<int64_t>(segs.size()), static_cast<int64_t>(chunks)};
}

void reduce_segments(const Tensor& plan, int64_t nseg, int64_t chunks, const Tensor& send0, const Tensor& send1,
                     const OptT& epoch, bool accumulate) {
  check_f32(send0, "send0");
  check_f32(send1, "send1");
  ok(rlb::reduce_segments(reinterpret_cast<const rlb::ReduceSegment*>(plan.data_ptr()), static_cast<int>(nseg),
                          static_cast<int>(chunks), P<float>(send0), P<float>(send1), P<const unsigned int>(epoch),
                          accumulate ? 1 : 0, cur()),
     "reduce_segments");
}

void rnd_intrinsic(const Tensor& target, int64_t ld_target, const Tensor& pred, int64_t ld_pred, int64_t rows,
                   int64_t dim, const Tensor& weight, const Tensor& out, const OptT& disc, double gamma) {
  check_f32(target, "target");
  check_f32(pred, "pred");
  check_f32(weight, "weight");
  check_f32(out, "out");
  TORCH_CHECK(dim <= 64 && out.numel() >= rows && target.numel() >= (rows - 1) * ld_target + dim &&
                  pred.numel() >= (rows - 1) * ld_pred + dim,
              "rnd_intrinsic: sizes");
  if (disc.has_value()) {
    check_f32(*disc, "disc");
    TORCH_CHECK(disc->numel() >= rows, "rnd_intrinsic: disc too small");
  }
  ok(rlb::rnd_intrinsic(P<const float>(target), static_cast<int>(ld_target), P<const float>(pred),
                        static_cast<int>(ld_pred), static_cast<int>(rows), static_cast<int>(dim), P<const float>(weight),
                        P<float>(out), P<float>(disc), static_cast<float>(gamma), cur()),
     "rnd_intrinsic");
}

void rnd_reward_scale(const Tensor& out, int64_t rows, const Tensor& weight, const Tensor& std) {
  check_f32(out, "out");
  check_f32(weight, "weight");
  check_f32(std, "std");
  TORCH_CHECK(out.numel() >= rows, "rnd_reward_scale: out too small");
  ok(rlb::rnd_reward_scale(P<float>(out), static_cast<int>(rows), P<const float>(weight), P<const float>(std), cur()),
     "rnd_reward_scale");
}

void lg_env_step(const Tensor& At, const Tensor& Bt, const Tensor& state, const Tensor& actions, const OptT& noise,
                 double noise_std, double reset_prob, int64_t max_len, const Tensor& ep_len, const Tensor& rewards,
                 const Tensor& dones, const Tensor& time_outs, const Tensor& obs_policy, const OptT& obs_critic,
                 int64_t priv, int64_t seed, const Tensor& counter, const Tensor& ticket) {
  for (const Tensor* t : {&At, &Bt, &state, &actions, &rewards, &dones, &time_outs, &obs_policy}) check_f32(*t, "env");
  const int64_t N = state.size(0), S = state.size(1), A = actions.size(1);
  TORCH_CHECK(At.is_contiguous() && Bt.is_contiguous() && state.is_contiguous() && obs_policy.is_contiguous() &&
                  actions.stride(1) == 1,
              "lg_env_step: contiguous rows expected");
  TORCH_CHECK(At.numel() == S * S && Bt.numel() == A * S && S <= 128 && S % 4 == 0 && A <= 64,
              "lg_env_step: A^T [S, S], B^T [A, S] with S <= 128, S % 4 == 0, A <= 64");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(state.data_ptr()) % 16) == 0 &&
                  (reinterpret_cast<uintptr_t>(obs_policy.data_ptr()) % 16) == 0,
              "lg_env_step: state and policy observations must be 16-byte aligned");
  TORCH_CHECK(obs_policy.numel() == N * S && rewards.numel() == N && dones.numel() == N && time_outs.numel() == N &&
                  ep_len.numel() == N && ep_len.scalar_type() == torch::kInt64,
              "lg_env_step: sizes");
  if (noise.has_value()) {
    check_f32(*noise, "noise");
    TORCH_CHECK(noise->is_contiguous() && noise->numel() == N * S &&
                    (reinterpret_cast<uintptr_t>(noise->data_ptr()) % 16) == 0,
                "lg_env_step: noise");
  }
  if (obs_critic.has_value()) {
    check_f32(*obs_critic, "obs_critic");
    TORCH_CHECK(obs_critic->is_contiguous() && obs_critic->numel() == N * (S + priv), "lg_env_step: critic obs");
  }
  TORCH_CHECK(counter.scalar_type() == torch::kInt64 && ticket.scalar_type() == torch::kInt32, "counter/ticket");
  rlb::LgEnvArgs a{};
  a.N = static_cast<int>(N);
  a.S = static_cast<int>(S);
  a.A = static_cast<int>(A);
  a.P = static_cast<int>(priv);
  a.At = P<const float>(At);
  a.Bt = P<const float>(Bt);
  a.state = P<float>(state);
  a.actions = P<const float>(actions);
  a.ld_act = static_cast<int>(actions.stride(0));
  a.noise = P<const float>(noise);
  a.noise_std = static_cast<float>(noise_std);
  a.reset_prob = static_cast<float>(reset_prob);
  a.max_len = max_len;
  a.ep_len = reinterpret_cast<long long*>(ep_len.data_ptr());
  a.rewards = P<float>(rewards);
  a.dones = P<float>(dones);
  a.time_outs = P<float>(time_outs);
  a.obs_policy = P<float>(obs_policy);
  a.obs_critic = P<float>(obs_critic);
  a.seed = static_cast<uint64_t>(seed);
  a.counter = reinterpret_cast<uint64_t*>(counter.data_ptr());
  a.ticket = reinterpret_cast<unsigned int*>(ticket.data_ptr());
  ok(rlb::lg_env_step(a, cur()), "lg_env_step");
}

int64_t adv_gather_blocks(int64_t n) { return rlb::adv_gather_blocks(n); }

void adv_gather_stats(const Tensor& adv, const Tensor& idx, int64_t n, const Tensor& out, const Tensor& partial,
                      const OptT& status) {
  check_f32(adv, "adv");
  check_f32(out, "out");
  TORCH_CHECK(idx.scalar_type() == torch::kInt32 && idx.numel() >= n && out.numel() >= n, "adv_gather_stats: sizes");
  TORCH_CHECK(partial.scalar_type() == torch::kFloat64 && partial.numel() >= 2 * rlb::adv_gather_blocks(n),
              "adv_gather_stats: partial must be float64 [2 * blocks]");
  ok(rlb::adv_gather_stats(P<const float>(adv), adv.numel(), P<const int>(idx), n, P<float>(out), P<double>(partial),
                           P<unsigned int>(status), cur()),
     "adv_gather_stats");
}

int64_t mse_blocks(int64_t rows) { return rlb::mse_blocks(static_cast<int>(rows)); }

void mse_grad(const Tensor& pred, int64_t ld_pred, const Tensor& target, int64_t ld_target, int64_t rows, int64_t A,
              bool huber, const Tensor& grad, int64_t ld_grad, int64_t head_cols, const Tensor& loss_partial,
              const Tensor& colsum_partial, const Tensor& loss_acc, const Tensor& ticket, const OptT& last_weight,
              int64_t denom_rows) {
  check_f32(pred, "pred");
  check_f32(target, "target");
  check_bf16(grad, "grad");
  check_f32(loss_acc, "loss_acc");
  const int64_t blocks = rlb::mse_blocks(static_cast<int>(rows));
  TORCH_CHECK(pred.numel() >= (rows - 1) * ld_pred + A && target.numel() >= (rows - 1) * ld_target + A &&
                  grad.numel() >= rows * ld_grad && ld_grad >= A && head_cols >= A,
              "mse_grad: sizes");
  TORCH_CHECK(loss_partial.numel() >= blocks && colsum_partial.numel() >= blocks * head_cols, "mse_grad: partials");
  TORCH_CHECK(ticket.scalar_type() == at::kInt && ticket.is_cuda(), "mse_grad: ticket must be int32 on the device");
  rlb::MseArgs a{P<const float>(pred), static_cast<int>(ld_pred), P<const float>(target), static_cast<int>(ld_target),
                 static_cast<int>(rows), static_cast<int>(A), huber ? 1 : 0, grad.data_ptr(),
                 static_cast<int>(ld_grad), static_cast<int>(head_cols), P<float>(loss_partial),
                 P<float>(colsum_partial), P<float>(loss_acc), reinterpret_cast<unsigned int*>(ticket.data_ptr()),
                 nullptr, static_cast<int>(denom_rows)};
  TORCH_CHECK(denom_rows >= 0 && !(denom_rows > 0 && last_weight.has_value()),
              "mse_grad: denom_rows and last_weight are exclusive");
  if (last_weight.has_value()) {
    check_f32(*last_weight, "last_weight");
    TORCH_CHECK(last_weight->numel() >= 1, "mse_grad: last_weight");
    a.last_weight = P<const float>(*last_weight);
  }
  ok(rlb::mse_grad(a, cur()), "mse_grad");
}

// ---- Adam plan -------------------------------------------------------------------------------------------------
// Per tensor: offset, numel, group, rows, cols, shadow (bf16 tensor or None), shadow_ld.
std::tuple<Tensor, Tensor, int64_t> make_adam_plan(const std::vector<int64_t>& offsets, const std::vector<int64_t>& numels,
                                                   const std::vector<int64_t>& groups, const std::vector<int64_t>& rows,
                                                   const std::vector<int64_t>& cols, const std::vector<OptT>& shadows,
                                                   const std::vector<int64_t>& shadow_lds, const Tensor& like) {
  const size_t n = offsets.size();
  TORCH_CHECK(numels.size() == n && groups.size() == n && rows.size() == n && cols.size() == n && shadows.size() == n &&
                  shadow_lds.size() == n,
              "make_adam_plan: list sizes");
  std::vector<rlb::AdamTensor> ts(n);
  std::vector<rlb::AdamChunk> chunks;
  for (size_t i = 0; i < n; ++i) {
    ts[i].offset = offsets[i];
    ts[i].numel = numels[i];
    ts[i].group = static_cast<int>(groups[i]);
    ts[i].rows = static_cast<int>(rows[i]);
    ts[i].cols = static_cast<int>(cols[i]);
    ts[i].shadow = P<void>(shadows[i]);
    ts[i].shadow_ld = static_cast<int>(shadow_lds[i]);
    // Division by the invariant column count (Granlund & Montgomery, "Division by invariant integers using
    // multiplication", PLDI 1994): for d > 1, l = ceil(log2 d), m = ceil(2^(31 + l) / d) < 2^32 and
    // idx / d == umulhi(idx, m) >> (l - 1) for every idx < 2^31. d == 1 is flagged with shift 32.
    {
      const uint64_t d = static_cast<uint64_t>(cols[i] > 0 ? cols[i] : 1);
      if (d == 1) {
        ts[i].cols_magic = 0;
        ts[i].cols_shift = 32;
      } else {
        unsigned int l = 0;
        while ((1ull << l) < d) ++l;
        ts[i].cols_magic = static_cast<unsigned int>(((1ull << (31 + l)) + d - 1) / d);
        ts[i].cols_shift = l - 1;
        const uint64_t probes[6] = {0ull, 1ull, d - 1, d, d + 1, static_cast<uint64_t>(numels[i] - 1)};
        for (uint64_t n : probes) {
          const uint64_t q = ((n * ts[i].cols_magic) >> 32) >> ts[i].cols_shift;
          TORCH_CHECK(q == n / d, "make_adam_plan: division constant check failed");
        }
      }
      TORCH_CHECK(numels[i] < (1ll << 31), "make_adam_plan: tensor too large");
    }
    if (ts[i].shadow) {
      TORCH_CHECK(shadows[i]->scalar_type() == torch::kBFloat16 && shadows[i]->numel() >= rows[i] * shadow_lds[i] &&
                      rows[i] * cols[i] == numels[i],
                  "make_adam_plan: bad shadow");
    }
    for (int64_t s = 0; s < numels[i]; s += rlb::kAdamChunk)
      chunks.push_back({static_cast<int>(i), static_cast<int>(s),
                        static_cast<int>(std::min<int64_t>(rlb::kAdamChunk, numels[i] - s))});
  }
  auto opts = torch::dtype(torch::kUInt8).device(like.device());
  auto dt = torch::empty({static_cast<int64_t>(n * sizeof(rlb::AdamTensor))}, opts);
  auto dc = torch::empty({static_cast<int64_t>(chunks.size() * sizeof(rlb::AdamChunk))}, opts);
  ok(cudaMemcpy(dt.data_ptr(), ts.data(), n * sizeof(rlb::AdamTensor), cudaMemcpyHostToDevice), "adam plan copy");
  ok(cudaMemcpy(dc.data_ptr(), chunks.data(), chunks.size() * sizeof(rlb::AdamChunk), cudaMemcpyHostToDevice),
     "adam plan copy");
  return {dt, dc, static_cast<int64_t>(chunks.size())};
}

int64_t adam_grid(int64_t device) { return rlb::adam_grid(static_cast<int>(device)); }

void adam_step(const Tensor& params, const Tensor& send0, const Tensor& send1, const Tensor& grads, const Tensor& exp_avg,
               const Tensor& exp_avg_sq, const Tensor& tensors, const Tensor& chunks, int64_t nchunks,
               const std::vector<double>& max_norm, const std::vector<double>& beta1, const std::vector<double>& beta2,
               const std::vector<double>& eps, const std::vector<int64_t>& lr_index, const Tensor& lr,
               const OptT& lr_out_slot, const Tensor& step,
               bool adaptive, const OptT& kl_mean, double desired_kl, double lr_min, double lr_max, int64_t world,
               int64_t rank, const OptT& peer_send, const OptT& peer_flags, const Tensor& epoch, int64_t timeout_ns,
               const Tensor& norm_partial, const Tensor& barrier, const OptT& status, const OptT& out_norms,
               int64_t grid, const std::vector<int64_t>& group_ranges, int64_t exchange_len,
               const OptT& peer_reduced, int64_t kl_offset) {
  for (const Tensor* t : {&params, &send0, &send1, &grads, &exp_avg, &exp_avg_sq}) check_f32(*t, "adam buffer");
  const size_t ng = max_norm.size();
  TORCH_CHECK(ng >= 1 && ng <= rlb::kAdamMaxGroups && beta1.size() == ng && beta2.size() == ng && eps.size() == ng,
              "adam_step: groups");
  TORCH_CHECK(lr.numel() >= static_cast<int64_t>(ng) && step.scalar_type() == torch::kInt64, "adam_step: lr/step");
  TORCH_CHECK(norm_partial.numel() >= grid * rlb::kAdamMaxGroups, "adam_step: norm_partial too small");
  TORCH_CHECK(world == 1 || (peer_send.has_value() && peer_flags.has_value()), "adam_step: peers required");
  TORCH_CHECK(barrier.numel() >= 4 && barrier.element_size() == 4, "adam_step: barrier must hold 4 uint32");
  if (world > 1) {
    TORCH_CHECK(peer_send->numel() >= 2 * world && peer_flags->numel() >= world, "adam_step: peer tables too small");
  }
  rlb::AdamArgs a{};
  a.params = P<float>(params);
  a.send[0] = P<float>(send0);
  a.send[1] = P<float>(send1);
  a.grads = P<float>(grads);
  a.exp_avg = P<float>(exp_avg);
  a.exp_avg_sq = P<float>(exp_avg_sq);
  a.tensors = reinterpret_cast<const rlb::AdamTensor*>(tensors.data_ptr());
  a.chunks = reinterpret_cast<const rlb::AdamChunk*>(chunks.data_ptr());
  a.nchunks = static_cast<int>(nchunks);
  a.ngroups = static_cast<int>(ng);
  for (size_t g = 0; g < ng; ++g) {
    a.max_norm[g] = static_cast<float>(max_norm[g]);
    a.beta1[g] = static_cast<float>(beta1[g]);
    a.beta2[g] = static_cast<float>(beta2[g]);
    a.eps[g] = static_cast<float>(eps[g]);
    TORCH_CHECK(g < lr_index.size() && lr_index[g] >= 0 && lr_index[g] < static_cast<int64_t>(ng), "adam_step: lr_index");
    a.lr_index[g] = static_cast<int>(lr_index[g]);
  }
  a.lr = P<float>(lr);
  a.lr_out_slot = P<float>(lr_out_slot);
  a.step = reinterpret_cast<long long*>(step.data_ptr());
  a.adaptive = adaptive;
  a.kl_mean = P<const float>(kl_mean);
  TORCH_CHECK(!adaptive || a.kl_mean, "adam_step: adaptive schedule needs kl_mean");
  a.desired_kl = static_cast<float>(desired_kl);
  a.lr_min = static_cast<float>(lr_min);
  a.lr_max = static_cast<float>(lr_max);
  a.world = static_cast<int>(world);
  a.rank = static_cast<int>(rank);
  a.peer_send = P<float* const>(peer_send);
  a.peer_flags = P<unsigned int* const>(peer_flags);
  a.epoch = reinterpret_cast<unsigned int*>(epoch.data_ptr());
  a.timeout_ns = static_cast<uint64_t>(timeout_ns);
  a.norm_partial = P<float>(norm_partial);
  a.barrier = reinterpret_cast<unsigned int*>(barrier.data_ptr());
  a.status = P<unsigned int>(status);
  a.out_norms = P<float>(out_norms);
  TORCH_CHECK(group_ranges.size() == 2 * ng, "adam_step: group_ranges must hold [begin, end) per group");
  for (size_t g = 0; g < ng; ++g) {
    a.group_begin[g] = group_ranges[2 * g];
    a.group_end[g] = group_ranges[2 * g + 1];
  }
  TORCH_CHECK(exchange_len % 4 == 0 && send0.numel() >= exchange_len && send1.numel() >= exchange_len &&
                  grads.numel() >= exchange_len,
              "adam_step: exchange_len must be a multiple of 4 within the buffers");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(send0.data_ptr()) % 16) == 0 &&
                  (reinterpret_cast<uintptr_t>(send1.data_ptr()) % 16) == 0 &&
                  (reinterpret_cast<uintptr_t>(grads.data_ptr()) % 16) == 0,
              "adam_step: exchange buffers must be 16-byte aligned");
  TORCH_CHECK(world <= 8, "adam_step: at most 8 ranks");
  a.exchange_len = exchange_len;
  // two-shot exchange: peer table of the ranks' reduced buffers (exchange_len + 8 floats each), shards of
  // ceil(n4 / world) float4 elements, the KL statistic read from its owner
  a.peer_reduced = nullptr;
  a.shard4 = 0;
  a.kl_offset = -1;
  if (peer_reduced.has_value() && peer_reduced->defined() && world > 1) {
    TORCH_CHECK(peer_reduced->numel() >= world && peer_reduced->scalar_type() == torch::kInt64,
                "adam_step: peer_reduced must hold one int64 device pointer per rank");
    TORCH_CHECK(!adaptive || (kl_offset >= 0 && kl_offset < exchange_len),
                "adam_step: the two-shot exchange with an adaptive schedule needs the KL statistic's offset");
    a.peer_reduced = P<float* const>(peer_reduced);
    const long long n4 = exchange_len / 4;
    a.shard4 = (n4 + world - 1) / world;
    a.kl_offset = kl_offset;
  }
  ok(rlb::adam_step(a, static_cast<int>(grid), cur()), "adam_step");
}

int64_t colstats_chunks(int64_t rows) { return rlb::colstats_chunks(rows); }

void colstats(const Tensor& x, int64_t rows, int64_t ld, int64_t dim, const Tensor& partial) {
  check_f32(x, "x");
  const int chunks = rlb::colstats_chunks(rows);
  TORCH_CHECK(partial.scalar_type() == torch::kFloat64 && partial.numel() >= 2LL * chunks * dim, "colstats: partial");
  TORCH_CHECK(avail(x) >= (rows - 1) * ld + dim, "colstats: x too small");
  rlb::ColStatsArgs a{P<const float>(x), rows, static_cast<int>(ld), static_cast<int>(dim), P<double>(partial), chunks};
  ok(rlb::colstats(a, cur()), "colstats");
}

void norm_update(const Tensor& partial, int64_t chunks, int64_t rows, int64_t dim, const Tensor& mean, const Tensor& var,
                 const Tensor& std, const Tensor& count, int64_t until, const OptT& moments_out, bool reduce_only) {
  TORCH_CHECK(count.scalar_type() == torch::kInt64, "norm_update: count must be int64");
  check_f32(mean, "mean");
  check_f32(var, "var");
  check_f32(std, "std");
  rlb::NormUpdateArgs a{P<const double>(partial), static_cast<int>(chunks), rows, static_cast<int>(dim),
                        P<float>(mean),           P<float>(var),            P<float>(std),
                        reinterpret_cast<long long*>(count.data_ptr()), until, P<double>(moments_out),
                        reduce_only ? 1 : 0};
  TORCH_CHECK(!reduce_only || a.moments_out, "norm_update: reduce_only needs moments_out");
  ok(rlb::norm_update(a, cur()), "norm_update");
}

void counter_add(const Tensor& p, int64_t delta) {
  TORCH_CHECK(p.is_cuda() && p.element_size() == 4, "counter_add: 32-bit counter");
  ok(rlb::counter_add(reinterpret_cast<unsigned int*>(p.data_ptr()), static_cast<unsigned int>(delta), cur()),
     "counter_add");
}

void to_bf16_padded(const Tensor& src, const Tensor& dst, int64_t ld) {
  check_f32(src, "src");
  check_bf16(dst, "dst");
  const int64_t rows = src.size(0), cols = src.numel() / src.size(0);
  TORCH_CHECK(ld >= cols && dst.numel() >= rows * ld, "to_bf16_padded: dst too small");
  ok(rlb::to_bf16_padded(P<const float>(src), static_cast<int>(rows), static_cast<int>(cols), dst.data_ptr(),
                         static_cast<int>(ld), cur()),
     "to_bf16_padded");
}

}  // namespace

void rlb_register_kernels(pybind11::module& m) {
  m.def("prep_obs", &prep_obs);
  m.def("gaussian_sample", &gaussian_sample);
  m.def("process_step", &process_step);
  m.def("gae_blocks", &gae_blocks);
  m.def("gae", &gae);
  m.def("adv_normalize", &adv_normalize);
  m.def("feistel_half_bits", &feistel_half_bits);
  m.def("feistel_permute", &feistel_permute);
  m.def("gather_minibatch", &gather_minibatch);
  m.def("ppo_loss_blocks", &ppo_loss_blocks);
  m.def("ppo_loss", &ppo_loss);
  m.def("make_reduce_plan", &make_reduce_plan);
  m.def("reduce_segments", &reduce_segments);
  m.def("mse_blocks", &mse_blocks);
  m.def("adv_gather_blocks", &adv_gather_blocks);
  m.def("lg_env_step", &lg_env_step);
  m.def("adv_gather_stats", &adv_gather_stats);
  m.def("debug_bounds_enabled", &rlb::debug_bounds_enabled,
        "whether the kernels were built with RL_DEBUG_BOUNDS (indices read from memory are checked)");
  m.def("mse_grad", &mse_grad);
  m.def("rnd_intrinsic", &rnd_intrinsic);
  m.def("rnd_reward_scale", &rnd_reward_scale);
  m.def("make_adam_plan", &make_adam_plan);
  m.def("adam_grid", &adam_grid);
  m.def("adam_step", &adam_step);
  m.def("colstats_chunks", &colstats_chunks);
  m.def("colstats", &colstats);
  m.def("norm_update", &norm_update);
  m.def("counter_add", &counter_add);
  m.def("to_bf16_padded", &to_bf16_padded);
}
