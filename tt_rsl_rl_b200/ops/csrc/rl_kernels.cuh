// Host-visible launchers of the RL kernels (rollout, GAE, minibatch gather, PPO loss, gradient reduction,
// clip + Adam, observation normaliser). All launchers enqueue on `stream` and never synchronise.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace rlb {

constexpr int kMaxObsGroups = 4;

// Concatenate up to four [N, w_g] fp32 observation groups into `store` ([N, ld_store] fp32, may be null) and write the
// normalised bf16 copy `x` ([N, ld_x]); mean/std (length D, may be null = identity) give (v - mean) / (std + eps).
struct PrepObsArgs {
  const float* src[kMaxObsGroups];
  int src_ld[kMaxObsGroups];
  int width[kMaxObsGroups];
  int groups;
  int rows;
  float* store;
  int ld_store;
  void* x;  // bf16
  int ld_x;
  const float* mean;
  const float* std;
  float eps;
};
cudaError_t prep_obs(const PrepObsArgs& a, cudaStream_t s);

// Gaussian head of the rollout: actions = mean + std * N(0, 1) (Philox4x32-10 + Box-Muller), log-probability, and the
// distribution parameters written into the rollout slot. `mean` is the last GEMM output [N, ld_mean]; for the
// heteroscedastic head the raw std columns follow the mean columns (hetero = 1).
struct SampleArgs {
  const float* head;
  int ld_head;
  int rows;
  int A;
  int hetero;
  int log_std;             // std parameterised as log (clamped in log space) instead of scalar
  const float* std_param;  // [A] (non-hetero)
  float std_lo, std_hi, log_std_lo, log_std_hi;
  uint64_t seed;
  uint64_t* counter;        // device call counter: read as the Philox offset, advanced by one per launch
  unsigned int* ticket;     // device scratch (zero-initialised) for the last-block counter update
  float* actions;   // [N, A]
  float* out_mean;  // [N, A]
  float* out_std;   // [N, A]
  float* out_logp;  // [N]
  float* actions_copy;  // optional second destination of the actions (user-visible buffer)
};
cudaError_t gaussian_sample(const SampleArgs& a, cudaStream_t s);

// rewards_slot[n] = rew[n] (+ intrinsic[n]) + gamma * values_slot[n] * timeouts[n]; dones_slot[n] = dones[n] != 0.
struct ProcessArgs {
  const float* rewards;
  const float* intrinsic;  // optional
  const void* dones;       // dtype: 0 float32, 1 bool/uint8, 2 int64
  int dones_dtype;
  const void* timeouts;    // optional, same dtype codes
  int timeouts_dtype;
  const float* values_slot;
  float gamma;
  int rows;
  float* rewards_slot;
  float* dones_slot;
  unsigned int* nonfinite_flag;  // optional: set to 1 if a reward is NaN/Inf
};
cudaError_t process_step(const ProcessArgs& a, cudaStream_t s);

// GAE reverse scan over [T, N] (upstream rsl_rl/algorithms/ppo.py:166-191) and the sums for advantage normalisation.
struct GaeArgs {
  const float* rewards;
  const float* dones;
  const float* values;
  const float* last_values;
  float* returns;
  float* advantages;
  int T, N;
  float gamma, lam;
  double* partial;  // [blocks, 2]: sum, sum of squares of advantages
};
int gae_blocks(int N);
cudaError_t gae(const GaeArgs& a, cudaStream_t s);
// advantages = (adv - mean) / (std_unbiased + 1e-8) over all T*N values; each block re-reduces `partial`.
cudaError_t adv_normalize(float* adv, long long n, const double* partial, int parts, cudaStream_t s);
// Per-minibatch advantages: out[i] = adv[idx[i]] with per-block (sum, sum of squares) partials in fp64, the input of
// adv_normalize (normalize_advantage_per_mini_batch). Returns the partial count through *parts.
int adv_gather_blocks(long long n);
cudaError_t adv_gather_stats(const float* adv, long long n_adv, const int* idx, long long n, float* out,
                             double* partial, unsigned int* status, cudaStream_t s);
// Whether this library was built with -DRL_DEBUG_BOUNDS (indices read from memory are checked before use).
bool debug_bounds_enabled();

constexpr int kGatherModels = 3;
// Minibatch gather: for rows i in [0, B) take storage row idx = perm(offset + i) (Feistel bijection of [0, total) keyed
// by *key_ptr) or idx_in[i]; write idx_out[i] and the normalised bf16 observations of up to two models.
struct GatherArgs {
  int B;               // original minibatch rows (n0)
  long long offset;
  long long total;
  const uint32_t* key_ptr;
  int half_bits;
  const int* idx_in;  // optional explicit permutation slice
  int* idx_out;
  int copies;          // symmetry copies K >= 1: row r of a model is copy r / B of sample r % B
  const float* obs[kGatherModels];
  int obs_ld[kGatherModels];
  int dim[kGatherModels];
  int rows[kGatherModels];          // rows written for each model: B or K * B
  const float* mean[kGatherModels];
  const float* std[kGatherModels];
  const int* perm[kGatherModels];   // [K, dim] source column of each output column per copy (null: identity)
  const float* sign[kGatherModels]; // [K, dim]
  int vec4[kGatherModels];          // 1: obs rows 16-byte aligned with a pitch that is a multiple of 4 floats
  float eps;
  void* x[kGatherModels];  // bf16
  int ld_x[kGatherModels];
  int models;
  unsigned int* status;
};
cudaError_t gather_minibatch(const GatherArgs& a, cudaStream_t s);
uint32_t feistel_half_bits(long long total);
uint32_t feistel_permute_host(uint32_t i, uint32_t n, uint32_t half_bits, uint32_t key);

// PPO loss terms and gradients with respect to the model outputs (upstream ppo.py:241-294), with per-block partial
// sums (deterministic) for the loss statistics, bias gradients of both heads and the std-parameter gradient.
struct PpoLossArgs {
  int B;       // actor rows = copies * n0
  int n0;      // original samples of the minibatch
  int copies;  // symmetry copies (1: none)
  int aug;     // 1: surrogate/value terms over all B rows (data augmentation); 0: rows < n0 only
  const int* act_perm;    // [copies, A] action column maps (copy 0 identity); null when copies == 1
  const float* act_sign;  // [copies, A]
  float mirror_coef;      // gradient weight of the mirror loss (0: statistics only)
  int A;
  int hetero;
  int log_std;
  const float* head;  // actor last-layer output [B, ld_head]
  int ld_head;
  const float* value;  // critic output [rows, ld_value] (rows = B if aug else n0)
  int ld_value;
  const float* std_param;
  float std_lo, std_hi, log_std_lo, log_std_hi;
  const int* idx;  // storage row per original minibatch row
  const float* st_actions;
  const float* st_mean;
  const float* st_std;
  const float* st_logp;
  const float* st_adv;
  const float* st_ret;
  const float* st_val;
  const float* adv_override;  // optional per-minibatch normalised advantages [n0] (normalize_advantage_per_mini_batch)
  float clip, value_coef, entropy_coef;
  int clipped_value;
  void* d_head;  // bf16 [B, ld_dhead]
  int ld_dhead;
  void* d_value;  // bf16 [rows, ld_dvalue]
  int ld_dvalue;
  float* stats_partial;   // [blocks, kLossStats]: surrogate, value, entropy, kl, symmetry (each a mean)
  float* dhead_colsum;    // [blocks, head_cols]
  float* dvalue_colsum;   // [blocks, 1]
  float* dstd_partial;    // [blocks, A] (non-hetero)
  long long total;        // storage rows (bound of idx in builds with RL_DEBUG_BOUNDS)
  unsigned int* status;   // optional status word (index errors of builds with RL_DEBUG_BOUNDS)
};
constexpr int kLossStats = 5;
int ppo_loss_blocks(int B);
cudaError_t ppo_loss(const PpoLossArgs& a, cudaStream_t s);

// Sum of split / per-block partial buffers into the flat gradient vector. One launch covers every segment.
// The destination vector is send[(*epoch + 1) & 1]: the data-parallel send buffers alternate by exchange parity so a
// rank never overwrites gradients a slower peer may still be reading.
struct ReduceSegment {
  const float* src;     // [parts, n]
  long long dst_offset; // into the flat gradient vector
  long long n;
  int parts;
  int first_chunk;      // prefix of chunk counts
};
cudaError_t reduce_segments(const ReduceSegment* segs_dev, int nseg, int total_chunks, float* send0, float* send1,
                            const unsigned int* epoch, int accumulate, cudaStream_t s);

// Behaviour-cloning loss (distillation), ``mse`` or ``huber`` (delta 1) averaged over rows x A. Writes the bf16
// gradient of the mean loss into grad [rows, ld_grad] (columns A .. ld_grad zero), per-block column sums of that
// gradient over head_cols columns (the output-layer bias gradient; columns >= A are zero) and adds the loss to
// *loss_acc (per-block partials summed by the last block in a fixed order, so the value is deterministic).
struct MseArgs {
  const float* pred;
  int ld_pred;
  const float* target;
  int ld_target;
  int rows, A;
  int huber;
  void* grad;
  int ld_grad;
  int head_cols;
  float* loss_partial;    // [blocks]
  float* colsum_partial;  // [blocks, head_cols]
  float* loss_acc;        // [1], accumulated
  unsigned int* ticket;   // [1], zero between launches
  // optional [1] on the device: the last row stands for this many identical rows (its loss and gradient are scaled
  // by it and the mean is over rows - 1 + weight rows); used for the zero-padded trajectory entries of recurrent
  // minibatches, which all share one input row
  const float* last_weight;
  // > 0: the mean is over this many rows instead (a window of several steps of denom_rows rows each, every step's
  // loss a mean of its own: the gradient of the sum of the step means)
  int denom_rows;
};
int mse_blocks(int rows);

// RND intrinsic reward: out[i] = weight[step] * || target[i] - pred[i] ||_2 over dim columns. With reward
// normalisation (disc != null) the kernel writes the unweighted distance and advances the per-environment discounted
// sum disc[i] = gamma * disc[i] + out[i]; rnd_reward_scale then applies out[i] = weight * out[i] / std once the running
// std of that sum has been updated (rsl_rl/modules/normalization.py EmpiricalDiscountedVariationNormalization).
cudaError_t rnd_intrinsic(const float* target, int ld_target, const float* pred, int ld_pred, int rows, int dim,
                          const float* weight, float* out, float* disc, float gamma, cudaStream_t s);
cudaError_t rnd_reward_scale(float* out, int rows, const float* weight, const float* std, cudaStream_t s);
cudaError_t mse_grad(const MseArgs& a, cudaStream_t s);
constexpr int kReduceChunk = 32;  // columns per block of the reduction kernel

// Fused (all-reduce over peers) + per-group global-norm clip + adaptive learning rate + Adam + bf16 weight shadows.
struct AdamTensor {
  long long offset;  // into the flat vectors
  long long numel;
  int group;
  int rows, cols;    // logical 2-D shape of weights (cols = fan-in) for the bf16 shadow
  void* shadow;      // bf16 [rows, shadow_ld] or null
  int shadow_ld;
  unsigned int cols_magic, cols_shift;  // idx / cols == umulhi(idx, cols_magic) >> cols_shift (shift 32: cols == 1)
};
struct AdamChunk {
  int tensor;
  int start;
  int count;
};
constexpr int kAdamMaxGroups = 4;
constexpr int kAdamChunk = 2048;
struct AdamArgs {
  float* params;
  float* send[2];      // this rank's gradient send buffers (parity (*epoch + 1) & 1 holds this step's gradients)
  float* grads;        // local output: rank-averaged gradients (before clipping)
  float* exp_avg;
  float* exp_avg_sq;
  const AdamTensor* tensors;
  const AdamChunk* chunks;
  int nchunks;
  int ngroups;
  long long group_begin[kAdamMaxGroups], group_end[kAdamMaxGroups];  // contiguous flat range of each clip group
  long long exchange_len;  // floats exchanged (multiple of 4, buffers 16-byte aligned): parameters + statistics
  float max_norm[kAdamMaxGroups];   // <= 0: no clipping
  float beta1[kAdamMaxGroups], beta2[kAdamMaxGroups], eps[kAdamMaxGroups];
  int lr_index[kAdamMaxGroups];     // learning-rate slot of each group (groups of one torch optimizer share slot 0)
  float* lr;                        // [ngroups] device learning-rate slots (slot 0 adapted by the KL rule)
  float* lr_out_slot;               // optional: learning rate after this step written here as well
  long long* step;                  // [ngroups] device step counters
  // adaptive KL schedule (group 0)
  int adaptive;
  const float* kl_mean;             // device scalar: mean KL of this minibatch (rank-averaged in the exchange)
  float desired_kl, lr_min, lr_max;
  // data-parallel exchange (world > 1): gradients of every rank read through peer pointers in rank order
  int world, rank;
  float* const* peer_send;          // [2 * world] device pointers: peer_send[parity * world + r]
  unsigned int* const* peer_flags;  // [world] flag arrays of every rank (each [world] uint32)
  unsigned int* epoch;              // device exchange counter (incremented by this kernel)
  uint64_t timeout_ns;
  // two-shot exchange (world >= 2 with peer_reduced): rank r averages float4 elements [r S4, (r + 1) S4) of the
  // exchanged vector over all ranks into its `reduced` buffer (followed by kAdamMaxGroups squared-norm slots), then
  // every rank reads each element's average from its owner. Flags carry 2 e (gradients sent) and 2 e + 1 (shard
  // averaged) for exchange e. Null peer_reduced: one-shot (every rank sums every element over all ranks).
  float* const* peer_reduced;       // [world] device pointers of every rank's reduced buffer (exchange_len + 8 floats)
  long long shard4;                 // S4: float4 elements per shard
  long long kl_offset;              // index of the KL statistic in the exchanged vector (two-shot), -1: none
  // scratch
  float* norm_partial;              // [gridDim, ngroups]
  unsigned int* barrier;            // [4] zero-initialised: grid-barrier count, generation, abort epoch, ticket
  unsigned int* status;
  float* out_norms;                 // [ngroups] (optional)
};
int adam_grid(int device);
cudaError_t adam_step(const AdamArgs& a, int grid, cudaStream_t s);

// Column moments of fp32 [rows, ld] (first `dim` columns), fp64 partial sums per row chunk, then the running
// EmpiricalNormalization update (upstream rsl_rl/modules/normalization.py:51-78).
struct ColStatsArgs {
  const float* x;
  long long rows;
  int ld;
  int dim;
  double* partial;  // [chunks, 2, dim]
  int chunks;
};
int colstats_chunks(long long rows);
cudaError_t colstats(const ColStatsArgs& a, cudaStream_t s);
struct NormUpdateArgs {
  const double* partial;  // [chunks, 2, dim]
  int chunks;
  long long rows;         // rows in this batch (summed over ranks if `global_partial`)
  int dim;
  float* mean;            // [dim]
  float* var;
  float* std;
  long long* count;
  long long until;        // <0: no limit
  double* moments_out;    // optional [2 + 2*dim] copy of (n, unused, sum[dim], sumsq[dim]) for cross-rank combine
  int reduce_only;        // 1: only write moments_out (the running statistics are left untouched)
};
cudaError_t norm_update(const NormUpdateArgs& a, cudaStream_t s);

// *p += delta (single thread); used for per-update permutation keys.
cudaError_t counter_add(unsigned int* p, unsigned int delta, cudaStream_t s);

// fp32 [rows, cols] -> bf16 [rows, ld] (zero padding in columns [cols, ld)).
cudaError_t to_bf16_padded(const float* src, int rows, int cols, void* dst, int ld, cudaStream_t s);

}  // namespace rlb
