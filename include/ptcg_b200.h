/*
 * ptcg_b200.h -- C-ABI of the B200-native (sm_100a) PTCG policy-learning
 * hot path.  Plain pointers and sizes only; every entry point returns 0 on
 * success and a nonzero PTCG_E* code on failure, with a message retrievable
 * from ptcg_last_error() (the reference aborts with a message to stderr).
 *
 * All device pointers are CUDA global memory on the model's device; `stream`
 * is a cudaStream_t passed as void*.  Nothing in the forward / backward /
 * loss / optimizer entry points allocates device memory or waits on the host
 * once ptcg_reserve() has sized the workspaces (the reference's trainer
 * replays these calls inside CUDA graphs, native/src/pufferlib.cu:771-780).
 *
 * Each declaration names the reference interface it replaces
 * (paths relative to the dipamc/kaggle-ptcg-ai-battle checkout).
 */
#ifndef PTCG_B200_H
#define PTCG_B200_H

#ifdef __cplusplus
extern "C" {
#endif

#define PTCG_B200_ABI_VERSION 1

enum {
    PTCG_OK = 0,
    PTCG_EINVAL = 1,     /* bad argument / shape */
    PTCG_ECUDA = 2,      /* CUDA runtime error */
    PTCG_ESTATE = 3,     /* call out of order (no weights, not reserved...) */
    PTCG_ERANGE = 4,     /* size beyond what was reserved */
    PTCG_ENCCL = 5       /* NCCL unavailable or a collective could not be issued */
};

enum { PTCG_FP32 = 0, PTCG_BF16 = 1 };

/* Flag bits of ptcg_backward's `accumulate` argument. */
enum {
    PTCG_BWD_ACCUMULATE = 1,   /* add into the grad arena instead of zeroing it first */
    PTCG_BWD_PARTIAL = 2       /* more micro-batches of this step follow: the grads are
                                  not final, so the grad hook does not fire */
};

/* Runtime model shape.  Replaces the compile-time PT_D/PT_H/PT_FFN/PT_LAYERS,
 * PT_LTOK, PT_NOPT, PT_NC/PT_NA/PT_NS and the token feature width
 * (native/model/ptcg_model.cu:14-82; native/tools/native_weights.py:24-37).
 * d/heads must give a head width of 32. */
typedef struct PtcgShape {
    int d, heads, ffn, layers;
    int ltok, nopt, tok_f;
    int n_cards, n_attacks, n_skills;
} PtcgShape;

typedef struct PtcgModel PtcgModel;

const char* ptcg_last_error(void);
int ptcg_abi_version(void);

/* ---- layout ------------------------------------------------------------
 * Packed fp32 weight blob order = PT_PARAMS (native/model/ptcg_model.cu:95-126,
 * mirrored by native/tools/native_weights.py:45-91).  cols == 0 for 1-D. */
long ptcg_obs_size(const PtcgShape* s);
/* Compact transfer form of observation rows, for the host -> device copy of
 * every rollout step (the reference copies fp32 rows, native/src/vecenv.h:
 * 310-345).  A packed row holds the fields that carry ids -- token ints,
 * option ints, the option mask, the decision ints and the oracle block's
 * card ids -- as int16, then every other field as fp32, in row order within
 * each part; ptcg_obs_packed_bytes gives its size (a 16-byte multiple; c0:
 * 21,376 bytes against 23,680 for the fp32 row).  ptcg_obs_pack (host)
 * refuses, with PTCG_EINVAL and *bad_index = row * obs_size + column, any id
 * field that is not an integer in [-32768, 32767], so the round trip is
 * exact (a -0.0 id comes back as +0.0); ptcg_obs_unpack (device, packed 16-
 * byte aligned) writes the fp32 rows the model reads. */
long ptcg_obs_packed_bytes(const PtcgShape* s);
int ptcg_obs_pack(const PtcgShape* s, const float* rows, long n, void* packed, long* bad_index);
int ptcg_obs_unpack(const PtcgShape* s, const void* packed, long n, float* rows, void* stream);

/* Column of the acting seat in an observation row: global_f[31]
 * (GlobF.ACTOR_SEAT, ptcg/rl/buffers.py:170; PT_SEAT_COL_M of
 * native/model/ptcg_model2.cu:287). */
long ptcg_seat_column(const PtcgShape* s);
int  ptcg_num_params(const PtcgShape* s);
int  ptcg_param_info(const PtcgShape* s, int i, const char** name, long* rows, long* cols);
long ptcg_param_total(const PtcgShape* s);

/* ---- lifetime ------------------------------------------------------------
 * ptcg_create replaces Encoder.create_weights + reg_params and the params /
 * grads Allocator arenas (native/src/models.cu:35-76, ocean.cu:5-46,
 * native/src/kernels.cu:412-474): it allocates the fp32 master-weight arena
 * (16-byte aligned per tensor, PT_PARAMS order), the mirrored grad arena and
 * the Adam moments on `device`.  precision = PTCG_FP32 (parity mode, SIMT fp32
 * GEMMs) or PTCG_BF16 (tcgen05 bf16 GEMMs, fp32 accumulate). */
int ptcg_create(const PtcgShape* s, int precision, int device, PtcgModel** out);
int ptcg_destroy(PtcgModel* m);

/* Static card/attack/skill tables, host pointers, row-major.  Replaces the
 * pt_tab_* imports from native/ptcg/tables.c (native/model/ptcg_model2.cu:390-419).
 * card_static NCx58, card_attacks NCx4 (int32), card_skills NCx2 (int32),
 * att_static NAx15, card_text NCx128, att_text NAx64, skill_text NSx64. */
int ptcg_set_tables(PtcgModel* m, const float* card_static, const int* card_attacks,
                    const int* card_skills, const float* att_static,
                    const float* card_text, const float* att_text,
                    const float* skill_text);

/* Packed fp32 blob <-> master weights (host pointer, n = ptcg_param_total).
 * Replaces ptcg_load_init_weights_regs (native/model/ptcg_model4.cu:196-233)
 * and the packed save path of native/src/bindings.cu:202-215.  Loading also
 * refreshes the bf16 compute copies and resets nothing else. */
int ptcg_load_weights(PtcgModel* m, const float* packed, long n);
int ptcg_save_weights(PtcgModel* m, float* packed, long n);

/* Files.  Weight files are the packed fp32 blob, exactly
 * (native/src/bindings.cu:202-215 save_weights, :343-367 load_weights, which
 * rejects a size mismatch).  State files, written atomically (tmp, fsync,
 * rename):
 *  - format 0, "PTCGSTA1" (bindings.cu:252-341): header {char magic[8];
 *    long global_step, epoch, n_params} (LP64, 32 bytes), packed weights,
 *    packed momentum.  The momentum slot carries the first-moment arena
 *    (Adam m, or the Muon momentum), so a state file round-trips with the
 *    reference's trainer;
 *  - format 1, "PTCGADM1" (new, for Adam resumes): header {magic; long
 *    global_step, epoch, n_params, adam_step} (40 bytes), packed weights, m, v.
 * ptcg_load_state reads either (by magic), restores weights (and bf16 copies),
 * the moments present in the file and, for PTCGADM1, the Adam step. */
int ptcg_save_weights_file(PtcgModel* m, const char* path);
int ptcg_load_weights_file(PtcgModel* m, const char* path);
int ptcg_save_state(PtcgModel* m, const char* path, long global_step, long epoch, int format);
int ptcg_load_state(PtcgModel* m, const char* path, long* global_step, long* epoch);

/* Size activation workspaces: rollout forward for up to `rollout_rows`
 * observations and train forward/backward for up to `train_rows` rows per
 * call (a minibatch larger than train_rows is processed in micro-batches by
 * ptcg_train_step).  Replaces Encoder.reg_rollout / reg_train
 * (native/model/ptcg_model4.cu:260-266; ptcg_model3.cu:112-210). */
int ptcg_reserve(PtcgModel* m, int rollout_rows, int train_rows);

/* ---- Encoder vtable slots ------------------------------------------------
 * Rollout forward: obs (n x obs_size, fp32, ids stored as floats) ->
 * out (n x (nopt+1)) = [raw option scores | oracle value].
 * Replaces Encoder.forward with train=0 (native/model/ptcg_model4.cu:269-275,
 * ptcg_forward_core native/model/ptcg_model3.cu:246-356). */
int ptcg_forward(PtcgModel* m, const float* obs, int n, float* out, void* stream);

/* Rollout forward with the sampler fused into its output step: writes out as
 * ptcg_forward does and, per row, the action drawn from the masked softmax
 * of the scores with the caller's uniform, its logprob and the value, in the
 * same kernel that assembles out -- bit-identical to ptcg_forward followed
 * by ptcg_sample_logits.  mask NULL takes the opt_mask columns of the obs
 * rows (mask_stride ignored).  Replaces the rollout's decoder forward +
 * sample_logits pair (native/src/pufferlib.cu:860-901, 584-718). */
int ptcg_forward_sample(PtcgModel* m, const float* obs, int n, const float* mask,
                        long mask_stride, const float* uniforms, float* out, float* actions,
                        float* logprobs, float* values, void* stream);

/* Train-path forward (saves activations for ptcg_backward, adds blind-V and
 * the belief aux heads).  Replaces policy_forward_train ->
 * ptcg_forward_core(train=1) (native/src/models.cu:791-797;
 * native/model/ptcg_model3.cu:357-369). */
int ptcg_forward_train(PtcgModel* m, const float* obs, int n, float* out, void* stream);

/* Caller-owned rollout workspace: activation buffers for `rows` rollout
 * rows plus the static-table activations, separate from the model's own
 * (ptcg_reserve).  The reference gives each rollout buffer its own
 * activation set (native/src/pufferlib.cu:2618-2627) and runs the buffers'
 * forwards concurrently on per-buffer streams (:503-509); one workspace per
 * buffer lets forwards on different streams run without sharing anything
 * they write.  Allocates once, at creation. */
typedef struct PtcgWorkspace PtcgWorkspace;
int ptcg_workspace_create(PtcgModel* m, int rows, PtcgWorkspace** out);
int ptcg_workspace_destroy(PtcgWorkspace* ws);
/* ptcg_forward into a caller-owned workspace (n <= its rows). */
int ptcg_forward_ws(PtcgModel* m, PtcgWorkspace* ws, const float* obs, int n, float* out,
                    void* stream);

/* Copy an fp32 parameter arena in this model's layout (PT_PARAMS order,
 * each tensor at a 16-byte-aligned offset, the layout of the reference's
 * Allocator, native/src/kernels.cu:433-466) into the model's master weights
 * and refresh the bf16 compute copies, on `stream`.  For trainers whose own
 * optimizer updates their own copy of the weights (the reference's
 * muon_step on its params arena).  n_floats may stop short of the model's
 * padded arena end. */
int ptcg_import_params(PtcgModel* m, const float* arena, long n_floats, void* stream);

/* Backward of the last ptcg_forward_train: grad (n x (nopt+1)) =
 * [d raw scores | d oracle value]; `returns` (n) feeds the blind-V aux loss
 * (the reference binds it through ptcg_bind_train_graph,
 * native/model/ptcg_model2.cu:323-330).  aux_norm_rows / prize_count give the
 * minibatch-wide normalisers of the aux losses (rows of the whole minibatch;
 * number of MY_UNSEEN tokens in it, <= 0 means "count these rows").
 * accumulate is a set of PTCG_BWD_* bits: without PTCG_BWD_ACCUMULATE the
 * grad arena is zeroed first (native/model/ptcg_model4.cu:15-21), with it the
 * call adds to the arena (micro-batching).  A micro-batched step passes
 * PTCG_BWD_PARTIAL on every call but its last, so that the grad hook
 * (ptcg_set_grad_hook) fires once per step, on final grads.  Replaces
 * Encoder.backward + Decoder.backward (ptcg_model4.cu:10-190, 277-306). */
int ptcg_backward(PtcgModel* m, const float* grad, const float* returns,
                  int aux_norm_rows, float prize_count, int accumulate, void* stream);

/* ---- trainer hooks ----------------------------------------------------------
 * Fused clipped-PPO + clipped value loss + entropy over the masked legal
 * logits, forward and backward in one kernel.  Replaces ppo_var_mean +
 * ppo_loss_compute + ppo_loss_reduce (native/src/pufferlib.cu:1010-1449).
 * dec_out (nt x (nopt+1)) [scores | value], mask (nt x nopt), rows ordered
 * (segment, t) with nt = n_seg*horizon; prio per segment.  Writes
 * grad_dec (nt x (nopt+1)), new_logp/ratio (nt), stats[8] = {total, pg, vf,
 * entropy, old_approx_kl, approx_kl, clipfrac, adv_var} (sums over rows,
 * already divided by nt).  `scratch` is PTCG_PPO_SCRATCH_FLOATS(nt) device
 * floats. */
#define PTCG_PPO_SCRATCH_FLOATS(nt) (16 + 7 * (((nt) + 7) / 8))
int ptcg_ppo_loss(const float* dec_out, int nopt, const float* mask,
                  const float* actions, const float* old_logp,
                  const float* advantages, const float* values,
                  const float* returns, const float* prio, int n_seg, int horizon,
                  float clip_coef, float vf_clip_coef, float vf_coef, float ent_coef,
                  float* grad_dec, float* new_logp, float* ratio, float* stats,
                  float* scratch, void* stream);

/* ptcg_ppo_loss without the `scratch` argument: the same kernels and results,
 * with the scratch held in a fixed device array inside this library.  No
 * counterpart in the reference (its loss keeps scratch in the trainer's
 * PPOBuffersPuf).  For callers that cannot hand the loss a scratch buffer:
 * a trainer whose device memory is carved up once at start-up and may not
 * grow afterwards, or a plugin slot whose signature has no room for one.
 * It allocates nothing, on any call.
 *  - Limit: n_seg * horizon <= PTCG_PPO_NOALLOC_MAX_ROWS rows (the static
 *    array is PTCG_PPO_SCRATCH_FLOATS(PTCG_PPO_NOALLOC_MAX_ROWS) floats,
 *    224 KiB per device); larger minibatches return PTCG_ERANGE.
 *  - Set-up: the first call on each device (with that device current)
 *    looks up the array's device address once and caches it; make that
 *    first call before any stream capture.  The cached address lives for
 *    the process: a cudaDeviceReset (or any teardown of the device's
 *    primary context) after that first call is not supported, since the
 *    library may be loaded again at another address.
 *  - Nothing in the array needs to start at zero: every value the kernels
 *    read is written earlier in the same call.
 *  - One array per device: calls that overlap on the same device (on
 *    different streams or host threads) race on it and must be serialised
 *    by the caller. */
#define PTCG_PPO_NOALLOC_MAX_ROWS 65536
int ptcg_ppo_loss_noalloc(const float* dec_out, int nopt, const float* mask,
                          const float* actions, const float* old_logp,
                          const float* advantages, const float* values,
                          const float* returns, const float* prio, int n_seg, int horizon,
                          float clip_coef, float vf_clip_coef, float vf_coef, float ent_coef,
                          float* grad_dec, float* new_logp, float* ratio, float* stats,
                          void* stream);

/* Global-norm clip + fused mixed-precision Adam over the whole arena
 * (fp32 master weights and moments, bf16 compute copies refreshed in the
 * same pass).  Replaces muon_step (native/src/muon.cu:209-297) with the
 * optimizer BASELINE names: torch.nn.utils.clip_grad_norm_(max_norm) +
 * torch.optim.Adam.  gate (device float or NULL) vetoes the step when it is
 * 0 or when the grad norm is not finite (native/src/pufferlib.cu:1286-1302).
 * stats (device, 2 floats) receives {grad_norm, applied}. */
int ptcg_adam_step(PtcgModel* m, float lr, float beta1, float beta2, float eps,
                   float max_norm, const float* gate, float* stats, void* stream);

/* ---- sharded Adam for data parallelism ----------------------------------
 * The reference reduces the whole gradient arena with one ncclAllReduce and
 * then every rank runs the same optimizer over all of it
 * (native/src/muon.cu:209-214).  These three calls let each rank update
 * only its own shard after a reduce-scatter and all-gather the result:
 *  - ptcg_sumsq: fp64 sum of squares of n device floats x into out[0]
 *    (device double); a rank's shard norm, summed over ranks by the caller;
 *  - ptcg_adam_segments: the Adam update of ptcg_adam_step (same clip,
 *    gate, non-finite veto, step counter and stats) applied to nseg arena
 *    segments, seg a device array of nseg triples {arena offset, offset in
 *    grad_src, length} in floats, with gradients read from grad_src and the
 *    clip taken from the global sum of squares sumsq[0] (device double).  It
 *    does not refresh the bf16 compute copies;
 *  - ptcg_refresh_copies: refresh every bf16 compute copy, and the
 *    static-table activations, from the master weights (after the updated
 *    segments of all ranks are gathered, or after any other write to them). */
int ptcg_sumsq(PtcgModel* m, const float* x, long n, double* out, void* stream);
int ptcg_adam_segments(PtcgModel* m, const float* grad_src, const long* seg, int nseg,
                       const double* sumsq, float lr, float beta1, float beta2, float eps,
                       float max_norm, const float* gate, float* stats, void* stream);
int ptcg_refresh_copies(PtcgModel* m, void* stream);

/* Muon step over the whole arena, the reference trainer's optimizer
 * (muon_step, native/src/muon.cu:209-297, with its local patches):
 *  - clip: g *= min(1, max_norm / (||g|| + 1e-6)) (always applied);
 *  - tensors with two dimensions: nesterov m = mu m + g, g += mu m; g / ||g||;
 *    five Newton-Schulz steps X <- a X + (b G + c G^2) X (G = X X^T, or
 *    X (b G + c G^2) with G = X^T X when rows > cols) with the reference's
 *    coefficient table; w = w (1 - lr wd) - lr sqrt(max(1, rows/cols)) X;
 *  - 1-D tensors: m = mu m + (1 - mu) g, w = w (1 - lr wd_1d) - lr (g + m).
 * The momentum lives in arena 2 (shared with Adam's first moment: use one
 * optimizer per model).  gate (device float or NULL) = 0 skips every state
 * and weight write.  stats (device, 2 floats) = {grad norm, applied}.  The
 * grad arena is overwritten (clipped, then the Nesterov / orthogonalised
 * update), as in the reference. */
int ptcg_muon_step(PtcgModel* m, float lr, float momentum, float weight_decay, float wd_1d,
                   float max_norm, const float* gate, float* stats, void* stream);

/* Prioritised segment replay over (B, T) advantages: w_b = (sum_t |A_bt|)^alpha
 * (0 when not finite), probs = (w + 1e-6) / (sum w + 1e-6), cdf = running sum
 * in index order, idx[i] = first b with cdf[b] >= uniforms[i] (clamped to
 * B - 1), mb_prio[i] = (total_agents * probs[idx[i]])^(-beta).  Replaces
 * prio_replay_cuda (native/src/pufferlib.cu:1451-1591); the n_sel uniforms in
 * [0, 1) come from the caller (the reference draws them from curand Philox).
 * probs and cdf are B-float device scratch (probs is also an output). */
int ptcg_prio_replay(const float* advantages, int B, int T, float alpha, float beta,
                     int total_agents, int n_sel, const float* uniforms, int* idx,
                     float* mb_prio, float* probs, float* cdf, void* stream);

/* Gather the selected segments into the minibatch buffers: rows of the
 * (B, T, ...) rollout arrays at idx -> (n_sel, T, ...); mb_returns = values +
 * advantages of the selected rows.  mask (B, T, nopt) and mb_mask are
 * optional (both NULL).  Replaces select_copy (native/src/pufferlib.cu:1777-1826)
 * for the observation / action / logprob / value / advantage / mask channels
 * (mb_prio comes from ptcg_prio_replay). */
int ptcg_select_copy(const int* idx, int n_sel, int T, long obs_size, int nopt,
                     const float* obs, const float* actions, const float* logprobs,
                     const float* values, const float* advantages, const float* mask,
                     float* mb_obs, float* mb_actions, float* mb_logprobs, float* mb_values,
                     float* mb_advantages, float* mb_returns, float* mb_mask, void* stream);

/* dst row idx[i] <- src row i (rows of row_floats floats): writes the new
 * ratio / value of the trained segments back into the rollout buffers.
 * Replaces index_copy (native/src/pufferlib.cu:2147-2160). */
int ptcg_index_copy(float* dst, const int* idx, const float* src, int n, long row_floats,
                    void* stream);

/* Masked inverse-CDF sampling of the option scores + logprob + value copy.
 * Replaces sample_logits (native/src/pufferlib.cu:584-718); uniforms (n)
 * are supplied by the caller instead of a curand Philox state.  Masked
 * logits are -1e4.  actions are written as float (the trainer's precision_t). */
int ptcg_sample_logits(const float* dec_out, int n, int nopt, const float* mask,
                       long mask_stride, const float* uniforms, float* actions,
                       float* logprobs, float* values, void* stream);

/* Seat-flipping GAE / V-trace over (B, T) rollouts on raw device pointers;
 * seats are read from obs[:, :, seat_col] with rows of obs_size floats.  The
 * computation of the reference's ptcg_puff_advantage
 * (native/model/ptcg_model2.cu:288-321); the export with the reference's
 * own name and PrecisionTensor signature is in ptcg_puffer.h. */
int ptcg_negamax_advantage(const float* values, const float* rewards,
                           const float* dones, const float* importance,
                           const float* obs, long obs_size, int seat_col, int B, int T,
                           float gamma, float lambda, float rho_clip, float c_clip,
                           float* advantages, void* stream);

/* Gradient-bucket hook for data parallelism: called on the host, in backward
 * order, each time the grads in arena floats [offset, offset+count) are final
 * for this step, with the compute stream: during ptcg_train_step's last
 * micro-batch, and during each ptcg_backward call without PTCG_BWD_PARTIAL.
 * The callee typically records an event and starts an all-reduce of that
 * bucket on its own stream.  Replaces the post-backward ncclAllReduce of
 * native/src/muon.cu:212-213. */
typedef void (*ptcg_grad_hook)(void* user, long offset, long count, void* stream);
int ptcg_set_grad_hook(PtcgModel* m, ptcg_grad_hook fn, void* user);

/* One PPO minibatch step: micro-batched forward_train -> PPO loss ->
 * backward (grads accumulated over micro-batches, normalised over the whole
 * minibatch), optional grad hook, then clip + Adam.  Replaces the body of the
 * minibatch loop of train_impl (native/src/pufferlib.cu:1964-2118).
 * obs (nt x obs_size) device; per-row arrays (nt); prio (n_seg).
 * stats (device, 16 floats): [0..7] PPO stats as in ptcg_ppo_loss,
 * [8] grad norm, [9] step applied, [10..12] aux losses (blind, hand, prize).
 * If skip_adam != 0 the optimizer is not run (the caller reduces the grads
 * and calls ptcg_adam_step itself). */
int ptcg_train_step(PtcgModel* m, const float* obs, const float* actions,
                    const float* old_logp, const float* advantages,
                    const float* values, const float* returns, const float* prio,
                    int n_seg, int horizon, float clip_coef, float vf_clip_coef,
                    float vf_coef, float ent_coef, float lr, float beta1,
                    float beta2, float eps, float max_norm, int skip_adam,
                    float* stats, void* stream);

/* ---- arenas (device memory owned by the model) -------------------------------
 * which: 0 = fp32 master params, 1 = fp32 grads, 2 = Adam m, 3 = Adam v.
 * n_floats includes the 16-byte alignment padding; arena offsets of each
 * parameter come from ptcg_param_offset.  The model keeps the static-table
 * activations (card / attack / skill tables through their MLPs) of the
 * current weights between forwards, recomputed by every call that changes
 * the weights; after writing the master weights through this pointer, call
 * ptcg_refresh_copies. */
int ptcg_arena(PtcgModel* m, int which, float** ptr, long* n_floats);
long ptcg_param_offset(PtcgModel* m, int i);
/* Adam step counter (for checkpoint/resume). */
int ptcg_get_step(PtcgModel* m, long* step);
int ptcg_set_step(PtcgModel* m, long step);
/* 64-bit checksum of the master weights (device, written to out[0] as two
 * uint32 halves) for the cross-rank "weights identical" check. */
int ptcg_weights_checksum(PtcgModel* m, unsigned int* out_dev, void* stream);

/* ---- native data-parallel exchange --------------------------------------------
 * The gradient average of data parallelism fused with a sharded Adam, run by
 * the library over NCCL (opened at run time: libnccl.so.2, or the file named
 * by $PTCG_NCCL_LIB).  Replaces the post-backward ncclAllReduce of the grad
 * arena and the optimizer every rank runs over all of it
 * (native/src/muon.cu:209-214).  Once ptcg_dp_init returned on every rank:
 *  - each final gradient span of backward (the spans ptcg_set_grad_hook would
 *    report, which it no longer does) is reduce-scattered (average) on a
 *    library stream while the rest of backward runs: in ptcg_train_step's last
 *    micro-batch and in ptcg_backward without PTCG_BWD_PARTIAL;
 *  - the Adam of ptcg_train_step (skip_adam == 0) and ptcg_adam_step clips
 *    with the global gradient norm (one fp64 all-reduce), updates this rank's
 *    piece of every span, all-gathers the updated master weights and
 *    refreshes the bf16 copies.  Weights stay identical on every rank; the
 *    grad arena keeps this rank's own (unaveraged) gradients, and the Adam
 *    moments are valid on this rank's pieces only.
 * Every rank must make the same calls in the same order (they are
 * collectives).  uid: ptcg_dp_unique_id on one rank (128 bytes), passed to
 * every rank by the caller.  ptcg_dp_init blocks until all `world` ranks
 * joined.  ptcg_dp_weights_agree takes the min and max over ranks of the
 * weight checksum (ptcg_weights_checksum) in one collective (a MAX
 * all-reduce of [v, ~v]) and writes them, in stream order, to minmax_dev
 * (2 device int64): equal when every rank holds the same weights.
 * ptcg_dp_finalize ends the exchange (abort != 0: ncclCommAbort, callable
 * while a peer is gone); ptcg_destroy also ends it. */
int ptcg_dp_unique_id(void* uid_out);
int ptcg_dp_init(PtcgModel* m, const void* uid, int rank, int world);
int ptcg_dp_weights_agree(PtcgModel* m, long long* minmax_dev, void* stream);
int ptcg_dp_finalize(PtcgModel* m, int abort);

/* CUDA-event timing of every launch of one GEMM kernel class (1 = tcgen05
 * tensor-core GEMM, 2 = SIMT GEMM, 3 = both, 0 = off), or of the optimizer
 * kernels of each ptcg_adam_step (4: norm and fused Adam, not the table
 * refresh after them), until the next call; read back total device
 * milliseconds, launch count and algorithmic FLOPs (2*M*N*K per GEMM launch).  The reference's analogue is its cudaEvent phase timing
 * (ProfileT, native/src/pufferlib.cu:59-63, 1851-1953). */
int ptcg_kernel_timer(PtcgModel* m, int mode);
/* Per-launch record of the timed region (mode 3 times every GEMM): for up to
 * max launches, ms[i] and meta[8 i ..] = {M, N, K, a_kmajor, b_kmajor, act,
 * engine (1 tcgen05, 2 SIMT), operand dtype}; returns the count. */
int ptcg_kernel_timer_entries(PtcgModel* m, int max, float* ms, int* meta);
/* Number of CUDA kernels this library has launched in this process. */
long long ptcg_launch_count(void);

/* ---- GEMM engine (exposed for tests and tools) -----------------------------
 * C[M,N] (+)= sum_k A(m,k) B(n,k) in fp32; A(m,k) = a_kmajor ? A[m*lda+k] :
 * A[k*lda+m], likewise B.  operand_dtype PTCG_BF16 or PTCG_FP32.  engine:
 * 0 auto, 1 tcgen05 only (PTCG_EINVAL if the shape is unsupported), 2 SIMT,
 * 3 tcgen05 with fp32 operands read as TF32 (kind::tf32).
 * The reference calls cuBLAS for every GEMM (native/model/ptcg_kernels.cuh:42-108). */
int ptcg_gemm(int M, int N, int K, const void* A, long lda, int a_kmajor, const void* B,
              long ldb, int b_kmajor, int operand_dtype, float* C, long ldc, int accumulate,
              int engine, void* stream);
/* Masked multi-head attention over packed QKV rows ([nseq*L, >=3*H*32], head
 * h of q/k/v at columns h*32, H*32 + h*32, 2*H*32 + h*32), key mask keep
 * [nseq, L] (0 = masked), head width 32, L <= 320.  Forward writes out
 * [nseq*L, >=H*32] and the row log-sum-exp lse [nseq, H, L]; backward writes
 * dqkv in the qkv layout and adds the fp32 column sums of dqkv into dbias
 * (3*H*32 floats, may be NULL).  bf16 runs on tensor cores, fp32 is exact.
 * Replaces the materialised-probability attention of the reference
 * (pt_attn_softmax_fwd/bwd + batched GEMMs, native/model/ptcg_kernels.cuh:223-289,
 * native/model/ptcg_model3.cu:12-95). */
int ptcg_attention_fwd(int operand_dtype, const void* qkv, long ldqkv, const unsigned char* keep,
                       void* out, long ldo, float* lse, int nseq, int L, int H, void* stream);
int ptcg_attention_bwd(int operand_dtype, const void* qkv, long ldqkv, const unsigned char* keep,
                       const void* out, long ldo, const void* dout, long lddo, const float* lse,
                       void* dqkv, long lddqkv, float* dbias, int nseq, int L, int H,
                       void* stream);
/* The GELU and GELU' that the tensor-core GEMM epilogues evaluate (the
 * normal tail erfc(|x|/sqrt 2)/2 as the normal pdf times a degree-7
 * polynomial in |x|, fitted for this library with its error weighted by the
 * pdf; |error| <= 5e-6), exposed so tests can bound their error against the
 * exact erf form of torch nn.GELU. */
int ptcg_eval_gelu(const float* x, float* gelu, float* gelu_grad, int n, void* stream);
/* tcgen05 GEMM role counters (clock cycles, summed over CTAs): {producer
 * waiting for free ring slots, MMA waiting for loaded slots, MMA waiting for
 * a free accumulator, epilogue waiting for a finished accumulator, epilogue
 * working, CTA lifetime, tiles, launches, epilogue TMEM loads, epilogue math,
 * epilogue store path} (12 counters).  Reads (if counters != NULL) and
 * resets them, then enables (1) or disables (0) collection. */
int ptcg_tc_profile(int enable, unsigned long long* counters);
/* ptcg_gemm with the fused epilogue of the model's GEMMs: output dtype
 * (PTCG_FP32 / PTCG_BF16), bias[N], act 1 = GELU (out2 <- GELU'(pre), may be
 * NULL), act 2 = multiply by aux (the saved GELU'), colsum[N] += fp32 column
 * sums (may be NULL).  aux / out2 use the output dtype. */
int ptcg_gemm_ex(int M, int N, int K, const void* A, long lda, int a_kmajor, const void* B,
                 long ldb, int b_kmajor, int operand_dtype, void* C, long ldc, int out_dtype,
                 const float* bias, int act, const void* aux, long ld_aux, void* out2, long ldo2,
                 float* colsum, int accumulate, int engine, void* stream);
/* 1 when the tcgen05 engine is usable on the current device (sm_100). */
int ptcg_tensor_cores(void);
/* First error code a bounded device-side wait recorded since the last call
 * (0 = none; the kernel that timed out returned early; 100 + code for the
 * tcgen05 attention, 200 + code for the fused rollout MLP).  Resets the flag. */
int ptcg_device_error(void);

/* Kernels of the bf16 attention (no counterpart in the reference, whose
 * attention materialises fp32 probabilities, native/model/ptcg_kernels.cuh:
 * 223-289): 0 = mma.sync flash attention for both passes, 1 = tcgen05 / TMEM
 * kernels for both, 2 = tcgen05 / TMEM backward with the mma.sync forward.
 * The tcgen05 backward takes the sequences whose row extent fits one
 * 128-row tile and leaves longer ones to the mma.sync backward.
 * Process-wide; takes effect at the next launch; PTCG_ATTN_TC=<impl> sets
 * it at load. */
int ptcg_set_attention_impl(int impl);
int ptcg_get_attention_impl(void);

/* The rollout forward (ptcg_forward, ptcg_forward_sample, bf16, d_model 256)
 * runs each block's FFN1 -> GELU -> FFN2 (+ bias + residual) as one tcgen05
 * kernel that keeps the hidden activation on chip (on = 1), or as the two
 * GEMMs of the training forward (on = 0, the default: faster here).  The reference runs
 * them as two linear layers around a GELU kernel
 * (native/model/ptcg_model3.cu:36-38).  Process-wide; takes effect at the
 * next launch. */
int ptcg_set_fused_mlp(int on);
int ptcg_kernel_timer_read(PtcgModel* m, double* ms, long* launches, double* flops);
/* Algorithmic HBM bytes of the launches timed since ptcg_kernel_timer(m, mode)
 * (operands read once, outputs written once; diagnostic, no counterpart in
 * the reference). */
int ptcg_kernel_timer_bytes(PtcgModel* m, double* bytes);

#ifdef __cplusplus
}
#endif
#endif /* PTCG_B200_H */
