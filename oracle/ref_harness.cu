// TEST INFRASTRUCTURE ONLY -- never part of the product path.
//
// C entry points around the reference's own CUDA code for the parts of the
// path whose CPU oracle restates a reference kernel that no torch code
// implements: the PPO loss (ppo_loss_fwd_bwd, native/src/pufferlib.cu:
// 1368-1449, with ppo_var_mean / ppo_loss_compute / ppo_loss_reduce), the
// rollout sampler (sample_logits, pufferlib.cu:584-718) and the negamax
// advantage (ptcg_puff_advantage, native/model/ptcg_model2.cu:288-321).
//
// This file holds no reference code: it includes the reference's
// pufferlib.cu from the checkout named at build time (build_ref.py), and
// compiles into oracle/_ref/libptcg_ref.so, which the GPU pin tests load
// (tests/test_gpu_ref_pin.py) to check the CPU oracle and this library's
// kernels against the reference's kernels on the same inputs.
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include <unistd.h>

#include "pufferlib.cu"

static PrecisionTensor pt(void* p, long a, long b = 0, long c = 0) {
    PrecisionTensor t{};
    t.data = (precision_t*)p;
    t.shape[0] = a; t.shape[1] = b; t.shape[2] = c;
    return t;
}

static FloatTensor ft(void* p, long a, long b = 0, long c = 0) {
    FloatTensor t{};
    t.data = (float*)p;
    t.shape[0] = a; t.shape[1] = b; t.shape[2] = c;
    return t;
}

// one curand_uniform per state from a copy: the draw sample_logits makes
// for its single action head
__global__ void k_harness_draw(const curandStatePhilox4_32_10_t* states, float* u, int n) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        curandStatePhilox4_32_10_t s = states[i];
        u[i] = curand_uniform(&s);
    }
}

extern "C" {

long ref_rng_state_bytes(void) { return (long)sizeof(curandStatePhilox4_32_10_t); }

int ref_rng_init(void* states, unsigned long long seed, int n, void* stream) {
    rng_init<<<grid_size(n), BLOCK_SIZE, 0, (cudaStream_t)stream>>>(
        (curandStatePhilox4_32_10_t*)states, seed, n);
    return (int)cudaGetLastError();
}

int ref_draw_uniforms(const void* states, float* u, int n, void* stream) {
    k_harness_draw<<<grid_size(n), BLOCK_SIZE, 0, (cudaStream_t)stream>>>(
        (const curandStatePhilox4_32_10_t*)states, u, n);
    return (int)cudaGetLastError();
}

// dec (n x (nopt+1)) fused [logits | value]; act_size: device int[1] = nopt
int ref_sample_logits(float* dec, int n, int nopt, const float* mask, int mask_stride,
                      int* act_size, float* actions, float* logprobs, float* values,
                      void* states, void* stream) {
    PrecisionTensor dec_out = pt(dec, n, nopt + 1);
    PrecisionTensor logstd{};
    IntTensor sizes{};
    sizes.data = act_size;
    sizes.shape[0] = 1;
    sample_logits<<<grid_size(n), BLOCK_SIZE, 0, (cudaStream_t)stream>>>(
        dec_out, logstd, sizes, actions, logprobs, values,
        (curandStatePhilox4_32_10_t*)states, mask, mask_stride, nullptr, 0);
    return (int)cudaGetLastError();
}

// PPO loss over (N segments, T steps): dec (N, T, nopt+1); per-row tensors
// (N, T); prio (N); mask (N, T, nopt).  ent_coef and act_size are device
// scalars; scratch holds 4 floats.  losses[8] accumulates {pg, vf, ent,
// total, old_approx_kl, approx_kl, clipfrac, count}; loss_out[1] the total.
int ref_ppo_loss(float* dec, int N, int T, int nopt, float* actions, float* old_logp,
                 float* advantages, float* values, float* returns, float* prio, float* mask,
                 float clip, float vf_clip, float vf_coef, const float* ent_coef_dev,
                 int* act_size, float* grad_logits, float* grad_values, float* ratio,
                 float* newvalue, float* losses, float* loss_out, float* scratch,
                 void* stream) {
    PrecisionTensor d = pt(dec, N, T, nopt + 1);
    PrecisionTensor logstd{};
    TrainGraph g{};
    g.mb_actions = pt(actions, N, T, 1);
    g.mb_logprobs = pt(old_logp, N, T);
    g.mb_advantages = pt(advantages, N, T);
    g.mb_values = pt(values, N, T);
    g.mb_returns = pt(returns, N, T);
    g.mb_ratio = pt(ratio, N, T);
    g.mb_newvalue = pt(newvalue, N, T);
    g.mb_prio = pt(prio, N);
    g.mb_action_mask = pt(mask, N, T, nopt);
    IntTensor sizes{};
    sizes.data = act_size;
    sizes.shape[0] = 1;
    FloatTensor acc = ft(losses, NUM_LOSSES);
    PPOBuffersPuf b{};
    b.loss_output = ft(loss_out, 1);
    b.grad_logits = ft(grad_logits, N, T, nopt);
    b.grad_values = ft(grad_values, N, T, 1);
    b.adv_scratch = ft(scratch, 4);
    ppo_loss_fwd_bwd(d, logstd, g, sizes, acc, nullptr, clip, vf_clip, vf_coef, ent_coef_dev, b,
                     false, (cudaStream_t)stream);
    return (int)cudaGetLastError();
}

// the reference's own export, on the reference default shape (its PT_OBS
// and seat column are compile-time constants): values (B, T), obs (B, T, OBS)
int ref_puff_advantage(float* values, float* rewards, float* dones, float* importance,
                       float* obs, float* advantages, int B, int T, float gamma, float lambda,
                       float rho_clip, float c_clip, void* stream) {
    PrecisionTensor v = pt(values, B, T), r = pt(rewards, B, T), dn = pt(dones, B, T),
                    im = pt(importance, B, T), o = pt(obs, B, T, PT_OBS),
                    a = pt(advantages, B, T);
    ptcg_puff_advantage(&v, &r, &dn, &im, &o, &a, gamma, lambda, rho_clip, c_clip,
                        (cudaStream_t)stream);
    return (int)cudaGetLastError();
}

long ref_obs_size(void) { return PT_OBS; }

}  // extern "C"
