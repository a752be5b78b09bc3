// Shared device helpers for the ptcg_b200 kernels (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <math.h>

typedef __nv_bfloat16 bf16;

#define PTCG_DEV __device__ __forceinline__

template <typename T> PTCG_DEV float to_f(T v);
template <> PTCG_DEV float to_f<float>(float v) { return v; }
template <> PTCG_DEV float to_f<bf16>(bf16 v) { return __bfloat162float(v); }
template <typename T> PTCG_DEV T from_f(float v);
template <> PTCG_DEV float from_f<float>(float v) { return v; }
template <> PTCG_DEV bf16 from_f<bf16>(float v) { return __float2bfloat16_rn(v); }

// exact (erf) GELU, torch nn.GELU() default
PTCG_DEV float gelu_f(float x) {
    return 0.5f * x * (1.f + erff(x * 0.70710678118654752f));
}
PTCG_DEV float gelu_grad_f(float x) {
    float cdf = 0.5f * (1.f + erff(x * 0.70710678118654752f));
    float pdf = 0.3989422804014327f * expf(-0.5f * x * x);
    return cdf + x * pdf;
}
// Fast GELU / GELU' for the tensor-core epilogues.  erf by Abramowitz &
// Stegun, Handbook of Mathematical Functions, eq. 7.1.26 (Hastings):
//   erf(a) = 1 - t (a1 + t (a2 + t (a3 + t (a4 + t a5)))) exp(-a^2),
//   t = 1 / (1 + p a), a >= 0, |error| <= 1.5e-7,
// one branch-free path; exp(-x^2/2) is shared with the normal pdf that
// GELU' needs.  The exact-fp32 (SIMT) path keeps erff.
PTCG_DEV void gelu_parts_fast(float x, float& cdf, float& pdf) {
    const float p = 0.3275911f, a1 = 0.254829592f, a2 = -0.284496736f,
                a3 = 1.421413741f, a4 = -1.453152027f, a5 = 1.061405429f;
    float u = x * 0.70710678118654752f;
    float a = fabsf(u);
    float t = __fdividef(1.f, fmaf(p, a, 1.f));
    float poly = t * fmaf(t, fmaf(t, fmaf(t, fmaf(t, a5, a4), a3), a2), a1);
    float e = __expf(-a * a);                                // exp(-x^2 / 2)
    float erf_a = 1.f - poly * e;
    float erf_u = copysignf(erf_a, u);
    cdf = 0.5f * (1.f + erf_u);
    pdf = 0.3989422804014327f * e;
}
PTCG_DEV float gelu_fast(float x) {
    float c, p;
    gelu_parts_fast(x, c, p);
    return x * c;
}
PTCG_DEV float gelu_grad_fast(float x) {
    float c, p;
    gelu_parts_fast(x, c, p);
    return fmaf(x, p, c);
}
// torch F.softplus (beta 1, threshold 20)
PTCG_DEV float softplus_f(float x) { return x > 20.f ? x : log1pf(expf(x)); }
PTCG_DEV float sigmoid_f(float x) { return 1.f / (1.f + expf(-x)); }

PTCG_DEV float warp_sum(float v) {
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
PTCG_DEV float warp_max(float v) {
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// id stored as float in the obs row -> int with C truncation, then clamp
PTCG_DEV int id_clamp(float v, int hi_excl) {
    int i = (int)v;
    return i < 0 ? 0 : (i >= hi_excl ? hi_excl - 1 : i);
}

static inline unsigned cdiv(long a, long b) { return (unsigned)((a + b - 1) / b); }
