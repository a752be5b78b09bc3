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
