// Shared device helpers for the ptcg_b200 kernels (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <math.h>

typedef __nv_bfloat16 bf16;

// Build-time configuration of the tensor-core GEMM epilogue.
#ifndef PTCG_EPI_WARPS
#define PTCG_EPI_WARPS 16       // epilogue warps per CTA (multiple of 4)
#endif
#ifndef PTCG_EPI_WARPS_LIGHT
#define PTCG_EPI_WARPS_LIGHT 12 // epilogue warps of the GEMMs without a GELU forward
#endif
#ifndef PTCG_STAGE_BUFS
#define PTCG_STAGE_BUFS 1       // TMA-store staging buffers per epilogue warp (1 or 2)
#endif
#ifndef PTCG_BIAS_SMEM
#define PTCG_BIAS_SMEM 1        // stage bias vectors in shared memory
#endif
#ifndef PTCG_AUX_TMA
#define PTCG_AUX_TMA 1          // prefetch the saved GELU' operand by TMA
#endif
#ifndef PTCG_EPI_WARPS_AUX
#define PTCG_EPI_WARPS_AUX 12   // epilogue warps of the GELU'-multiply GEMM (FFN2 dX)
#endif
#ifndef PTCG_GEMM_M2
#define PTCG_GEMM_M2 1          // 256-row CTA tiles for the fp32-accumulate (weight-gradient) GEMMs
#endif
#ifndef PTCG_AUX_BN_MAX
#define PTCG_AUX_BN_MAX 256     // widest CTA tile of the GELU'-multiply GEMM
#endif

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
// GELU and GELU' for the tensor-core epilogues (bf16 mode; the exact-fp32
// SIMT path keeps erff): two values at once on the packed f32x2 FP32 path
// (fma/mul/add.rn.f32x2), one exponential per value and no division:
//   pdf(x)   = 2^(-x^2 log2(e) / 2 + log2(1 / sqrt(2 pi)))      (ex2.approx)
//   q(x)     = erfc(|x| / sqrt 2) / 2 = pdf(x) P(min(|x|, 4 sqrt 2))
//   Phi(x)   = 1/2 + sign(x) (1/2 - q(x)),  GELU = x Phi,  GELU' = Phi + x pdf
// P(u) = sqrt(pi / 2) erfcx(u / sqrt 2), a degree-7 polynomial fitted with
// its error weighted by pdf (the error that reaches Phi; fit_gelu.py beside
// this file prints the coefficients, negated so that 1/2 - q is one fma).
// Beyond |x| = 4 sqrt 2, q < 1e-8 and the clamp changes nothing in fp32.
// |Phi error| <= 4e-6, so |GELU error| <= 4e-6 max(|x|, 1) and |GELU'
// error| <= 5e-6 over [-12, 12] (checked against fp64 torch on the device),
// far below the bf16 rounding (2^-9 relative) of the stored activations.
PTCG_DEV unsigned long long pk2(float a, float b) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
PTCG_DEV void upk2(unsigned long long r, float& a, float& b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
PTCG_DEV unsigned long long fma2(unsigned long long a, unsigned long long b, unsigned long long c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
PTCG_DEV unsigned long long mul2(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
PTCG_DEV unsigned long long add2(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
PTCG_DEV float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
PTCG_DEV unsigned long long splat2(float c) { return pk2(c, c); }

// coefficients of -P (fit_gelu.py, degree 7), highest first
#define PTCG_GELU_PN7 4.224045551e-04f
#define PTCG_GELU_PN6 -5.811933428e-03f
#define PTCG_GELU_PN5 3.489678726e-02f
#define PTCG_GELU_PN4 -1.251721382e-01f
#define PTCG_GELU_PN3 3.153921962e-01f
#define PTCG_GELU_PN2 -6.215380430e-01f
#define PTCG_GELU_PN1 9.994421005e-01f
#define PTCG_GELU_PN0 -1.253304124e+00f
#define PTCG_GELU_UMAX 5.656854249f            // 4 sqrt 2
#define PTCG_GELU_S2 -0.72134752044448170f     // -log2(e) / 2
#define PTCG_GELU_S0 -1.3257480647361595f      // log2(1 / sqrt(2 pi))
#ifndef PTCG_GELU_SCALAR
#define PTCG_GELU_SCALAR 0
#endif
#if PTCG_GELU_SCALAR
PTCG_DEV void gelu1(float x, float& y, float& g) {
    const float u = fminf(fabsf(x), PTCG_GELU_UMAX);
    float p = PTCG_GELU_PN7;
    p = fmaf(p, u, PTCG_GELU_PN6);
    p = fmaf(p, u, PTCG_GELU_PN5);
    p = fmaf(p, u, PTCG_GELU_PN4);
    p = fmaf(p, u, PTCG_GELU_PN3);
    p = fmaf(p, u, PTCG_GELU_PN2);
    p = fmaf(p, u, PTCG_GELU_PN1);
    p = fmaf(p, u, PTCG_GELU_PN0);
    const float e = ex2_approx(fmaf(x * x, PTCG_GELU_S2, PTCG_GELU_S0));   // pdf(x)
    const float cdf = 0.5f + copysignf(fmaf(e, p, 0.5f), x);
    g = fmaf(x, e, cdf);
    y = x * cdf;
}
PTCG_DEV void gelu2(float x0, float x1, float& y0, float& y1, float& g0, float& g1) {
    gelu1(x0, y0, g0);
    gelu1(x1, y1, g1);
}
#else
PTCG_DEV void gelu2(float x0, float x1, float& y0, float& y1, float& g0, float& g1) {
    const unsigned long long x = pk2(x0, x1);
    const unsigned long long u = pk2(fminf(fabsf(x0), PTCG_GELU_UMAX), fminf(fabsf(x1), PTCG_GELU_UMAX));
    unsigned long long p = splat2(PTCG_GELU_PN7);
    p = fma2(p, u, splat2(PTCG_GELU_PN6));
    p = fma2(p, u, splat2(PTCG_GELU_PN5));
    p = fma2(p, u, splat2(PTCG_GELU_PN4));
    p = fma2(p, u, splat2(PTCG_GELU_PN3));
    p = fma2(p, u, splat2(PTCG_GELU_PN2));
    p = fma2(p, u, splat2(PTCG_GELU_PN1));
    p = fma2(p, u, splat2(PTCG_GELU_PN0));
    float s0, s1;
    upk2(fma2(mul2(x, x), splat2(PTCG_GELU_S2), splat2(PTCG_GELU_S0)), s0, s1);
    const unsigned long long e = pk2(ex2_approx(s0), ex2_approx(s1));   // pdf(x)
    float h0, h1;
    upk2(fma2(e, p, splat2(0.5f)), h0, h1);                              // 1/2 - q(x)
    const unsigned long long cdf = add2(splat2(0.5f), pk2(copysignf(h0, x0), copysignf(h1, x1)));
    upk2(mul2(x, cdf), y0, y1);
    upk2(fma2(x, e, cdf), g0, g1);
}
#endif
// a0 += b0, a1 += b1 as one packed add
PTCG_DEV void add_pair(float& a0, float& a1, float b0, float b1) {
    upk2(add2(pk2(a0, a1), pk2(b0, b1)), a0, a1);
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

// 16-byte vector helpers for the row-per-warp gather / scatter kernels
PTCG_DEV float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
PTCG_DEV void st4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
PTCG_DEV void st4(bf16* p, float4 v) {
    uint2 q;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&q);
    h[0] = __floats2bfloat162_rn(v.x, v.y);
    h[1] = __floats2bfloat162_rn(v.z, v.w);
    *reinterpret_cast<uint2*>(p) = q;
}
PTCG_DEV float4 add4(float4 a, float4 b) { return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w); }
PTCG_DEV bool nz4(float4 v) { return v.x != 0.f || v.y != 0.f || v.z != 0.f || v.w != 0.f; }
// four fp32 atomic adds in one vector reduction (16-byte aligned target)
PTCG_DEV void red_add4(float* p, float4 v) {
    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};"
                 :: "l"(p), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w) : "memory");
}

// id stored as float in the obs row -> int with C truncation, then clamp
PTCG_DEV int id_clamp(float v, int hi_excl) {
    int i = (int)v;
    return i < 0 ? 0 : (i >= hi_excl ? hi_excl - 1 : i);
}

static inline unsigned cdiv(long a, long b) { return (unsigned)((a + b - 1) / b); }
