// Masked multi-head attention over packed QKV rows, head width 32.
// Semantics: torch F.scaled_dot_product_attention(q, k, v, attn_mask=keep)
// with a boolean key-padding mask (ptcg/rl/model.py:86-89): masked keys get
// -inf, scale 1/sqrt(32).  Probabilities are never materialised in HBM; the
// forward saves the per-row log-sum-exp and the backward recomputes P.
//
// One CTA per (sequence, head); the whole K/V (and Q/dO in backward) of that
// head stays in shared memory (L <= 257 -> <= 142 KB), so neither pass needs
// atomics.  This SIMT version is the exact-fp32 path.
#include "common.cuh"
#include "internal.h"

namespace {

constexpr int DH = 32, PADW = 33, NW = 4;

template <typename T>
__global__ void __launch_bounds__(NW * 32) k_attn_fwd(
        const T* __restrict__ qkv, long ldqkv, const uint8_t* __restrict__ keep,
        T* __restrict__ out, long ldo, float* __restrict__ lse, int L, int H) {
    extern __shared__ float sm[];
    const int nh = blockIdx.x, n = nh / H, h = nh % H;
    const int D = H * DH;
    float* Ks = sm;
    float* Vs = Ks + L * PADW;
    float* qb = Vs + L * PADW;                  // [NW][32]
    float* pb = qb + NW * DH;                   // [NW][Lr]
    const int Lr = (L + 31) & ~31;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const T* base = qkv + (long)n * L * ldqkv;
    for (int i = threadIdx.x; i < L * DH; i += blockDim.x) {
        int l = i / DH, d = i % DH;
        Ks[l * PADW + d] = to_f<T>(base[(long)l * ldqkv + D + h * DH + d]);
        Vs[l * PADW + d] = to_f<T>(base[(long)l * ldqkv + 2 * D + h * DH + d]);
    }
    __syncthreads();
    const float scale = 0.17677669529663687f;   // 1/sqrt(32)
    const uint8_t* kp = keep + (long)n * L;
    float* q = qb + w * DH;
    float* p = pb + w * Lr;
    for (int i = w; i < L; i += NW) {
        q[lane] = to_f<T>(base[(long)i * ldqkv + h * DH + lane]);
        __syncwarp();
        float mx = -INFINITY;
        for (int j = lane; j < L; j += 32) {
            float s = -INFINITY;
            if (kp[j]) {
                float acc = 0.f;
                #pragma unroll
                for (int d = 0; d < DH; d++) acc = fmaf(q[d], Ks[j * PADW + d], acc);
                s = acc * scale;
            }
            p[j] = s;
            mx = fmaxf(mx, s);
        }
        mx = warp_max(mx);
        float sum = 0.f;
        for (int j = lane; j < L; j += 32) {
            float e = p[j] == -INFINITY ? 0.f : expf(p[j] - mx);
            p[j] = e;
            sum += e;
        }
        sum = warp_sum(sum);
        __syncwarp();
        float o = 0.f;
        for (int j = 0; j < L; j++) o = fmaf(p[j], Vs[j * PADW + lane], o);
        out[((long)n * L + i) * ldo + h * DH + lane] = from_f<T>(o / sum);
        if (lane == 0) lse[((long)n * H + h) * L + i] = mx + logf(sum);
        __syncwarp();
    }
}

template <typename T>
__global__ void __launch_bounds__(NW * 32) k_attn_bwd(
        const T* __restrict__ qkv, long ldqkv, const uint8_t* __restrict__ keep,
        const T* __restrict__ out, long ldo, const T* __restrict__ dout, long lddo,
        const float* __restrict__ lse, T* __restrict__ dqkv, long lddqkv,
        float* __restrict__ dbias, int L, int H) {
    extern __shared__ float sm[];
    __shared__ float red[3][NW][32];
    const int nh = blockIdx.x, n = nh / H, h = nh % H;
    const int D = H * DH;
    const int Lr = (L + 31) & ~31;
    float* Qs = sm;
    float* Ks = Qs + L * PADW;
    float* Vs = Ks + L * PADW;
    float* Gs = Vs + L * PADW;                  // dO
    float* ls = Gs + L * PADW;                  // lse [L]
    float* dl = ls + Lr;                        // delta [L]
    float* b1 = dl + Lr;                        // [NW][Lr]
    float* b2 = b1 + NW * Lr;                   // [NW][Lr]
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const T* base = qkv + (long)n * L * ldqkv;
    for (int i = threadIdx.x; i < L * DH; i += blockDim.x) {
        int l = i / DH, d = i % DH;
        Qs[l * PADW + d] = to_f<T>(base[(long)l * ldqkv + h * DH + d]);
        Ks[l * PADW + d] = to_f<T>(base[(long)l * ldqkv + D + h * DH + d]);
        Vs[l * PADW + d] = to_f<T>(base[(long)l * ldqkv + 2 * D + h * DH + d]);
        Gs[l * PADW + d] = to_f<T>(dout[((long)n * L + l) * lddo + h * DH + d]);
    }
    for (int i = threadIdx.x; i < L; i += blockDim.x)
        ls[i] = lse[((long)n * H + h) * L + i];
    __syncthreads();
    // delta_i = dO_i . O_i
    for (int i = w; i < L; i += NW) {
        float v = Gs[i * PADW + lane] * to_f<T>(out[((long)n * L + i) * ldo + h * DH + lane]);
        v = warp_sum(v);
        if (lane == 0) dl[i] = v;
    }
    __syncthreads();
    const float scale = 0.17677669529663687f;
    const uint8_t* kp = keep + (long)n * L;
    float* bufA = b1 + w * Lr;
    float* bufB = b2 + w * Lr;
    T* dbase = dqkv + (long)n * L * lddqkv;
    float cq = 0.f, ck = 0.f, cv = 0.f;      // fp32 column sums for the bias grad
    // pass 1: dQ, one warp per query row
    for (int i = w; i < L; i += NW) {
        for (int j = lane; j < L; j += 32) {
            float ds = 0.f;
            if (kp[j]) {
                float s = 0.f, dp = 0.f;
                #pragma unroll
                for (int d = 0; d < DH; d++) {
                    s = fmaf(Qs[i * PADW + d], Ks[j * PADW + d], s);
                    dp = fmaf(Gs[i * PADW + d], Vs[j * PADW + d], dp);
                }
                float pr = expf(s * scale - ls[i]);
                ds = pr * (dp - dl[i]);
            }
            bufA[j] = ds;
        }
        __syncwarp();
        float dq = 0.f;
        for (int j = 0; j < L; j++) dq = fmaf(bufA[j], Ks[j * PADW + lane], dq);
        dbase[(long)i * lddqkv + h * DH + lane] = from_f<T>(dq * scale);
        cq += dq * scale;
        __syncwarp();
    }
    // pass 2: dK, dV, one warp per key row
    for (int j = w; j < L; j += NW) {
        float dk = 0.f, dv = 0.f;
        if (kp[j]) {
            for (int i = lane; i < L; i += 32) {
                float s = 0.f, dp = 0.f;
                #pragma unroll
                for (int d = 0; d < DH; d++) {
                    s = fmaf(Qs[i * PADW + d], Ks[j * PADW + d], s);
                    dp = fmaf(Gs[i * PADW + d], Vs[j * PADW + d], dp);
                }
                float pr = expf(s * scale - ls[i]);
                bufA[i] = pr;
                bufB[i] = pr * (dp - dl[i]);
            }
            __syncwarp();
            for (int i = 0; i < L; i++) {
                dv = fmaf(bufA[i], Gs[i * PADW + lane], dv);
                dk = fmaf(bufB[i], Qs[i * PADW + lane], dk);
            }
            __syncwarp();
        }
        dbase[(long)j * lddqkv + D + h * DH + lane] = from_f<T>(dk * scale);
        dbase[(long)j * lddqkv + 2 * D + h * DH + lane] = from_f<T>(dv);
        ck += dk * scale;
        cv += dv;
    }
    if (dbias) {
        red[0][w][lane] = cq; red[1][w][lane] = ck; red[2][w][lane] = cv;
        __syncthreads();
        if (w < 3) {
            float t = 0.f;
            for (int k = 0; k < NW; k++) t += red[w][k][lane];
            atomicAdd(&dbias[w * D + h * DH + lane], t);
        }
    }
}

size_t fwd_smem(int L) {
    int Lr = (L + 31) & ~31;
    return sizeof(float) * (2 * L * PADW + NW * DH + NW * Lr);
}
size_t bwd_smem(int L) {
    int Lr = (L + 31) & ~31;
    return sizeof(float) * (4 * L * PADW + 2 * Lr + 2 * NW * Lr);
}

template <typename K>
void set_smem(K k, size_t bytes) {
    if (bytes > 48 * 1024)
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

}  // namespace

void attn_fwd(int dtype, const void* qkv, long ldqkv, const uint8_t* keep,
              void* out, long ldo, float* lse, int nseq, int L, int H, cudaStream_t s) {
    if (nseq <= 0) return;
    size_t sm = fwd_smem(L);
    if (dtype == DT_F32) {
        set_smem(k_attn_fwd<float>, sm);
        ++g_ptcg_launches, k_attn_fwd<float><<<nseq * H, NW * 32, sm, s>>>((const float*)qkv, ldqkv, keep,
            (float*)out, ldo, lse, L, H);
    } else {
        set_smem(k_attn_fwd<bf16>, sm);
        ++g_ptcg_launches, k_attn_fwd<bf16><<<nseq * H, NW * 32, sm, s>>>((const bf16*)qkv, ldqkv, keep,
            (bf16*)out, ldo, lse, L, H);
    }
}

void attn_bwd(int dtype, const void* qkv, long ldqkv, const uint8_t* keep,
              const void* out, long ldo, const void* dout, long lddo,
              const float* lse, void* dqkv, long lddqkv, float* dbias, int nseq, int L, int H,
              cudaStream_t s) {
    if (nseq <= 0) return;
    size_t sm = bwd_smem(L);
    if (dtype == DT_F32) {
        set_smem(k_attn_bwd<float>, sm);
        ++g_ptcg_launches, k_attn_bwd<float><<<nseq * H, NW * 32, sm, s>>>((const float*)qkv, ldqkv, keep,
            (const float*)out, ldo, (const float*)dout, lddo, lse, (float*)dqkv, lddqkv, dbias, L, H);
    } else {
        set_smem(k_attn_bwd<bf16>, sm);
        ++g_ptcg_launches, k_attn_bwd<bf16><<<nseq * H, NW * 32, sm, s>>>((const bf16*)qkv, ldqkv, keep,
            (const bf16*)out, ldo, (const bf16*)dout, lddo, lse, (bf16*)dqkv, lddqkv, dbias, L, H);
    }
}
