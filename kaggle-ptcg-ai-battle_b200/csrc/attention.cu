// Masked multi-head attention over packed QKV rows, head width 32.
// Semantics: torch F.scaled_dot_product_attention(q, k, v, attn_mask=keep)
// with a boolean key-padding mask (ptcg/rl/model.py:86-89): masked keys get
// -inf, scale 1/sqrt(32).  Probabilities are never materialised in HBM; the
// forward saves the per-row log-sum-exp and the backward recomputes P.
//
// One CTA per (sequence, head); the whole K/V (and Q/dO in backward) of that
// head stays in shared memory (L <= 257 -> <= 142 KB), so neither pass needs
// atomics.  This SIMT version is the exact-fp32 path.
#include <algorithm>
#include <cstdlib>

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


// ===================================================================== bf16
// Tensor-core (mma.sync m16n8k16 bf16, fp32 accumulate) flash attention.
// One CTA per (sequence, head); Q/K/V (and dO in backward) of the head are
// staged in shared memory as [Lp][40] bf16 rows (80-byte pitch: conflict-free
// ldmatrix).  Softmax runs in the exp2 domain; key blocks whose 16 keys are
// all masked are skipped (their probabilities are exactly 0).
constexpr int RS = 40;                      // smem row stride (elements)
// exponentials of the max-shifted (<= 0 or -inf) log2-domain scores use the
// ex2.approx instruction directly (ex2_approx, common.cuh); the probabilities
// are rounded to bf16 for the P.V products right after

PTCG_DEV uint32_t s_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
PTCG_DEV void ldsm4(uint32_t (&r)[4], uint32_t a) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(a));
}
PTCG_DEV void ldsm4t(uint32_t (&r)[4], uint32_t a) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(a));
}
PTCG_DEV void mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
                 "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
PTCG_DEV uint32_t pack2(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *(uint32_t*)&v;
}
// A fragment of the 16x16 block at (r0, c0) of a row-major [rows][RS] tile
PTCG_DEV void lda(uint32_t (&a)[4], const bf16* X, int r0, int c0, int lane) {
    int mi = lane >> 3;
    ldsm4(a, s_addr(X + (r0 + (mi & 1) * 8 + (lane & 7)) * RS + c0 + (mi >> 1) * 8));
}
// B fragments (b[0],b[1] for n-tile 0; b[2],b[3] for n-tile 1) of B[k][n] =
// X[n][k]: 16 n-rows starting n0, 16 k-cols starting k0
PTCG_DEV void ldb_nk(uint32_t (&b)[4], const bf16* X, int n0, int k0, int lane) {
    int mi = lane >> 3;
    ldsm4(b, s_addr(X + (n0 + (mi >> 1) * 8 + (lane & 7)) * RS + k0 + (mi & 1) * 8));
}
// B fragments of B[k][n] = X[k][n]: 16 k-rows from k0, 16 n-cols from n0
PTCG_DEV void ldb_kn(uint32_t (&b)[4], const bf16* X, int k0, int n0, int lane) {
    int mi = lane >> 3;
    ldsm4t(b, s_addr(X + (k0 + (mi & 1) * 8 + (lane & 7)) * RS + n0 + (mi >> 1) * 8));
}

// Rows [0, L) of a 32-wide head slice into smem (zero rows L..Lp) with
// cp.async: every 16-byte piece of every row is in flight at once; the
// caller commits and waits (cp_async_wait_all + __syncthreads).
PTCG_DEV void cp_async16(void* dst, const void* src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;"
                 :: "r"(s_addr(dst)), "l"(src), "r"(src_bytes) : "memory");
}
PTCG_DEV void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
PTCG_DEV void stage_rows(bf16* dst, const bf16* src, long ld, int L, int Lp) {
    for (int i = threadIdx.x; i < Lp * 4; i += blockDim.x) {
        int r = i >> 2, c = (i & 3) * 8;
        bool in = r < L;
        cp_async16(dst + r * RS + c, src + (long)(in ? r : 0) * ld + c, in ? 16 : 0);
    }
}
PTCG_DEV float dot8_bf16(uint4 a, uint4 b) {
    const __nv_bfloat162* x = (const __nv_bfloat162*)&a;
    const __nv_bfloat162* y = (const __nv_bfloat162*)&b;
    float d = 0.f;
    #pragma unroll
    for (int k = 0; k < 4; k++) {
        float2 u = __bfloat1622float2(x[k]), v = __bfloat1622float2(y[k]);
        d = fmaf(u.x, v.x, fmaf(u.y, v.y, d));
    }
    return d;
}

constexpr float LOG2E = 1.4426950408889634f;

__global__ void __launch_bounds__(128) k_attn_fwd_mma(
        const bf16* __restrict__ qkv, long ldqkv, const uint8_t* __restrict__ keep,
        bf16* __restrict__ out, long ldo, float* __restrict__ lse, int L, int H,
        const int* __restrict__ extent) {
    extern __shared__ __align__(16) uint8_t smraw[];
    const int nh = blockIdx.x, n = nh / H, h = nh % H, D = H * DH;
    const int Lp = (L + 15) & ~15, nkb = Lp / 16;
    bf16* Qs = (bf16*)smraw;
    bf16* Ks = Qs + Lp * RS;
    bf16* Vs = Ks + Lp * RS;
    float* kb_bias = (float*)(Vs + Lp * RS);        // [Lp] 0 or -inf (log2 domain)
    int* kb_any = (int*)(kb_bias + Lp);             // [nkb] block has a kept key
    const bf16* base = qkv + (long)n * L * ldqkv + h * DH;
    // rows at or past the extent are neither queries anyone reads nor kept
    // keys: they are zero-filled instead of loaded
    const int ext = extent ? min(extent[n], L) : L;
    stage_rows(Qs, base, ldqkv, ext, Lp);
    stage_rows(Ks, base + D, ldqkv, ext, Lp);
    stage_rows(Vs, base + 2 * D, ldqkv, ext, Lp);
    const uint8_t* kp = keep + (long)n * L;
    for (int i = threadIdx.x; i < nkb; i += blockDim.x) kb_any[i] = 0;
    __syncthreads();
    for (int j = threadIdx.x; j < Lp; j += blockDim.x) {
        bool k = j < L && kp[j];
        kb_bias[j] = k ? 0.f : -INFINITY;
        if (k) kb_any[j >> 4] = 1;
    }
    cp_async_wait_all();
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const float sc = 0.17677669529663687f * LOG2E;
    // query rows at or past the sequence's extent are read by nothing
    // downstream: they get zero output (finite for the row-wise layers
    // after) and a zero log-sum-exp instead of the softmax
    for (int qb = warp; qb < nkb; qb += 4) {
        if (qb * 16 >= ext) {
            bf16* ob = out + (long)n * L * ldo + h * DH;
            for (int i = lane; i < 16 * 4; i += 32) {
                const int r = qb * 16 + (i >> 2);
                if (r < L) *(uint4*)(ob + (long)r * ldo + (i & 3) * 8) = make_uint4(0, 0, 0, 0);
            }
            if (lane < 16 && qb * 16 + lane < L) lse[((long)n * H + h) * L + qb * 16 + lane] = 0.f;
            continue;
        }
        uint32_t qa[2][4];
        lda(qa[0], Qs, qb * 16, 0, lane);
        lda(qa[1], Qs, qb * 16, 16, lane);
        float o[4][4];
        #pragma unroll
        for (int i = 0; i < 4; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
        float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
        // the key blocks with a kept key, two at a time: one max / rescale
        // step per 32 keys (the second slot is empty for an odd count)
        uint32_t rem = __ballot_sync(0xffffffffu, lane < nkb && kb_any[lane]);
        while (rem) {
            const int k0 = __ffs(rem) - 1;
            rem &= rem - 1;
            const bool two = rem != 0;
            const int k1 = two ? __ffs(rem) - 1 : k0;
            if (two) rem &= rem - 1;
            float s[4][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}, {0, 0, 0, 0}, {0, 0, 0, 0}};
            #pragma unroll
            for (int ks = 0; ks < 2; ks++) {
                uint32_t b[4];
                ldb_nk(b, Ks, k0 * 16, ks * 16, lane);
                mma(s[0], qa[ks], b[0], b[1]);
                mma(s[1], qa[ks], b[2], b[3]);
                if (two) {
                    ldb_nk(b, Ks, k1 * 16, ks * 16, lane);
                    mma(s[2], qa[ks], b[0], b[1]);
                    mma(s[3], qa[ks], b[2], b[3]);
                }
            }
            float bm0 = -INFINITY, bm1 = -INFINITY;
            #pragma unroll
            for (int nt = 0; nt < 4; nt++) {
                const int kb = nt < 2 ? k0 : k1;
                float b0 = kb_bias[kb * 16 + (nt & 1) * 8 + 2 * t];
                float b1 = kb_bias[kb * 16 + (nt & 1) * 8 + 2 * t + 1];
                if (nt >= 2 && !two) b0 = b1 = -INFINITY;
                s[nt][0] = s[nt][0] * sc + b0;
                s[nt][1] = s[nt][1] * sc + b1;
                s[nt][2] = s[nt][2] * sc + b0;
                s[nt][3] = s[nt][3] * sc + b1;
                bm0 = fmaxf(bm0, fmaxf(s[nt][0], s[nt][1]));
                bm1 = fmaxf(bm1, fmaxf(s[nt][2], s[nt][3]));
            }
            bm0 = fmaxf(bm0, __shfl_xor_sync(0xffffffffu, bm0, 1));
            bm0 = fmaxf(bm0, __shfl_xor_sync(0xffffffffu, bm0, 2));
            bm1 = fmaxf(bm1, __shfl_xor_sync(0xffffffffu, bm1, 1));
            bm1 = fmaxf(bm1, __shfl_xor_sync(0xffffffffu, bm1, 2));
            float nm0 = fmaxf(m0, bm0), nm1 = fmaxf(m1, bm1);
            // rescale the running sums only when some row's max moved (the
            // factor is exactly 1 otherwise)
            if (__any_sync(0xffffffffu, nm0 != m0 || nm1 != m1)) {
                float c0 = nm0 == -INFINITY ? 1.f : ex2_approx(m0 - nm0);
                float c1 = nm1 == -INFINITY ? 1.f : ex2_approx(m1 - nm1);
                l0 *= c0; l1 *= c1;
                #pragma unroll
                for (int i = 0; i < 4; i++) { o[i][0] *= c0; o[i][1] *= c0; o[i][2] *= c1; o[i][3] *= c1; }
            }
            m0 = nm0; m1 = nm1;
            #pragma unroll
            for (int nt = 0; nt < 4; nt++) {
                s[nt][0] = ex2_approx(s[nt][0] - m0); s[nt][1] = ex2_approx(s[nt][1] - m0);
                s[nt][2] = ex2_approx(s[nt][2] - m1); s[nt][3] = ex2_approx(s[nt][3] - m1);
                l0 += s[nt][0] + s[nt][1];
                l1 += s[nt][2] + s[nt][3];
            }
            #pragma unroll
            for (int j = 0; j < 2; j++) {
                if (j == 1 && !two) break;
                const uint32_t pa[4] = {pack2(s[2 * j][0], s[2 * j][1]), pack2(s[2 * j][2], s[2 * j][3]),
                                        pack2(s[2 * j + 1][0], s[2 * j + 1][1]),
                                        pack2(s[2 * j + 1][2], s[2 * j + 1][3])};
                const int kb = j == 0 ? k0 : k1;
                #pragma unroll
                for (int dn = 0; dn < 2; dn++) {
                    uint32_t b[4];
                    ldb_kn(b, Vs, kb * 16, dn * 16, lane);
                    mma(o[dn * 2], pa, b[0], b[1]);
                    mma(o[dn * 2 + 1], pa, b[2], b[3]);
                }
            }
        }
        l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
        l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
        l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
        l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
        float i0 = 1.f / l0, i1 = 1.f / l1;
        int r0 = qb * 16 + g, r1 = r0 + 8;
        bf16* ob = out + (long)n * L * ldo + h * DH;
        #pragma unroll
        for (int i = 0; i < 4; i++) {
            int c = i * 8 + 2 * t;
            if (r0 < L) *(uint32_t*)(ob + (long)r0 * ldo + c) = pack2(o[i][0] * i0, o[i][1] * i0);
            if (r1 < L) *(uint32_t*)(ob + (long)r1 * ldo + c) = pack2(o[i][2] * i1, o[i][3] * i1);
        }
        if (t == 0) {
            float* lb = lse + ((long)n * H + h) * L;
            if (r0 < L) lb[r0] = (m0 + log2f(l0)) * 0.6931471805599453f;
            if (r1 < L) lb[r1] = (m1 + log2f(l1)) * 0.6931471805599453f;
        }
    }
}

__global__ void __launch_bounds__(128) k_attn_bwd_mma(
        const bf16* __restrict__ qkv, long ldqkv, const uint8_t* __restrict__ keep,
        const bf16* __restrict__ out, long ldo, const bf16* __restrict__ dout, long lddo,
        const float* __restrict__ lse, bf16* __restrict__ dqkv, long lddqkv,
        float* __restrict__ dbias, int L, int H, const int* __restrict__ extent,
        int skip_ext_le) {
    extern __shared__ __align__(16) uint8_t smraw[];
    const int nh = blockIdx.x, n = nh / H, h = nh % H, D = H * DH;
    const int Lp = (L + 15) & ~15, nkb = Lp / 16;
    // rows at or past the extent: masked keys, and queries whose dO is zero
    // (nothing reads them): zero-filled instead of loaded
    const int ext = extent ? min(extent[n], L) : L;
    // sequences the tcgen05 backward took (extent <= skip_ext_le)
    if (ext <= skip_ext_le) return;
    bf16* Qs = (bf16*)smraw;
    bf16* Ks = Qs + Lp * RS;
    bf16* Vs = Ks + Lp * RS;
    bf16* Gs = Vs + Lp * RS;                        // dO
    float* kbias = (float*)(Gs + Lp * RS);          // [Lp] key mask (0 / -inf)
    float* lse2 = kbias + Lp;                       // [Lp] lse (log2 domain), +inf past L
    float* dl = lse2 + Lp;                          // [Lp] delta = dO . O
    int* kany = (int*)(dl + Lp);                    // [nkb]
    int* qany = kany + nkb;                         // [nkb] query block has a nonzero dO row
    float* cs = (float*)(qany + nkb);               // [3][32] bias-grad column sums
    const bf16* base = qkv + (long)n * L * ldqkv + h * DH;
    stage_rows(Qs, base, ldqkv, ext, Lp);
    stage_rows(Ks, base + D, ldqkv, ext, Lp);
    stage_rows(Vs, base + 2 * D, ldqkv, ext, Lp);
    stage_rows(Gs, dout + (long)n * L * lddo + h * DH, lddo, ext, Lp);
    const uint8_t* kp = keep + (long)n * L;
    for (int i = threadIdx.x; i < nkb; i += blockDim.x) kany[i] = qany[i] = 0;
    for (int i = threadIdx.x; i < 96; i += blockDim.x) cs[i] = 0.f;
    __syncthreads();
    const float* lrow = lse + ((long)n * H + h) * L;
    const bf16* orow = out + (long)n * L * ldo + h * DH;
    const bf16* grow = dout + (long)n * L * lddo + h * DH;
    for (int j = threadIdx.x; j < Lp; j += blockDim.x) {
        bool k = j < L && kp[j];
        kbias[j] = k ? 0.f : -INFINITY;
        if (k) kany[j >> 4] = 1;
        lse2[j] = j < L ? lrow[j] * LOG2E : INFINITY;
    }
    // delta_i = dO_i . O_i: four threads per row, 16-byte loads, shuffle sum.
    // A query block whose dO rows are all zero (rows nothing downstream
    // reads, e.g. padding) contributes exactly nothing to dQ, dK or dV
    // (dP = dO V^T = 0 and delta = 0, so dS = 0): qany marks the others.
    for (int i0 = 0; i0 < Lp * 4; i0 += blockDim.x) {
        int i = i0 + threadIdx.x, r = i >> 2, c = (i & 3) * 8;
        float d = 0.f;
        bool nz = false;
        if (r < ext) {
            const uint4 gv = *(const uint4*)(grow + (long)r * lddo + c);
            d = dot8_bf16(*(const uint4*)(orow + (long)r * ldo + c), gv);
            nz = ((gv.x | gv.y | gv.z | gv.w) & 0x7fff7fffu) != 0u;   // +-0 count as zero
        }
        d += __shfl_xor_sync(0xffffffffu, d, 1);
        d += __shfl_xor_sync(0xffffffffu, d, 2);
        if ((i & 3) == 0 && r < Lp) dl[r] = d;
        if (nz) qany[r >> 4] = 1;
    }
    cp_async_wait_all();
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const float sc = 0.17677669529663687f * LOG2E;
    const float scale = 0.17677669529663687f;
    bf16* db = dqkv + (long)n * L * lddqkv + h * DH;
    float colk[8], colv[8], colq[8];
    #pragma unroll
    for (int i = 0; i < 8; i++) colk[i] = colv[i] = colq[i] = 0.f;
    // ---- phase 1: dK, dV, one warp per 16-key block
    for (int kb = warp; kb < nkb; kb += 4) {
        float dk[4][4], dv[4][4];
        #pragma unroll
        for (int i = 0; i < 4; i++)
            #pragma unroll
            for (int j = 0; j < 4; j++) dk[i][j] = dv[i][j] = 0.f;
        if (kany[kb]) {
            uint32_t ka[2][4], va[2][4];
            lda(ka[0], Ks, kb * 16, 0, lane);
            lda(ka[1], Ks, kb * 16, 16, lane);
            lda(va[0], Vs, kb * 16, 0, lane);
            lda(va[1], Vs, kb * 16, 16, lane);
            float kb0 = kbias[kb * 16 + g], kb1 = kbias[kb * 16 + g + 8];
            for (int qb = 0; qb < nkb; qb++) {
                if (!qany[qb]) continue;
                float s[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
                float dp[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
                #pragma unroll
                for (int ks = 0; ks < 2; ks++) {
                    uint32_t b[4];
                    ldb_nk(b, Qs, qb * 16, ks * 16, lane);   // S^T = K Q^T
                    mma(s[0], ka[ks], b[0], b[1]);
                    mma(s[1], ka[ks], b[2], b[3]);
                    ldb_nk(b, Gs, qb * 16, ks * 16, lane);   // dP^T = V dO^T
                    mma(dp[0], va[ks], b[0], b[1]);
                    mma(dp[1], va[ks], b[2], b[3]);
                }
                float p[2][4], ds[2][4];
                #pragma unroll
                for (int nt = 0; nt < 2; nt++) {
                    int q0 = qb * 16 + nt * 8 + 2 * t;
                    float la = lse2[q0], lb = lse2[q0 + 1];
                    float da = dl[q0], dd = dl[q0 + 1];
                    p[nt][0] = ex2_approx(s[nt][0] * sc + kb0 - la);
                    p[nt][1] = ex2_approx(s[nt][1] * sc + kb0 - lb);
                    p[nt][2] = ex2_approx(s[nt][2] * sc + kb1 - la);
                    p[nt][3] = ex2_approx(s[nt][3] * sc + kb1 - lb);
                    ds[nt][0] = p[nt][0] * (dp[nt][0] - da);
                    ds[nt][1] = p[nt][1] * (dp[nt][1] - dd);
                    ds[nt][2] = p[nt][2] * (dp[nt][2] - da);
                    ds[nt][3] = p[nt][3] * (dp[nt][3] - dd);
                }
                uint32_t pa[4] = {pack2(p[0][0], p[0][1]), pack2(p[0][2], p[0][3]),
                                  pack2(p[1][0], p[1][1]), pack2(p[1][2], p[1][3])};
                uint32_t sa[4] = {pack2(ds[0][0], ds[0][1]), pack2(ds[0][2], ds[0][3]),
                                  pack2(ds[1][0], ds[1][1]), pack2(ds[1][2], ds[1][3])};
                #pragma unroll
                for (int dn = 0; dn < 2; dn++) {
                    uint32_t b[4];
                    ldb_kn(b, Gs, qb * 16, dn * 16, lane);   // dV += P^T dO
                    mma(dv[dn * 2], pa, b[0], b[1]);
                    mma(dv[dn * 2 + 1], pa, b[2], b[3]);
                    ldb_kn(b, Qs, qb * 16, dn * 16, lane);   // dK += dS^T Q
                    mma(dk[dn * 2], sa, b[0], b[1]);
                    mma(dk[dn * 2 + 1], sa, b[2], b[3]);
                }
            }
        }
        int r0 = kb * 16 + g, r1 = r0 + 8;
        #pragma unroll
        for (int i = 0; i < 4; i++) {
            int c = i * 8 + 2 * t;
            float k00 = dk[i][0] * scale, k01 = dk[i][1] * scale;
            float k10 = dk[i][2] * scale, k11 = dk[i][3] * scale;
            if (r0 < L) {
                *(uint32_t*)(db + (long)r0 * lddqkv + D + c) = pack2(k00, k01);
                *(uint32_t*)(db + (long)r0 * lddqkv + 2 * D + c) = pack2(dv[i][0], dv[i][1]);
                colk[2 * i] += k00; colk[2 * i + 1] += k01;
                colv[2 * i] += dv[i][0]; colv[2 * i + 1] += dv[i][1];
            }
            if (r1 < L) {
                *(uint32_t*)(db + (long)r1 * lddqkv + D + c) = pack2(k10, k11);
                *(uint32_t*)(db + (long)r1 * lddqkv + 2 * D + c) = pack2(dv[i][2], dv[i][3]);
                colk[2 * i] += k10; colk[2 * i + 1] += k11;
                colv[2 * i] += dv[i][2]; colv[2 * i + 1] += dv[i][3];
            }
        }
    }
    // ---- phase 2: dQ, one warp per 16-query block; warps take the blocks in
    // reverse order so that the warp with an extra key block in phase 1 has
    // one fewer query block here
    for (int qb = 3 - warp; qb < nkb; qb += 4) {
        float dq[4][4];
        #pragma unroll
        for (int i = 0; i < 4; i++) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;
        uint32_t qa[2][4], ga[2][4];
        lda(qa[0], Qs, qb * 16, 0, lane);
        lda(qa[1], Qs, qb * 16, 16, lane);
        lda(ga[0], Gs, qb * 16, 0, lane);
        lda(ga[1], Gs, qb * 16, 16, lane);
        int q0 = qb * 16 + g, q1 = q0 + 8;
        float la = lse2[q0], lb = lse2[q1], da = dl[q0], dd = dl[q1];
        const int nkq = qany[qb] ? nkb : 0;         // all-zero dO rows: dQ = 0
        for (int kb = 0; kb < nkq; kb++) {
            if (!kany[kb]) continue;
            float s[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
            float dp[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
            #pragma unroll
            for (int ks = 0; ks < 2; ks++) {
                uint32_t b[4];
                ldb_nk(b, Ks, kb * 16, ks * 16, lane);       // S = Q K^T
                mma(s[0], qa[ks], b[0], b[1]);
                mma(s[1], qa[ks], b[2], b[3]);
                ldb_nk(b, Vs, kb * 16, ks * 16, lane);       // dP = dO V^T
                mma(dp[0], ga[ks], b[0], b[1]);
                mma(dp[1], ga[ks], b[2], b[3]);
            }
            float ds[2][4];
            #pragma unroll
            for (int nt = 0; nt < 2; nt++) {
                float b0 = kbias[kb * 16 + nt * 8 + 2 * t], b1 = kbias[kb * 16 + nt * 8 + 2 * t + 1];
                float p0 = ex2_approx(s[nt][0] * sc + b0 - la), p1 = ex2_approx(s[nt][1] * sc + b1 - la);
                float p2 = ex2_approx(s[nt][2] * sc + b0 - lb), p3 = ex2_approx(s[nt][3] * sc + b1 - lb);
                ds[nt][0] = p0 * (dp[nt][0] - da);
                ds[nt][1] = p1 * (dp[nt][1] - da);
                ds[nt][2] = p2 * (dp[nt][2] - dd);
                ds[nt][3] = p3 * (dp[nt][3] - dd);
            }
            uint32_t sa[4] = {pack2(ds[0][0], ds[0][1]), pack2(ds[0][2], ds[0][3]),
                              pack2(ds[1][0], ds[1][1]), pack2(ds[1][2], ds[1][3])};
            #pragma unroll
            for (int dn = 0; dn < 2; dn++) {
                uint32_t b[4];
                ldb_kn(b, Ks, kb * 16, dn * 16, lane);       // dQ += dS K
                mma(dq[dn * 2], sa, b[0], b[1]);
                mma(dq[dn * 2 + 1], sa, b[2], b[3]);
            }
        }
        #pragma unroll
        for (int i = 0; i < 4; i++) {
            int c = i * 8 + 2 * t;
            float a0 = dq[i][0] * scale, a1 = dq[i][1] * scale;
            float a2 = dq[i][2] * scale, a3 = dq[i][3] * scale;
            if (q0 < L) {
                *(uint32_t*)(db + (long)q0 * lddqkv + c) = pack2(a0, a1);
                colq[2 * i] += a0; colq[2 * i + 1] += a1;
            }
            if (q1 < L) {
                *(uint32_t*)(db + (long)q1 * lddqkv + c) = pack2(a2, a3);
                colq[2 * i] += a2; colq[2 * i + 1] += a3;
            }
        }
    }
    if (dbias) {
        // thread (g, t) holds columns i*8 + 2t + {0,1}: reduce over g (lanes
        // with equal t), then one shared atomic per column per warp
        #pragma unroll
        for (int i = 0; i < 8; i++) {
            #pragma unroll
            for (int o = 4; o < 32; o <<= 1) {
                colq[i] += __shfl_xor_sync(0xffffffffu, colq[i], o);
                colk[i] += __shfl_xor_sync(0xffffffffu, colk[i], o);
                colv[i] += __shfl_xor_sync(0xffffffffu, colv[i], o);
            }
        }
        if (g == 0) {
            #pragma unroll
            for (int i = 0; i < 4; i++)
                #pragma unroll
                for (int e = 0; e < 2; e++) {
                    int c = i * 8 + 2 * t + e;
                    atomicAdd(&cs[c], colq[2 * i + e]);
                    atomicAdd(&cs[32 + c], colk[2 * i + e]);
                    atomicAdd(&cs[64 + c], colv[2 * i + e]);
                }
        }
        __syncthreads();
        if (threadIdx.x < 96) {
            int w = threadIdx.x / 32, c = threadIdx.x % 32;
            atomicAdd(&dbias[w * D + h * DH + c], cs[threadIdx.x]);
        }
    }
}

size_t fwd_mma_smem(int L) {
    int Lp = (L + 15) & ~15;
    return (size_t)3 * Lp * RS * 2 + Lp * 4 + (Lp / 16) * 4 + 16;
}
size_t bwd_mma_smem(int L) {
    int Lp = (L + 15) & ~15;
    return (size_t)4 * Lp * RS * 2 + 3 * Lp * 4 + 2 * (Lp / 16) * 4 + 96 * 4 + 16;
}

size_t fwd_smem(int L) {
    int Lr = (L + 31) & ~31;
    return sizeof(float) * (2 * L * PADW + NW * DH + NW * Lr);
}
size_t bwd_smem(int L) {
    int Lr = (L + 31) & ~31;
    return sizeof(float) * (4 * L * PADW + 2 * Lr + 2 * NW * Lr);
}

// ============================================================ first row only
// The critic block's output is read at its readout row alone
// (ptcg/rl/model.py:305-308: oracle_v1(cat[x[:, 0], g])), so only query row
// 0 of each sequence needs attention; keys and values still span every row.
// One warp per head.  Lane 4 * rg + c covers key row rg of each group of 8
// consecutive keys and head columns [8c, 8c + 8): one 16-byte access per
// lane reads or writes 8 whole 64-byte head rows of K, V, dK or dV, and a
// dot product over the head takes two shuffles.  (A lane per key made
// every access touch 32 rows 1 KB apart, and the L1 wavefronts, not DRAM,
// bounded the kernels.)  fp32 arithmetic throughout; K and V are streamed
// once.

PTCG_DEV void ld8(const float* p, float* f) {
    float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}
PTCG_DEV void ld8(const bf16* p, float* f) {
    uint4 u = *reinterpret_cast<const uint4*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
    #pragma unroll
    for (int i = 0; i < 4; i++) {
        float2 t = __bfloat1622float2(h[i]);
        f[2 * i] = t.x; f[2 * i + 1] = t.y;
    }
}
PTCG_DEV void st8(float* p, const float* f) {
    reinterpret_cast<float4*>(p)[0] = make_float4(f[0], f[1], f[2], f[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(f[4], f[5], f[6], f[7]);
}
PTCG_DEV void st8(bf16* p, const float* f) {
    uint4 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
    #pragma unroll
    for (int i = 0; i < 4; i++) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    *reinterpret_cast<uint4*>(p) = u;
}

// out[n, :] = softmax(q_n K^T / sqrt(32)) V per head; lse[n, h] natural-log
// log-sum-exp of the scaled scores (-inf when every key is masked).
// q: the query row of sequence n at q + n * ldq; kv: rows [K | V] (2D wide,
// row stride ldkv) of every position, sequence n at rows n * L ..
// One CTA per sequence; shared memory holds each head's scores [H][Lr].
template <typename T>
__global__ void __launch_bounds__(512) k_attn_row0_fwd(
        const T* __restrict__ qrows, long ldq, const T* __restrict__ kv, long ldkv,
        const uint8_t* __restrict__ keep, T* __restrict__ out, long ldo,
        float* __restrict__ lse, int L, int H) {
    extern __shared__ float sm[];
    const int n = blockIdx.x, h = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rg = lane >> 2, c8 = (lane & 3) * 8;
    const int D = H * DH, Lr = (L + 31) & ~31;
    float* p = sm + h * Lr;
    const T* base = kv + (long)n * L * ldkv + h * DH + c8;
    const uint8_t* kp = keep + (long)n * L;
    const float scale = 0.17677669529663687f;   // 1/sqrt(32)
    float q8[8];
    ld8(qrows + (long)n * ldq + h * DH + c8, q8);
    #pragma unroll
    for (int e = 0; e < 8; e++) q8[e] *= scale;
    float mx = -INFINITY;
    for (int j0 = 0; j0 < L; j0 += 8) {
        const int j = j0 + rg;
        const bool live = j < L && kp[j];
        float s = 0.f;
        if (live) {
            float k8[8];
            ld8(base + (long)j * ldkv, k8);
            #pragma unroll
            for (int e = 0; e < 8; e++) s = fmaf(q8[e], k8[e], s);
        }
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        s += __shfl_xor_sync(0xffffffffu, s, 2);
        if (!live) s = -INFINITY;
        if (j < L && (lane & 3) == 0) p[j] = s;
        mx = fmaxf(mx, s);
    }
    mx = warp_max(mx);
    __syncwarp();
    float sum = 0.f;
    for (int j = lane; j < L; j += 32) {
        float e = p[j] == -INFINITY ? 0.f : expf(p[j] - mx);
        p[j] = e;
        sum += e;
    }
    sum = warp_sum(sum);
    __syncwarp();
    float o8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j0 = 0; j0 < L; j0 += 8) {
        const int j = j0 + rg;
        const float pj = j < L ? p[j] : 0.f;
        if (pj != 0.f) {
            float v8[8];
            ld8(base + (long)j * ldkv + D, v8);
            #pragma unroll
            for (int e = 0; e < 8; e++) o8[e] = fmaf(pj, v8[e], o8[e]);
        }
    }
    #pragma unroll
    for (int e = 0; e < 8; e++) {
        #pragma unroll
        for (int o = 4; o < 32; o <<= 1) o8[e] += __shfl_xor_sync(0xffffffffu, o8[e], o);
        o8[e] = sum > 0.f ? o8[e] / sum : 0.f;
    }
    if (rg == 0) st8(out + (long)n * ldo + h * DH + c8, o8);
    if (lane == 0) lse[(long)n * H + h] = sum > 0.f ? mx + logf(sum) : -INFINITY;
}

// Backward of k_attn_row0_fwd: dq (one row per sequence, dq + n * lddq) and
// dK / dV at every key of dkv (rows [dK | dV], zero where masked).  The QKV
// bias gradient (fp32, before rounding) accumulates into dbias[3D] = [q | k |
// v]: per-head partials over the sequences a CTA visits in shared memory
// [H][96], one atomic per column per CTA.
template <typename T>
__global__ void __launch_bounds__(512) k_attn_row0_bwd(
        const T* __restrict__ qv, long ldq, const T* __restrict__ kv, long ldkv,
        const uint8_t* __restrict__ keep, const T* __restrict__ out, long ldo,
        const T* __restrict__ dout, long lddo, const float* __restrict__ lse,
        T* __restrict__ dqo, long lddq, T* __restrict__ dkv, long lddkv,
        float* __restrict__ dbias, int R, int L, int H) {
    extern __shared__ float sm[];
    const int h = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rg = lane >> 2, c8 = (lane & 3) * 8;
    const int D = H * DH;
    float* acc = sm + h * 96;                    // [q | k | v] bias-grad columns of the head
    for (int i = lane; i < 96; i += 32) acc[i] = 0.f;
    __syncwarp();
    const float scale = 0.17677669529663687f;
    for (int n = blockIdx.x; n < R; n += gridDim.x) {
        const T* base = kv + (long)n * L * ldkv + h * DH + c8;
        T* dbase = dkv + (long)n * L * lddkv + h * DH + c8;
        const uint8_t* kp = keep + (long)n * L;
        float q8[8], g8[8], t8[8];
        ld8(qv + (long)n * ldq + h * DH + c8, q8);
        ld8(dout + (long)n * lddo + h * DH + c8, g8);
        ld8(out + (long)n * ldo + h * DH + c8, t8);
        float delta = 0.f;
        #pragma unroll
        for (int e = 0; e < 8; e++) delta = fmaf(g8[e], t8[e], delta);
        delta += __shfl_xor_sync(0xffffffffu, delta, 1);
        delta += __shfl_xor_sync(0xffffffffu, delta, 2);
        const float l = lse[(long)n * H + h];
        float dq8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        float sds = 0.f, sp = 0.f;
        for (int j0 = 0; j0 < L; j0 += 8) {
            const int j = j0 + rg;
            const bool live = j < L && kp[j] && l != -INFINITY;
            float k8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            float s = 0.f, dp = 0.f;
            if (live) {
                float v8[8];
                ld8(base + (long)j * ldkv, k8);
                ld8(base + (long)j * ldkv + D, v8);
                #pragma unroll
                for (int e = 0; e < 8; e++) {
                    s = fmaf(q8[e], k8[e], s);
                    dp = fmaf(g8[e], v8[e], dp);
                }
            }
            s += __shfl_xor_sync(0xffffffffu, s, 1);
            s += __shfl_xor_sync(0xffffffffu, s, 2);
            dp += __shfl_xor_sync(0xffffffffu, dp, 1);
            dp += __shfl_xor_sync(0xffffffffu, dp, 2);
            float pj = 0.f, dsj = 0.f;
            if (live) {
                pj = expf(s * scale - l);
                dsj = pj * (dp - delta);
            }
            #pragma unroll
            for (int e = 0; e < 8; e++) dq8[e] = fmaf(dsj, k8[e], dq8[e]);
            if (j < L) {
                const float sd = scale * dsj;
                #pragma unroll
                for (int e = 0; e < 8; e++) t8[e] = sd * q8[e];
                st8(dbase + (long)j * lddkv, t8);
                #pragma unroll
                for (int e = 0; e < 8; e++) t8[e] = pj * g8[e];
                st8(dbase + (long)j * lddkv + D, t8);
            }
            if ((lane & 3) == 0) { sds += dsj; sp += pj; }
        }
        // dq: the 8 key-row groups' partial sums; sds / sp: one lane per row
        #pragma unroll
        for (int e = 0; e < 8; e++) {
            #pragma unroll
            for (int o = 4; o < 32; o <<= 1) dq8[e] += __shfl_xor_sync(0xffffffffu, dq8[e], o);
            dq8[e] *= scale;
        }
        sds = warp_sum(sds);
        sp = warp_sum(sp);
        if (rg == 0) {
            st8(dqo + (long)n * lddq + h * DH + c8, dq8);
            #pragma unroll
            for (int e = 0; e < 8; e++) {
                acc[c8 + e] += dq8[e];
                acc[32 + c8 + e] += scale * sds * q8[e];
                acc[64 + c8 + e] += sp * g8[e];
            }
        }
    }
    __syncwarp();
    if (dbias)
        for (int i = lane; i < 96; i += 32) atomicAdd(&dbias[(i >> 5) * D + h * DH + (i & 31)], acc[i]);
}

}  // namespace

// attention implementation for bf16 operands: 0 = mma.sync both passes,
// 1 = tcgen05 / TMEM both passes, 2 = tcgen05 backward with the mma.sync
// forward; set by ptcg_set_attention_impl or, at load, by PTCG_ATTN_TC
#ifndef ATTN_IMPL_DEFAULT
#define ATTN_IMPL_DEFAULT 0
#endif
static std::atomic<int> g_attn_impl{-1};

static int attn_impl() {
    int v = g_attn_impl.load();
    if (v < 0) {
        const char* e = getenv("PTCG_ATTN_TC");
        v = (e && (e[0] == '0' || e[0] == '1' || e[0] == '2') && !e[1]) ? e[0] - '0'
                                                                         : ATTN_IMPL_DEFAULT;
        int expect = -1;
        g_attn_impl.compare_exchange_strong(expect, v);
        v = g_attn_impl.load();
    }
    return v;
}
bool attn_tc_fwd() { return attn_impl() == 1; }
int attn_get_impl() { return attn_impl(); }
bool attn_tc_bwd() { return attn_impl() != 0; }

void attn_set_impl(int impl) { g_attn_impl.store(impl >= 0 && impl <= 2 ? impl : 0); }

namespace {

int num_sms() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 1;
    }
    return n;
}

template <typename K>
void set_smem(K k, size_t bytes) {
    if (bytes > 48 * 1024)
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

}  // namespace

// run fn(key words): the caller's, or, for callers without them (the
// attention test entries), words built in stream-ordered scratch
template <class F>
static bool with_key_words(const uint32_t* kw, const uint8_t* keep, const int* extent, int nseq,
                           int L, cudaStream_t s, F fn) {
    if (kw) return fn(kw);
    uint32_t* tmp = nullptr;
    if (cudaMallocAsync((void**)&tmp, (size_t)nseq * ATTN_KW_WORDS * 4, s) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    attn_keep_words(tmp, keep, extent, nseq, L, s);
    const bool done = fn(tmp);
    cudaFreeAsync(tmp, s);
    return done;
}

void attn_fwd(int dtype, const void* qkv, long ldqkv, const uint8_t* keep,
              void* out, long ldo, float* lse, int nseq, int L, int H, cudaStream_t s,
              const int* extent, const uint32_t* kw) {
    if (nseq <= 0) return;
    size_t sm = fwd_smem(L);
    if (dtype == DT_F32) {
        set_smem(k_attn_fwd<float>, sm);
        ++g_ptcg_launches, k_attn_fwd<float><<<nseq * H, NW * 32, sm, s>>>((const float*)qkv, ldqkv, keep,
            (float*)out, ldo, lse, L, H);
    } else {
        // tcgen05 / TMEM path first; the mma.sync kernel serves shapes it
        // does not take and runs when PTCG_ATTN_TC=0
        if (attn_tc_fwd() && with_key_words(kw, keep, extent, nseq, L, s, [&](const uint32_t* w) {
                return attn_fwd_tc(qkv, ldqkv, w, out, ldo, lse, nseq, L, H, s);
            }))
            return;
        size_t sm2 = fwd_mma_smem(L);
        set_smem(k_attn_fwd_mma, sm2);
        ++g_ptcg_launches, k_attn_fwd_mma<<<nseq * H, 128, sm2, s>>>((const bf16*)qkv, ldqkv, keep,
            (bf16*)out, ldo, lse, L, H, extent);
    }
}

void attn_row0_fwd(int dtype, const void* q, long ldq, const void* kv, long ldkv,
                   const uint8_t* keep, void* out, long ldo, float* lse, int nseq, int L, int H,
                   cudaStream_t s) {
    if (nseq <= 0) return;
    size_t sm = sizeof(float) * H * ((L + 31) & ~31);
    if (dtype == DT_F32) {
        set_smem(k_attn_row0_fwd<float>, sm);
        ++g_ptcg_launches, k_attn_row0_fwd<float><<<nseq, H * 32, sm, s>>>((const float*)q, ldq,
            (const float*)kv, ldkv, keep, (float*)out, ldo, lse, L, H);
    } else {
        set_smem(k_attn_row0_fwd<bf16>, sm);
        ++g_ptcg_launches, k_attn_row0_fwd<bf16><<<nseq, H * 32, sm, s>>>((const bf16*)q, ldq,
            (const bf16*)kv, ldkv, keep, (bf16*)out, ldo, lse, L, H);
    }
}

void attn_row0_bwd(int dtype, const void* q, long ldq, const void* kv, long ldkv,
                   const uint8_t* keep, const void* out, long ldo, const void* dout, long lddo,
                   const float* lse, void* dq, long lddq, void* dkv, long lddkv, float* dbias,
                   int nseq, int L, int H, cudaStream_t s) {
    if (nseq <= 0) return;
    size_t sm = sizeof(float) * H * 96;
    int per_sm = H * 32 <= 256 ? 8 : 4;
    unsigned grid = (unsigned)std::min<long>(nseq, (long)num_sms() * per_sm);
    if (dtype == DT_F32) {
        set_smem(k_attn_row0_bwd<float>, sm);
        ++g_ptcg_launches, k_attn_row0_bwd<float><<<grid, H * 32, sm, s>>>((const float*)q, ldq,
            (const float*)kv, ldkv, keep, (const float*)out, ldo, (const float*)dout, lddo, lse,
            (float*)dq, lddq, (float*)dkv, lddkv, dbias, nseq, L, H);
    } else {
        set_smem(k_attn_row0_bwd<bf16>, sm);
        ++g_ptcg_launches, k_attn_row0_bwd<bf16><<<grid, H * 32, sm, s>>>((const bf16*)q, ldq,
            (const bf16*)kv, ldkv, keep, (const bf16*)out, ldo, (const bf16*)dout, lddo, lse,
            (bf16*)dq, lddq, (bf16*)dkv, lddkv, dbias, nseq, L, H);
    }
}

void attn_bwd(int dtype, const void* qkv, long ldqkv, const uint8_t* keep,
              const void* out, long ldo, const void* dout, long lddo,
              const float* lse, void* dqkv, long lddqkv, float* dbias, int nseq, int L, int H,
              cudaStream_t s, const int* extent, const uint32_t* kw) {
    if (nseq <= 0) return;
    size_t sm = bwd_smem(L);
    if (dtype == DT_F32) {
        set_smem(k_attn_bwd<float>, sm);
        ++g_ptcg_launches, k_attn_bwd<float><<<nseq * H, NW * 32, sm, s>>>((const float*)qkv, ldqkv, keep,
            (const float*)out, ldo, (const float*)dout, lddo, lse, (float*)dqkv, lddqkv, dbias, L, H);
        return;
    }
    // tcgen05 backward for the sequences whose extent fits one 128-row
    // tile; the mma.sync kernel takes the rest (all of them without it)
    int skip = 0;
    if (attn_tc_bwd()) {
        const bool done = with_key_words(kw, keep, extent, nseq, L, s, [&](const uint32_t* w) {
            return attn_bwd_tc(qkv, ldqkv, w, out, ldo, dout, lddo, lse, dqkv, lddqkv, dbias, nseq,
                               L, H, s);
        });
        if (done) {
            if (L <= 128) return;
            skip = 128;
        }
    }
    size_t sm2 = bwd_mma_smem(L);
    set_smem(k_attn_bwd_mma, sm2);
    ++g_ptcg_launches, k_attn_bwd_mma<<<nseq * H, 128, sm2, s>>>((const bf16*)qkv, ldqkv, keep,
        (const bf16*)out, ldo, (const bf16*)dout, lddo, lse, (bf16*)dqkv, lddqkv, dbias, L, H,
        extent, skip);
}
