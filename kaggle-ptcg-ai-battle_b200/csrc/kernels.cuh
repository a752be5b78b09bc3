// Model-specific kernels of the PTCG policy path: observation gathers and
// their gradient scatters, LayerNorm, N=1 heads, aux losses, PPO loss,
// sampler, negamax advantage and the fused Adam.  Included once, by model.cu.
//
// Semantics follow the reference kernels cited per kernel; layouts are this
// library's own (activations row-major with padded leading dimensions).
#pragma once
#include "common.cuh"
#include "internal.h"

// Observation-row field offsets, computed on the host from PtcgShape
// (ptcg/rl/buffers.py:212-237).
struct ObsLayout {
    int obs, toki, tokf, opti, optf, mask, glob, deci, decf, orc;
    int ltok, lseq, nopt, tok_f, nc, na, ns;
};

static inline __device__ void st(float* p, float v) { *p = v; }
static inline __device__ void st(bf16* p, float v) { *p = __float2bfloat16_rn(v); }

// ------------------------------------------------------------ concat rows
struct Seg { const float* src; int ld, src_off, width, dst_off; };
struct Segs { Seg s[8]; int n; };

// out[r, seg.dst_off + c] = seg.src[r * seg.ld + seg.src_off + c]
// (k_att_in / k_sk_in / k_card_in, native/model/ptcg_model.cu:231-286)
__global__ void k_concat_rows(float* out, int ldo, int rows, int width, Segs g) {
    long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i >= (long)rows * width) return;
    int r = (int)(i / width), c = (int)(i % width);
    for (int k = 0; k < g.n; k++) {
        const Seg& s = g.s[k];
        if (c >= s.dst_off && c < s.dst_off + s.width) {
            out[(long)r * ldo + c] = s.src[(long)r * s.ld + s.src_off + (c - s.dst_off)];
            return;
        }
    }
}

// masked mean / max pools of gathered attack / skill vectors; masked slots
// are 0-valued participants of the max (ptcg_model.cu:243-266,
// model.py:194-204).  arg = first index attaining the max.
__global__ void k_pool(float* mean, float* mx, int ldm, int8_t* arg,
                       const float* tab, const int* idx, int NC, int K, int E) {
    long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i >= (long)NC * E) return;
    int n = (int)(i / E), e = (int)(i % E);
    float s = 0.f, m2 = -INFINITY;
    int cnt = 0, am = 0;
    for (int k = 0; k < K; k++) {
        int id = idx[n * K + k];
        float v = id > 0 ? tab[(long)id * E + e] : 0.f;
        if (id > 0) { cnt++; s += v; }
        if (v > m2) { m2 = v; am = k; }
    }
    mean[(long)n * ldm + e] = s / (float)(cnt > 0 ? cnt : 1);
    mx[(long)n * ldm + e] = m2;
    arg[i] = (int8_t)am;
}

// pool backward (ptcg_model2.cu:15-33): d_mean spread over unmasked slots,
// d_max to the arg-max slot when unmasked.
__global__ void k_pool_bwd(float* d_tab, const float* dsrc, int ld, int off_mean,
                           int off_max, const int8_t* arg, const int* idx,
                           int NC, int K, int E) {
    long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i >= (long)NC * E) return;
    int n = (int)(i / E), e = (int)(i % E);
    int cnt = 0;
    for (int k = 0; k < K; k++) cnt += idx[n * K + k] > 0;
    float dm = dsrc[(long)n * ld + off_mean + e] / (float)(cnt > 0 ? cnt : 1);
    float dx = dsrc[(long)n * ld + off_max + e];
    int am = arg[i];
    for (int k = 0; k < K; k++) {
        int id = idx[n * K + k];
        if (id <= 0) continue;
        float g = dm + (k == am ? dx : 0.f);
        if (g != 0.f) atomicAdd(&d_tab[(long)id * E + e], g);
    }
}

// ------------------------------------------------------------- LayerNorm
// one warp per row, eps 1e-5 (torch nn.LayerNorm), two-pass statistics.
// VEC: D % 128 == 0 and 16-byte aligned rows -> each lane owns 4 consecutive
// columns of every 128-column chunk (float4 loads, 8-byte bf16 stores).
// ext (nullable): rows of each lseq-row sequence that anything reads;
// rowkeep (nullable): per row, 0 for rows read by nothing (masked keys of a
// sequence whose only query is its first row).  Skipped rows are left as
// they are (finite: the workspace starts zeroed and only ever holds finite
// values), since nothing reads them
// CRIT (vector path): the rows are the critic's crit_lcrit-row sequences
// [readout | trunk rows | oracle tokens], whose crit_lseq trunk rows are read
// from crit_h (the trunk output, rows n * crit_lseq .., ld D) instead of x
template <typename TO, int VEC, bool CRIT = false>
__global__ void k_ln_fwd(TO* y, long ldy, float* mean, float* rstd, const float* x,
                         long ldx, const float* w, const float* b, int rows, int D,
                         const int* ext = nullptr, int lseq = 1,
                         const uint8_t* rowkeep = nullptr, const float* crit_h = nullptr,
                         int crit_lseq = 0, int crit_lcrit = 0) {
    int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    int lane = threadIdx.x & 31;
    if (row >= rows) return;
    if (ext) {
        const int n = row / lseq;
        if (row - n * lseq >= ext[n]) return;
    }
    if (rowkeep && !rowkeep[row]) return;
    const float* xr = x + (long)row * ldx;
    if (CRIT) {
        const int n = row / crit_lcrit, l = row - n * crit_lcrit;
        if (l >= 1 && l <= crit_lseq) xr = crit_h + ((long)n * crit_lseq + l - 1) * D;
    }
    TO* yr = y + (long)row * ldy;
    if (VEC > 0) {
        float4 v[VEC > 0 ? VEC : 1];
        float s = 0.f;
        #pragma unroll
        for (int c = 0; c < VEC; c++) {
            v[c] = *(const float4*)(xr + c * 128 + lane * 4);
            s += v[c].x + v[c].y + v[c].z + v[c].w;
        }
        float mu = warp_sum(s) / D;
        float q = 0.f;
        #pragma unroll
        for (int c = 0; c < VEC; c++) {
            float a0 = v[c].x - mu, a1 = v[c].y - mu, a2 = v[c].z - mu, a3 = v[c].w - mu;
            q += a0 * a0 + a1 * a1 + a2 * a2 + a3 * a3;
        }
        float rs = rsqrtf(warp_sum(q) / D + 1e-5f);
        if (lane == 0) { mean[row] = mu; rstd[row] = rs; }
        #pragma unroll
        for (int c = 0; c < VEC; c++) {
            int i = c * 128 + lane * 4;
            float4 wv = *(const float4*)(w + i), bv = *(const float4*)(b + i);
            float o0 = (v[c].x - mu) * rs * wv.x + bv.x, o1 = (v[c].y - mu) * rs * wv.y + bv.y;
            float o2 = (v[c].z - mu) * rs * wv.z + bv.z, o3 = (v[c].w - mu) * rs * wv.w + bv.w;
            if (sizeof(TO) == 4) {
                *(float4*)((float*)yr + i) = make_float4(o0, o1, o2, o3);
            } else {
                __nv_bfloat162 h0 = __floats2bfloat162_rn(o0, o1), h1 = __floats2bfloat162_rn(o2, o3);
                uint2 u; u.x = *(uint32_t*)&h0; u.y = *(uint32_t*)&h1;
                *(uint2*)((bf16*)yr + i) = u;
            }
        }
        return;
    }
    float s = 0.f;
    for (int i = lane; i < D; i += 32) s += xr[i];
    float mu = warp_sum(s) / D;
    float v = 0.f;
    for (int i = lane; i < D; i += 32) { float d = xr[i] - mu; v += d * d; }
    float rs = rsqrtf(warp_sum(v) / D + 1e-5f);
    if (lane == 0) { mean[row] = mu; rstd[row] = rs; }
    for (int i = lane; i < D; i += 32) st(&yr[i], (xr[i] - mu) * rs * w[i] + b[i]);
}

// dx = LN'(dy) (+ dx if accumulate), optional copy in T; dw/db accumulate.
// One warp per row with every load of the row (x, dy and the dx being
// accumulated into) issued before the reductions; the dw/db partials stay in
// registers across the block's rows, reach shared memory once per warp and
// global memory once per block.  VEC > 0: D = 128 * VEC, float4 access (lane
// owns 4 consecutive columns of each 128-column chunk); VEC == 0: generic D
// (<= 32 * MAXC) with scalar access.
// four consecutive values of a float or bf16 row as a float4
PTCG_DEV float4 ld4any(const float* p) { return *reinterpret_cast<const float4*>(p); }
PTCG_DEV float4 ld4any(const bf16* p) {
    uint2 u = *reinterpret_cast<const uint2*>(p);
    float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
    float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
    return make_float4(a.x, a.y, b.x, b.y);
}

// dy is float or bf16 (TY); statistics, dx and the parameter grads are fp32
template <typename TC, int VEC, int MAXC, typename TY = float, bool CRIT = false>
__global__ void __launch_bounds__(256, VEC == 2 ? 3 : 1) k_ln_bwd(float* dx, long lddx, int accumulate, TC* dxc, long lddxc,
                         float* dw, float* db, const TY* dy, long lddy,
                         const float* x, long ldx, const float* w, const float* mean,
                         const float* rstd, int rows, int D, int rows_per_block,
                         float* out_cs, const int* ext = nullptr, int lseq = 1,
                         const uint8_t* rowkeep = nullptr, float* crit_dh = nullptr,
                         int crit_lseq = 0, int crit_lcrit = 0, const float* crit_h = nullptr) {
    // out_cs (nullable): += column sums of the resulting dx (the bias grad
    // of the layer that produced this residual stream).  ext (nullable):
    // rows of each lseq-row sequence that anything reads; past it dy is zero
    // and so is the residual gradient, which is written as zeros without
    // reading anything.  rowkeep (nullable): the same for rows marked 0.
    // crit_dh (CRIT instantiations, vector path): the rows are the critic's
    // crit_lcrit-row sequences [readout | trunk rows | oracle tokens]; the
    // crit_lseq trunk rows of sequence n go to crit_dh rows n * crit_lseq ..
    // (d_h, ld D) instead of dx, the oracle-token rows also to dxc rows
    // n * (crit_lcrit - 1 - crit_lseq) .., and row 0 to dx alone.  crit_h
    // (nullable): the trunk rows' x is read from there (rows n * crit_lseq
    // .., ld D), as the CRIT forward did
    extern __shared__ float sh[];               // [3][D]
    float* sw = sh;
    float* sb = sh + D;
    float* so = sh + 2 * D;
    for (int i = threadIdx.x; i < 3 * D; i += blockDim.x) sh[i] = 0.f;
    __syncthreads();
    int nw = blockDim.x >> 5, wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int r0 = blockIdx.x * rows_per_block;
    int r1 = min(rows, r0 + rows_per_block);
    if (VEC > 0) {
        float4 pw[VEC > 0 ? VEC : 1], pb[VEC > 0 ? VEC : 1], wv[VEC > 0 ? VEC : 1];
        float4 po[VEC > 0 ? VEC : 1];
        #pragma unroll
        for (int c = 0; c < VEC; c++) {
            pw[c] = make_float4(0, 0, 0, 0); pb[c] = make_float4(0, 0, 0, 0);
            po[c] = make_float4(0, 0, 0, 0);
            wv[c] = *(const float4*)(w + c * 128 + lane * 4);
        }
        for (int row = r0 + wid; row < r1; row += nw) {
            const float* xr = x + (long)row * ldx;
            const TY* dyr = dy + (long)row * lddy;
            float* dxr = dx + (long)row * lddx;
            TC* dxcr = dxc ? dxc + (long)row * lddxc : nullptr;
            if (CRIT) {
                const int n = row / crit_lcrit, l = row - n * crit_lcrit;
                if (l >= 1 && l <= crit_lseq) {
                    dxr = crit_dh + ((long)n * crit_lseq + l - 1) * D;
                    dxcr = nullptr;
                    if (crit_h) xr = crit_h + ((long)n * crit_lseq + l - 1) * D;
                } else if (l == 0) {
                    dxcr = nullptr;
                } else if (dxc) {
                    dxcr = dxc + ((long)n * (crit_lcrit - 1 - crit_lseq) + (l - 1 - crit_lseq)) * lddxc;
                }
            }
            bool unread = rowkeep && !rowkeep[row];
            if (ext) {
                const int n = row / lseq;
                unread = unread || row - n * lseq >= ext[n];
            }
            if (unread) {
                #pragma unroll
                for (int c = 0; c < VEC; c++) {
                    const int i = c * 128 + lane * 4;
                    *(float4*)(dxr + i) = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (dxcr) {
                        if (sizeof(TC) == 4) *(float4*)((float*)dxcr + i) = make_float4(0.f, 0.f, 0.f, 0.f);
                        else *(uint2*)((bf16*)dxcr + i) = make_uint2(0u, 0u);
                    }
                }
                continue;
            }
            float4 xv[VEC > 0 ? VEC : 1], gv[VEC > 0 ? VEC : 1], av[VEC > 0 ? VEC : 1];
            #pragma unroll
            for (int c = 0; c < VEC; c++) {
                int i = c * 128 + lane * 4;
                xv[c] = *(const float4*)(xr + i);
                gv[c] = ld4any(dyr + i);
                av[c] = accumulate ? *(const float4*)(dxr + i) : make_float4(0, 0, 0, 0);
            }
            float mu = mean[row], rs = rstd[row];
            float s1 = 0.f, s2 = 0.f;
            #pragma unroll
            for (int c = 0; c < VEC; c++) {
                float h0 = (xv[c].x - mu) * rs, h1 = (xv[c].y - mu) * rs;
                float h2 = (xv[c].z - mu) * rs, h3 = (xv[c].w - mu) * rs;
                pw[c].x += gv[c].x * h0; pw[c].y += gv[c].y * h1;
                pw[c].z += gv[c].z * h2; pw[c].w += gv[c].w * h3;
                pb[c].x += gv[c].x; pb[c].y += gv[c].y; pb[c].z += gv[c].z; pb[c].w += gv[c].w;
                float g0 = gv[c].x * wv[c].x, g1 = gv[c].y * wv[c].y;
                float g2 = gv[c].z * wv[c].z, g3 = gv[c].w * wv[c].w;
                s1 += g0 + g1 + g2 + g3;
                s2 += g0 * h0 + g1 * h1 + g2 * h2 + g3 * h3;
                xv[c] = make_float4(h0, h1, h2, h3);          // keep x-hat
                gv[c] = make_float4(g0, g1, g2, g3);          // keep dy * w
            }
            float m1 = warp_sum(s1) / D, m2 = warp_sum(s2) / D;
            #pragma unroll
            for (int c = 0; c < VEC; c++) {
                int i = c * 128 + lane * 4;
                float o0 = (gv[c].x - m1 - xv[c].x * m2) * rs + av[c].x;
                float o1 = (gv[c].y - m1 - xv[c].y * m2) * rs + av[c].y;
                float o2 = (gv[c].z - m1 - xv[c].z * m2) * rs + av[c].z;
                float o3 = (gv[c].w - m1 - xv[c].w * m2) * rs + av[c].w;
                *(float4*)(dxr + i) = make_float4(o0, o1, o2, o3);
                po[c].x += o0; po[c].y += o1; po[c].z += o2; po[c].w += o3;
                if (dxcr) {
                    if (sizeof(TC) == 4) {
                        *(float4*)((float*)dxcr + i) = make_float4(o0, o1, o2, o3);
                    } else {
                        __nv_bfloat162 q0 = __floats2bfloat162_rn(o0, o1), q1 = __floats2bfloat162_rn(o2, o3);
                        uint2 u; u.x = *(uint32_t*)&q0; u.y = *(uint32_t*)&q1;
                        *(uint2*)((bf16*)dxcr + i) = u;
                    }
                }
            }
        }
        #pragma unroll
        for (int c = 0; c < VEC; c++) {
            int i = c * 128 + lane * 4;
            atomicAdd(&sw[i], pw[c].x); atomicAdd(&sw[i + 1], pw[c].y);
            atomicAdd(&sw[i + 2], pw[c].z); atomicAdd(&sw[i + 3], pw[c].w);
            atomicAdd(&sb[i], pb[c].x); atomicAdd(&sb[i + 1], pb[c].y);
            atomicAdd(&sb[i + 2], pb[c].z); atomicAdd(&sb[i + 3], pb[c].w);
            if (out_cs) {
                atomicAdd(&so[i], po[c].x); atomicAdd(&so[i + 1], po[c].y);
                atomicAdd(&so[i + 2], po[c].z); atomicAdd(&so[i + 3], po[c].w);
            }
        }
    } else {
        float pw[MAXC], pb[MAXC], po[MAXC];
        #pragma unroll
        for (int c = 0; c < MAXC; c++) { pw[c] = 0.f; pb[c] = 0.f; po[c] = 0.f; }
        const int nc = (D + 31) / 32;
        for (int row = r0 + wid; row < r1; row += nw) {
            const float* xr = x + (long)row * ldx;
            const TY* dyr = dy + (long)row * lddy;
            float* dxr = dx + (long)row * lddx;
            float mu = mean[row], rs = rstd[row];
            float xh[MAXC], g[MAXC], acc[MAXC];
            float s1 = 0.f, s2 = 0.f;
            #pragma unroll
            for (int c = 0; c < MAXC; c++) {
                int i = lane + 32 * c;
                if (c < nc && i < D) {
                    xh[c] = (xr[i] - mu) * rs;
                    float dyv = to_f<TY>(dyr[i]);
                    acc[c] = accumulate ? dxr[i] : 0.f;
                    g[c] = dyv * w[i];
                    s1 += g[c]; s2 += g[c] * xh[c];
                    pw[c] += dyv * xh[c];
                    pb[c] += dyv;
                }
            }
            float m1 = warp_sum(s1) / D, m2 = warp_sum(s2) / D;
            #pragma unroll
            for (int c = 0; c < MAXC; c++) {
                int i = lane + 32 * c;
                if (c < nc && i < D) {
                    float v = (g[c] - m1 - xh[c] * m2) * rs + acc[c];
                    dxr[i] = v;
                    po[c] += v;
                    if (dxc) st(&dxc[(long)row * lddxc + i], v);
                }
            }
        }
        #pragma unroll
        for (int c = 0; c < MAXC; c++) {
            int i = lane + 32 * c;
            if (c < nc && i < D) {
                atomicAdd(&sw[i], pw[c]); atomicAdd(&sb[i], pb[c]);
                if (out_cs) atomicAdd(&so[i], po[c]);
            }
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < D; i += blockDim.x) {
        if (sw[i] != 0.f) atomicAdd(&dw[i], sw[i]);
        if (sb[i] != 0.f) atomicAdd(&db[i], sb[i]);
        if (out_cs && so[i] != 0.f) atomicAdd(&out_cs[i], so[i]);
    }
}

// ---------------------------------------------------------- token gather
// [card_vec(cid) | sum tool card_vecs (id > 0) | tok_f | zone_emb | owner_emb]
// (k_tok_cat, ptcg_model.cu:289-321; model.py:211-221)
template <typename T>
__global__ void k_tok_cat(T* out, long ldo, const float* obs, ObsLayout L,
                          const float* cv, const float* zemb, const float* oemb,
                          int R, int tok_in, const int* ext = nullptr) {
    // one warp per token row, four consecutive columns per lane; tokens at
    // or past the sequence's extent (row l + 1) are read by nothing and are
    // left as they are
    long nl = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (nl >= (long)R * L.ltok) return;
    const int n = (int)(nl / L.ltok), l = (int)(nl - (long)n * L.ltok);
    if (ext && l + 1 >= ext[n]) return;
    const float* row = obs + (long)n * L.obs;
    const float* ti = row + L.toki + l * 5;
    const float* c0 = cv + (long)id_clamp(ti[0], L.nc) * 128;
    const int t0 = (int)ti[3], t1 = (int)ti[4];
    const float* ca = t0 > 0 ? cv + (long)(t0 >= L.nc ? L.nc - 1 : t0) * 128 : nullptr;
    const float* cb = t1 > 0 ? cv + (long)(t1 >= L.nc ? L.nc - 1 : t1) * 128 : nullptr;
    const float* ze = zemb + id_clamp(ti[1], 16) * 8;
    const float* oe = oemb + id_clamp(ti[2], 4) * 4;
    const float* tf = row + L.tokf + l * L.tok_f;
    T* o = out + nl * ldo;
    for (int c4 = lane * 4; c4 < tok_in; c4 += 128) {
        float4 v;
        if (c4 + 4 <= 128) {
            v = ld4(c0 + c4);
        } else if (c4 >= 128 && c4 + 4 <= 256) {
            float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
            v = add4(ca ? ld4(ca + c4 - 128) : z, cb ? ld4(cb + c4 - 128) : z);
        } else {
            float e[4];
            #pragma unroll
            for (int k = 0; k < 4; k++) {
                int c = c4 + k;
                float x = 0.f;
                if (c >= tok_in) x = 0.f;
                else if (c < 256 + L.tok_f) x = tf[c - 256];
                else if (c < 264 + L.tok_f) x = ze[c - 256 - L.tok_f];
                else x = oe[c - 264 - L.tok_f];
                e[k] = x;
            }
            v = make_float4(e[0], e[1], e[2], e[3]);
        }
        if (c4 + 4 <= tok_in || c4 + 4 <= ldo) st4(o + c4, v);
    }
}

// x0 readout rows + key mask keep = [1, zone > 0] (k_x0, ptcg_model.cu:348-368)
__global__ void k_x0_readout(float* x0, uint8_t* keep, const float* readout,
                             const float* obs, ObsLayout L, int R, int D) {
    long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    long nrd = (long)R * D;
    if (i < nrd) {
        int n = (int)(i / D), d = (int)(i % D);
        x0[(long)n * L.lseq * D + d] = readout[d];
    }
    if (i < (long)R * L.lseq) {
        int n = (int)(i / L.lseq), l = (int)(i % L.lseq);
        uint8_t kp = 1;
        if (l > 0) kp = obs[(long)n * L.obs + L.toki + (l - 1) * 5 + 1] > 0.f;
        keep[i] = kp;
    }
}

// Rows of each trunk sequence that anything reads: 1 + the largest of the
// last kept row (readout row 0 and tokens with zone > 0: attention keys,
// the aux heads' rows) and the largest option pointer in [1, LTOK] (the
// gathers of ln_f rows).  Rows past it are read by nothing (masked as keys,
// never gathered), so the attention forward may skip them.  One warp per
// sequence.
// kw (nullable): also the key words of the tcgen05 attention, ATTN_KW_WORDS
// per sequence: bits of the kept keys 32j.. in word j, the extent in the last
// (no key at or past the extent is kept, so the bits need no clipping)
__global__ void k_row_extent(int* ext, const uint8_t* keep, const float* obs, ObsLayout L, int R,
                             uint32_t* kw) {
    const int n = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (n >= R) return;
    int e = 0;
    uint32_t word = 0;
    for (int j = 0; j * 32 < L.lseq; j++) {
        const int l = 32 * j + lane;
        const bool k = l < L.lseq && keep[(long)n * L.lseq + l];
        if (k) e = max(e, l);
        const uint32_t b = __ballot_sync(0xffffffffu, k);
        if (lane == j) word = b;
    }
    const float* oi = obs + (long)n * L.obs + L.opti;
    for (int j = lane; j < L.nopt; j += 32) {
        const int p1 = (int)oi[j * 6 + 1], p2 = (int)oi[j * 6 + 2];
        if (p1 >= 1 && p1 <= L.ltok) e = max(e, p1);
        if (p2 >= 1 && p2 <= L.ltok) e = max(e, p2);
    }
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) e = max(e, __shfl_xor_sync(0xffffffffu, e, o));
    if (lane == 0) ext[n] = e + 1;
    if (kw && lane < ATTN_KW_WORDS)
        kw[(long)n * ATTN_KW_WORDS + lane] = lane == ATTN_KW_WORDS - 1 ? (uint32_t)(e + 1) : word;
}

// decision-encoder input (696): [sel8, ctx32, cv_eff, cv_ctx, av_my, av_opp,
// cv_msup, cv_osup, decf16] (k_dec_in, ptcg_model.cu:324-344)
__global__ void k_dec_in(float* out, const float* obs, ObsLayout L, const float* cv,
                         const float* av, const float* semb, const float* cemb, int R) {
    const int W = 696;
    long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i >= (long)R * W) return;
    int n = (int)(i / W), c = (int)(i % W);
    const float* row = obs + (long)n * L.obs;
    const float* di = row + L.deci;
    float v;
    if (c < 8) v = semb[id_clamp(di[0], 29) * 8 + c];
    else if (c < 40) v = cemb[id_clamp(di[1], 65) * 32 + (c - 8)];
    else if (c < 168) v = cv[(long)id_clamp(di[2], L.nc) * 128 + (c - 40)];
    else if (c < 296) v = cv[(long)id_clamp(di[3], L.nc) * 128 + (c - 168)];
    else if (c < 360) v = av[(long)id_clamp(di[4], L.na) * 64 + (c - 296)];
    else if (c < 424) v = av[(long)id_clamp(di[5], L.na) * 64 + (c - 360)];
    else if (c < 552) v = cv[(long)id_clamp(di[6], L.nc) * 128 + (c - 424)];
    else if (c < 680) v = cv[(long)id_clamp(di[7], L.nc) * 128 + (c - 552)];
    else v = row[L.decf + (c - 680)];
    out[i] = v;
}

__global__ void k_dec_in_bwd(float* d_cv, float* d_av, float* d_semb, float* d_cemb,
                             const float* g, const float* obs, ObsLayout L, int R) {
    const int W = 696;
    long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i >= (long)R * W) return;
    int n = (int)(i / W), c = (int)(i % W);
    float v = g[i];
    if (v == 0.f || c >= 680) return;
    const float* di = obs + (long)n * L.obs + L.deci;
    if (c < 8) atomicAdd(&d_semb[id_clamp(di[0], 29) * 8 + c], v);
    else if (c < 40) atomicAdd(&d_cemb[id_clamp(di[1], 65) * 32 + (c - 8)], v);
    else if (c < 168) atomicAdd(&d_cv[(long)id_clamp(di[2], L.nc) * 128 + (c - 40)], v);
    else if (c < 296) atomicAdd(&d_cv[(long)id_clamp(di[3], L.nc) * 128 + (c - 168)], v);
    else if (c < 360) atomicAdd(&d_av[(long)id_clamp(di[4], L.na) * 64 + (c - 296)], v);
    else if (c < 424) atomicAdd(&d_av[(long)id_clamp(di[5], L.na) * 64 + (c - 360)], v);
    else if (c < 552) atomicAdd(&d_cv[(long)id_clamp(di[6], L.nc) * 128 + (c - 424)], v);
    else atomicAdd(&d_cv[(long)id_clamp(di[7], L.nc) * 128 + (c - 552)], v);
}

// ------------------------------------------------------------ options
// q_in: [type16 | h(ptr1) | h(ptr2) | opt_card(cv(cid)) | opt_attack(av(aid)) | optf8]
// ptr p in (0, LTOK] reads h row p, otherwise zeros (ptcg_model.cu:371-419).
// The two projections are applied per table row beforehand (poc = opt_card
// over all NC card vectors, poa = opt_attack over all NA attack vectors):
// gathering a projected row equals projecting the gathered row.
// one warp per option row, four consecutive columns per lane (every
// segment boundary is a multiple of 4)
__global__ void k_q_in(float* out, long ldo, const float* obs, ObsLayout L, const float* h,
                       int D, const float* temb, const float* poc, const float* poa,
                       int R, int q_in) {
    long nj = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (nj >= (long)R * L.nopt) return;
    const int n = (int)(nj / L.nopt), j = (int)(nj - (long)n * L.nopt);
    const float* row = obs + (long)n * L.obs;
    const float* oi = row + L.opti + j * 6;
    const float* te = temb + id_clamp(oi[0], 33) * 16;
    const int p1 = (int)oi[1], p2 = (int)oi[2];
    const float* h1 = (p1 <= 0 || p1 > L.ltok) ? nullptr : h + ((long)n * L.lseq + p1) * D;
    const float* h2 = (p2 <= 0 || p2 > L.ltok) ? nullptr : h + ((long)n * L.lseq + p2) * D;
    const float* pc = poc + (long)id_clamp(oi[3], L.nc) * 64;
    const float* pa = poa + (long)id_clamp(oi[4], L.na) * 64;
    const float* of = row + L.optf + j * 8;
    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
    float* o = out + nj * ldo;
    for (int c = lane * 4; c < q_in; c += 128) {
        float4 v;
        if (c < 16) v = ld4(te + c);
        else if (c < 16 + D) v = h1 ? ld4(h1 + (c - 16)) : z;
        else if (c < 16 + 2 * D) v = h2 ? ld4(h2 + (c - 16 - D)) : z;
        else if (c < 16 + 2 * D + 64) v = ld4(pc + (c - 16 - 2 * D));
        else if (c < 16 + 2 * D + 128) v = ld4(pa + (c - 80 - 2 * D));
        else {
            int e = c - 144 - 2 * D;                    // the obs row may be unaligned here
            v = make_float4(of[e], of[e + 1], of[e + 2], of[e + 3]);
        }
        st4(o + c, v);
    }
}

__global__ void k_q_in_bwd(float* d_temb, float* d_h, float* d_poc, float* d_poa,
                           const float* g, long ldg, const float* obs, ObsLayout L,
                           int D, int R, int q_in) {
    long nj = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (nj >= (long)R * L.nopt) return;
    const int n = (int)(nj / L.nopt), j = (int)(nj - (long)n * L.nopt);
    const float* oi = obs + (long)n * L.obs + L.opti + j * 6;
    float* te = d_temb + id_clamp(oi[0], 33) * 16;
    const int p1 = (int)oi[1], p2 = (int)oi[2];
    float* h1 = (p1 <= 0 || p1 > L.ltok) ? nullptr : d_h + ((long)n * L.lseq + p1) * D;
    float* h2 = (p2 <= 0 || p2 > L.ltok) ? nullptr : d_h + ((long)n * L.lseq + p2) * D;
    float* pc = d_poc + (long)id_clamp(oi[3], L.nc) * 64;
    float* pa = d_poa + (long)id_clamp(oi[4], L.na) * 64;
    const float* gr = g + nj * ldg;
    for (int c = lane * 4; c < 16 + 2 * D + 128; c += 128) {
        float4 v = ld4(gr + c);
        if (!nz4(v)) continue;
        float* t;
        if (c < 16) t = te + c;
        else if (c < 16 + D) t = h1 ? h1 + (c - 16) : nullptr;
        else if (c < 16 + 2 * D) t = h2 ? h2 + (c - 16 - D) : nullptr;
        else if (c < 16 + 2 * D + 64) t = pc + (c - 16 - 2 * D);
        else t = pa + (c - 80 - 2 * D);
        if (t) red_add4(t, v);
    }
}

// ---- score1 split: score1(cat[q, r, g, d, q*r]) = [q | q*r] Wqq^T +
//      ([r | g | d] Wrgd^T + b) broadcast over the sample's options
// qq = [q | q*r] (NO x 2D): the second half from the first and r = h[n, 0]
__global__ void k_qr_fill(float* qq, int D, const float* h, int lseq, int nopt, long rows) {
    long nj = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (nj >= rows) return;
    const int n = (int)(nj / nopt);
    const float* r = h + (long)n * lseq * D;
    float* row = qq + nj * 2 * D;
    for (int c = lane * 4; c < D; c += 128) {
        float4 q = ld4(row + c), rr = ld4(r + c);
        st4(row + D + c, make_float4(q.x * rr.x, q.y * rr.y, q.z * rr.z, q.w * rr.w));
    }
}
// per-sample [r | g | d] (R x (D + 192)), gd = [g | d] (R x 192)
__global__ void k_rgd_fill(float* out, const float* h, int lseq, const float* gd, int D, int R) {
    const int W = D + 192;
    long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i >= (long)R * W) return;
    int n = (int)(i / W), c = (int)(i % W);
    out[i] = c < D ? h[(long)n * lseq * D + c] : gd[(long)n * 192 + (c - D)];
}
// [W_q | W_qr] (rows x 2D) from score1_w (rows x (3D + 192)): columns
// [0, D) and [2D + 192, 3D + 192)
__global__ void k_pack_wqq(float* out, const float* w, int D, long ldw, int rows) {
    long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i >= (long)rows * 2 * D) return;
    int o = (int)(i / (2 * D)), c = (int)(i % (2 * D));
    out[i] = w[(long)o * ldw + (c < D ? c : c + D + 192)];
}
// backward of qq and of [r | g | d], one block per sample:
//   d_q[nj, c] = dqq[nj, c] + dqq[nj, D + c] r[c]        (+ q2 bias colsum)
//   d_h[n, 0, c] += sum_j dqq[nj, D + c] q[nj, c] + drgd[n, c]
//   d_gd[n, e]  += drgd[n, D + e]
// Thread t takes the 4 columns 4 (t % (D/4)) .. of the options j = t / (D/4)
// (mod blockDim / (D/4)); the option groups' sums meet in shared memory.
// D % 4 == 0, D / 4 <= blockDim.x, 16-byte aligned rows.
template <typename T>
__global__ void k_qq_bwd(T* d_q, long lddq, float* d_h, float* d_gd, const float* dqq,
                         const float* qq, const float* drgd, const float* h, int D, int lseq,
                         int nopt, float* dq_colsum) {
    __shared__ float4 part[2][256];
    const int n = blockIdx.x, t = threadIdx.x;
    const int nc4 = D >> 2, G = blockDim.x / nc4;
    const int grp = t / nc4, c = (t - grp * nc4) * 4;
    const float* dr = drgd + (long)n * (D + 192);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f), cs = acc;
    if (grp < G) {
        const float4 rr = ld4(h + (long)n * lseq * D + c);
        for (int j = grp; j < nopt; j += G) {
            const long nj = (long)n * nopt + j;
            const float4 ga = ld4(dqq + nj * 2 * D + c), gb = ld4(dqq + nj * 2 * D + D + c);
            const float4 q = ld4(qq + nj * 2 * D + c);
            const float4 dqv = make_float4(ga.x + gb.x * rr.x, ga.y + gb.y * rr.y,
                                           ga.z + gb.z * rr.z, ga.w + gb.w * rr.w);
            st4(d_q + nj * lddq + c, dqv);
            cs = add4(cs, dqv);
            acc = make_float4(acc.x + gb.x * q.x, acc.y + gb.y * q.y,
                              acc.z + gb.z * q.z, acc.w + gb.w * q.w);
        }
    }
    part[0][t] = acc;
    part[1][t] = cs;
    __syncthreads();
    if (t < nc4) {
        for (int g = 1; g < G; g++) {
            acc = add4(acc, part[0][g * nc4 + t]);
            cs = add4(cs, part[1][g * nc4 + t]);
        }
        float* dh = d_h + (long)n * lseq * D + c;
        const float4 o = ld4(dh);
        st4(dh, make_float4(o.x + (acc.x + dr[c]), o.y + (acc.y + dr[c + 1]),
                            o.z + (acc.z + dr[c + 2]), o.w + (acc.w + dr[c + 3])));
        if (dq_colsum) red_add4(dq_colsum + c, cs);
    }
    for (int e = t; e < 192; e += blockDim.x) d_gd[(long)n * 192 + e] += dr[D + e];
}

// ------------------------------------------------------------ N=1 heads
// out[r * os] = dot(in[inrow(r), :K], w) + b  (score2 / value2 / oracle_v2 /
// aux_prize), warp per row.  inrow(r) = (r / g) * s + o + r % g when g > 0.
template <typename TI>
__global__ void k_rowdot(float* out, long os, const TI* in, long ldi, const float* w,
                         const float* b, int rows, int K, int g, int gs, int go) {
    int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    int lane = threadIdx.x & 31;
    if (r >= rows) return;
    long ir = g > 0 ? (long)(r / g) * gs + go + (r % g) : r;
    const TI* x = in + ir * ldi;
    float s = 0.f;
    for (int k = lane; k < K; k += 32) s += to_f<TI>(x[k]) * w[k];
    s = warp_sum(s);
    if (lane == 0) out[r * os] = s + b[0];
}

// backward of out = dot(gelu(pre), w) + b:  d_pre = d * w * gp (TO) where
// gp = GELU'(pre) saved by the forward epilogue,
// dw += sum_r d * in, db += sum_r d.  d from a strided buffer, or (mode 1,
// blind-V aux) d = coef * (v - ret) / norm with v from the strided buffer.
template <typename TI, typename TO>
__global__ void k_rowdot_bwd(TO* d_pre, long ldd, const TI* pre, long ldp, const TI* in,
                             long ldi, const float* w, float* dw, float* db, const float* dsrc,
                             long ds_stride, const float* ret, float coef, int rows, int K,
                             int rows_per_block, float* loss, float* dpre_colsum,
                             float* dpre_blocksum = nullptr) {
    extern __shared__ float shd[];             // [K] dw partials, [1] db
    for (int k = threadIdx.x; k <= K; k += blockDim.x) shd[k] = 0.f;
    __syncthreads();
    int r0 = blockIdx.x * rows_per_block, r1 = min(rows, r0 + rows_per_block);
    float dbp = 0.f;
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
        float wk = w[k], acc = 0.f, csum = 0.f;
        for (int r = r0; r < r1; r++) {
            float d = dsrc[r * ds_stride];
            if (ret) {
                float e = d - ret[r];
                if (loss && k == 0) atomicAdd(loss, 0.5f * coef * e * e);
                d = coef * e;
            }
            acc += d * to_f<TI>(in[(long)r * ldi + k]);
            float v = d * wk;
            if (pre) v *= to_f<TI>(pre[(long)r * ldp + k]);          // saved GELU'
            st(&d_pre[(long)r * ldd + k], v);
            csum += v;
            if (k == 0) dbp += d;
        }
        shd[k] = acc;
        if (dpre_colsum) atomicAdd(&dpre_colsum[k], csum);
        if (dpre_blocksum) dpre_blocksum[(long)blockIdx.x * K + k] = csum;   // [block, K]
    }
    if (threadIdx.x == 0) shd[K] = dbp;
    __syncthreads();
    for (int k = threadIdx.x; k < K; k += blockDim.x) atomicAdd(&dw[k], shd[k]);
    if (threadIdx.x == 0) atomicAdd(db, shd[K]);
}

// k_rowdot_bwd for fp32 rows with a saved GELU' and no aux-loss mode (the
// option scorer's score2, NOPT rows per block): float4 columns, the block's
// rows split over blockDim / (K/4) thread groups whose partial sums meet in
// shared memory.  K % 4 == 0, K / 4 <= blockDim.x <= 256, 16-byte aligned
// rows and vectors.
__global__ void k_rowdot_bwd_v4(float* d_pre, long ldd, const float* pre, long ldp,
                                const float* in, long ldi, const float* w, float* dw, float* db,
                                const float* dsrc, long ds_stride, int rows, int K,
                                int rows_per_block, float* dpre_colsum, float* dpre_blocksum) {
    __shared__ float4 part[2][256];
    const int t = threadIdx.x, nc4 = K >> 2, G = blockDim.x / nc4;
    const int grp = t / nc4, c = (t - grp * nc4) * 4;
    const int r0 = blockIdx.x * rows_per_block, r1 = min(rows, r0 + rows_per_block);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f), cs = acc;
    float dsum = 0.f;
    if (grp < G) {
        const float4 w4 = ld4(w + c);
        for (int r = r0 + grp; r < r1; r += G) {
            const float d = dsrc[(long)r * ds_stride];
            const float4 x = ld4(in + (long)r * ldi + c);
            const float4 p = ld4(pre + (long)r * ldp + c);
            acc = make_float4(acc.x + d * x.x, acc.y + d * x.y, acc.z + d * x.z, acc.w + d * x.w);
            const float4 v = make_float4(d * w4.x * p.x, d * w4.y * p.y, d * w4.z * p.z, d * w4.w * p.w);
            st4(d_pre + (long)r * ldd + c, v);
            cs = add4(cs, v);
            dsum += d;
        }
    }
    part[0][t] = acc;
    part[1][t] = cs;
    __syncthreads();
    if (t < nc4) {
        for (int g = 1; g < G; g++) {
            acc = add4(acc, part[0][g * nc4 + t]);
            cs = add4(cs, part[1][g * nc4 + t]);
        }
        red_add4(dw + c, acc);
        if (dpre_colsum) red_add4(dpre_colsum + c, cs);
        if (dpre_blocksum) st4(dpre_blocksum + (long)blockIdx.x * K + c, cs);
    }
    if (c == 0 && grp < G && dsum != 0.f) atomicAdd(db, dsum);
}

// ------------------------------------------------------------ critic
// oracle tokens [card_vec(id) | is_hand, is_split, is_prize, f3, f4, f5] and
// critic keep [1, keep(LSEQ), id > 0] (k_otok_in, ptcg_model.cu:442-490)
// One warp per oracle token: lanes 0..31 move the 128-float card vector as
// float4s, lanes 0..5 the six trailing columns
template <typename T>
__global__ void k_otok_in(T* out, long ldo, uint8_t* ckeep, const float* obs, ObsLayout L,
                          const float* cv, const uint8_t* keep, int R) {
    const int NO = 56;
    const int lcrit = 1 + L.lseq + NO;
    const long nk = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (nk >= (long)R * NO) return;
    const int n = (int)(nk / NO), k = (int)(nk - (long)n * NO);
    const float* o = obs + (long)n * L.obs + L.orc;
    float idf, f3 = 0.f, f4 = 0.f, f5 = 0.f;
    int kind;
    if (k < 24) { kind = 0; idf = o[k * 2]; f3 = o[k * 2 + 1]; }
    else if (k < 48) { kind = 1; int s = k - 24; idf = o[48 + s * 3]; f4 = o[49 + s * 3]; f5 = o[50 + s * 3]; }
    else { kind = 2; int s = k - 48; idf = o[120 + s * 2]; f3 = o[121 + s * 2]; }
    T* orow = out + nk * ldo;
    st4(orow + lane * 4, ld4(cv + (long)id_clamp(idf, L.nc) * 128 + lane * 4));
    if (lane < 6) {
        const int c = 128 + lane;
        const float v = c < 131 ? ((c - 128) == kind ? 1.f : 0.f) : c == 131 ? f3 : c == 132 ? f4 : f5;
        st(&orow[c], v);
    }
    uint8_t* ck = ckeep + (long)n * lcrit;
    if (k == 0) {
        if (lane == 0) ck[0] = 1;
        for (int l = lane; l < L.lseq; l += 32) ck[1 + l] = keep[(long)n * L.lseq + l];
    }
    if (lane == 0) ck[1 + L.lseq + k] = (int)idf > 0;
}

// d card_vec rows += the card-vector columns of the oracle-token input
// gradient (g: [R * 56, >= 128], 16-byte rows); one thread per 4 columns,
// vector reductions
__global__ void k_otok_bwd(float* d_cv, const float* g, long ldg, const float* obs,
                           ObsLayout L, int R) {
    const int NO = 56;
    long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i >= (long)R * NO * 32) return;
    const int c = (int)(i & 31) * 4;
    const long nk = i >> 5;
    const int k = (int)(nk % NO), n = (int)(nk / NO);
    const float4 v = ld4(g + nk * ldg + c);
    if (!nz4(v)) return;
    const float* o = obs + (long)n * L.obs + L.orc;
    float idf = k < 24 ? o[k * 2] : k < 48 ? o[48 + (k - 24) * 3] : o[120 + (k - 48) * 2];
    red_add4(&d_cv[(long)id_clamp(idf, L.nc) * 128 + c], v);
}

// critic sequence rows 0 (critic readout) and 1..LSEQ (trunk output h);
// rows 1+LSEQ.. are written by the oracle_proj GEMM (row remap)
__global__ void k_xc_fill(float* xc, const float* h, const float* cread, int lseq,
                          int lcrit, int D, int R, const int* ext = nullptr) {
    long r = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);   // warp per row
    const int lane = threadIdx.x & 31;
    if (r >= (long)R * (1 + lseq)) return;
    const int n = (int)(r / (1 + lseq)), l = (int)(r - (long)n * (1 + lseq));
    // trunk rows past the extent are masked critic keys: left as they are
    // (finite), since they contribute nothing
    if (ext && l > 0 && l - 1 >= ext[n]) return;
    const float* src = l == 0 ? cread : h + ((long)n * lseq + l - 1) * D;
    float* dst = xc + ((long)n * lcrit + l) * D;
    for (int c = lane * 4; c < D; c += 128) st4(dst + c, ld4(src + c));
}

// [seq[n, 0] | g]  (k_val_in, ptcg_model.cu:500-506) in f32 and optional T copy
template <typename T>
__global__ void k_val_in(float* out, T* outc, long ldc, const float* seq, int seqlen, int D,
                         const float* gd, int R) {
    int W = D + 128;
    long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i >= (long)R * W) return;
    int n = (int)(i / W), c = (int)(i % W);
    float v = c < D ? seq[(long)n * seqlen * D + c] : gd[(long)n * 192 + (c - D)];
    out[i] = v;
    if (outc) st(&outc[(long)n * ldc + c], v);
}

// d [seq0 | g] -> d_seq[n, 0] += , d_gd[n, :128] +=
__global__ void k_val_in_bwd(float* d_seq, int seqlen, int D, float* d_gd, const float* g,
                             int R, int accum_seq) {
    int W = D + 128;
    long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i >= (long)R * W) return;
    int n = (int)(i / W), c = (int)(i % W);
    float v = g[i];
    if (c < D) {
        float* p = &d_seq[(long)n * seqlen * D + c];
        *p = accum_seq ? *p + v : v;
    } else d_gd[(long)n * 192 + (c - D)] += v;
}

// dst[n * seq_stride + c] += src[n * D + c]: the readout-row residual grad
// of a block computed on its first row only
__global__ void k_add_rows(float* dst, long seq_stride, const float* src, int R, int D) {
    long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i >= (long)R * D) return;
    int n = (int)(i / D), c = (int)(i % D);
    dst[(long)n * seq_stride + c] += src[i];
}

// critic input grad split: row 0 -> d_creadout, rows 1..LSEQ -> d_h +=,
// rows 1+LSEQ.. -> d_otok (T, compact) (k_xc_bwd, ptcg_model2.cu:174-187)
template <typename T>
__global__ void k_xc_bwd(T* d_otok, float* d_h, const float* dxc, int lseq, int lcrit, int D,
                         int R, const int* ext = nullptr) {
    // rows 1..lcrit-1 of every sample, warp per row (row 0 -> d_creadout is
    // a column sum over samples, done separately).  The first writer of d_h:
    // every trunk row is stored (no read-modify-write, no prior zeroing);
    // rows past the extent are masked keys with a zero gradient, stored as
    // zeros without reading
    long r = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (r >= (long)R * (lcrit - 1)) return;
    const int n = (int)(r / (lcrit - 1)), l = 1 + (int)(r - (long)n * (lcrit - 1));
    const float* g = dxc + ((long)n * lcrit + l) * D;
    if (l <= lseq) {
        float* dh = d_h + ((long)n * lseq + l - 1) * D;
        if (ext && l - 1 >= ext[n]) {
            for (int c = lane * 4; c < D; c += 128) st4(dh + c, make_float4(0.f, 0.f, 0.f, 0.f));
            return;
        }
        for (int c = lane * 4; c < D; c += 128) st4(dh + c, ld4(g + c));
    } else {
        T* o = d_otok + ((long)n * 56 + (l - 1 - lseq)) * D;
        for (int c = lane * 4; c < D; c += 128) st4(o + c, ld4(g + c));
    }
}

// trunk input grad split: rows 1.. -> d_tokp (T, compact); d_bc[n] = sum
// over token rows (one block per sample, no atomics); row 0 -> d_readout is
// a column sum over samples, done separately
template <typename T>
__global__ void k_x0_bwd(T* d_tokp, float* d_bc, const float* dx0, int ltok, int D,
                         const int* ext = nullptr) {
    // one block (8 warps) per sample: warp w takes token rows w, w + 8, ..;
    // each lane 4 consecutive columns of every 128 (float4 loads); rows past
    // the extent carry a zero gradient and are written as zeros unread.  D is
    // a multiple of 4 and at most 512.
    __shared__ float part[8][512];
    const int n = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int lseq = ltok + 1;
    const int e = ext ? ext[n] : lseq;
    float4 acc[4];
    #pragma unroll
    for (int k = 0; k < 4; k++) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int l = 1 + warp; l < lseq; l += 8) {
        T* o = d_tokp + ((long)n * ltok + l - 1) * D;
        const float* g = dx0 + ((long)n * lseq + l) * D;
        #pragma unroll
        for (int k = 0; k < 4; k++) {
            const int c = k * 128 + lane * 4;
            if (c >= D) break;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (l < e) v = ld4(g + c);
            st4(o + c, v);
            acc[k] = add4(acc[k], v);
        }
    }
    #pragma unroll
    for (int k = 0; k < 4; k++)
        if (k * 128 + lane * 4 < D) st4(&part[warp][k * 128 + lane * 4], acc[k]);
    __syncthreads();
    for (int c = threadIdx.x; c < D; c += blockDim.x) {
        float v = 0.f;
        #pragma unroll
        for (int w = 0; w < 8; w++) v += part[w][c];
        d_bc[(long)n * D + c] = v;
    }
}

__global__ void k_tok_cat_bwd(float* d_cv, float* d_zemb, float* d_oemb, const float* g,
                              long ldg, const float* obs, ObsLayout L, int R, int tok_in,
                              const int* ext = nullptr) {
    // warp per token row, grid-stride; the zone (16 x 8) and owner (4 x 4)
    // embedding grads, which every token hits, accumulate in shared memory
    // and leave with one atomic per entry per block
    __shared__ float sz[16 * 8], so[4 * 4];
    for (int i = threadIdx.x; i < 16 * 8; i += blockDim.x) sz[i] = 0.f;
    if (threadIdx.x < 16) so[threadIdx.x] = 0.f;
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const long nrows = (long)R * L.ltok;
    const bool vec = (ldg & 3) == 0;
    for (long nl = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); nl < nrows;
         nl += (long)gridDim.x * (blockDim.x >> 5)) {
        const int n = (int)(nl / L.ltok), l = (int)(nl - (long)n * L.ltok);
        if (ext && l + 1 >= ext[n]) continue;   // zero gradient past the extent
        const float* ti = obs + (long)n * L.obs + L.toki + l * 5;
        const float* gr = g + nl * ldg;
        float* c0 = d_cv + (long)id_clamp(ti[0], L.nc) * 128;
        const int t0 = (int)ti[3], t1 = (int)ti[4];
        float* ca = t0 > 0 ? d_cv + (long)(t0 >= L.nc ? L.nc - 1 : t0) * 128 : nullptr;
        float* cb = t1 > 0 ? d_cv + (long)(t1 >= L.nc ? L.nc - 1 : t1) * 128 : nullptr;
        for (int c = lane * 4; c < 256; c += 128) {
            float4 v = vec ? ld4(gr + c) : make_float4(gr[c], gr[c + 1], gr[c + 2], gr[c + 3]);
            if (!nz4(v)) continue;
            if (c < 128) red_add4(c0 + c, v);
            else {
                if (ca) red_add4(ca + (c - 128), v);
                if (cb) red_add4(cb + (c - 128), v);
            }
        }
        if (lane < 12) {
            float v = gr[256 + L.tok_f + lane];
            if (v != 0.f) {
                if (lane < 8) atomicAdd(&sz[id_clamp(ti[1], 16) * 8 + lane], v);
                else atomicAdd(&so[id_clamp(ti[2], 4) * 4 + (lane - 8)], v);
            }
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < 16 * 8; i += blockDim.x) if (sz[i] != 0.f) atomicAdd(&d_zemb[i], sz[i]);
    if (threadIdx.x < 16 && so[threadIdx.x] != 0.f) atomicAdd(&d_oemb[threadIdx.x], so[threadIdx.x]);
}

// ------------------------------------------------------------ aux losses
// opp-hand count MSE on softplus (ptcg_model2.cu:219-249): one block per row;
// targets built in shared memory (ids 0 < id < NC, id != UNK, count != 0).
template <typename TO>
__global__ void k_hand_grad(TO* d_lin, long ldd, float* lin, long ldl,
                            const float* obs, ObsLayout L, float scale, float* loss) {
    extern __shared__ float tg[];
    int n = blockIdx.x;
    for (int c = threadIdx.x; c < L.nc; c += blockDim.x) tg[c] = 0.f;
    __syncthreads();
    const float* o = obs + (long)n * L.obs + L.orc;
    if (threadIdx.x < 24) {
        int k = threadIdx.x;
        int id = (int)o[k * 2];
        float cnt = o[k * 2 + 1] * 4.0f;
        if (id > 0 && id < L.nc && id != L.nc - 1 && cnt != 0.f) atomicAdd(&tg[id], cnt);
    }
    __syncthreads();
    float lsum = 0.f;
    for (int c = threadIdx.x; c < L.nc; c += blockDim.x) {
        float x = lin[(long)n * ldl + c];
        float pred = softplus_f(x);
        float e = pred - tg[c];
        lsum += e * e;
        float g = scale * 2.f * e;
        g = x > 20.f ? g : g * sigmoid_f(x);
        st(&d_lin[(long)n * ldd + c], g);
        lin[(long)n * ldl + c] = g;             // fp32 copy (bias grad), logits no longer needed
    }
    lsum = warp_sum(lsum);
    if ((threadIdx.x & 31) == 0) atomicAdd(loss, lsum * scale);
}

// number of MY_UNSEEN tokens (prize-loss normaliser, ptcg_model2.cu:251-267)
__global__ void k_count_unseen(float* cnt, const float* obs, ObsLayout L, int R) {
    float s = 0.f;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < (long)R * L.ltok;
         i += (long)gridDim.x * blockDim.x) {
        long n = i / L.ltok;
        int l = (int)(i % L.ltok);
        if ((int)obs[n * L.obs + L.toki + l * 5 + 1] == 9) s += 1.f;
    }
    s = warp_sum(s);
    if ((threadIdx.x & 31) == 0) atomicAdd(cnt, s);
}

// prize BCE grad over MY_UNSEEN tokens + aux_prize head backward
// (k_prize_grad / k_prize_head_bwd, ptcg_model2.cu:269-281, ptcg_model3.cu:425-438).
// One warp per token; target = my-prize indicator of the token's card.
__global__ void k_prize_bwd(float* d_h, float* dw, float* db, const float* logit,
                            const float* h, const float* w, const float* obs, ObsLayout L,
                            const float* cnt_dev, float cnt_host, int D, int R, float* loss) {
    // warp per token, grid-stride.  dw (D), db and the loss accumulate in
    // shared memory (every counted token hits them); each token's d_h row
    // belongs to this warp alone, so it is a plain add.
    extern __shared__ float sp[];               // [D] dw, [1] db, [1] loss
    for (int i = threadIdx.x; i < D + 2; i += blockDim.x) sp[i] = 0.f;
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const float c = cnt_host > 0.f ? cnt_host : (cnt_dev[0] > 0.f ? cnt_dev[0] : 1.f);
    for (int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < R * L.ltok;
         t += gridDim.x * (blockDim.x >> 5)) {
        int n = t / L.ltok, l = t % L.ltok;
        const float* row = obs + (long)n * L.obs;
        if ((int)row[L.toki + l * 5 + 1] != 9) continue;
        int cid = id_clamp(row[L.toki + l * 5], L.nc);
        float tgt = 0.f;
        const float* o = row + L.orc;
        for (int k = 0; k < 8; k++) {
            int id = (int)o[120 + 2 * k];
            if (id > 0 && id < L.nc && o[121 + 2 * k] > 0.f && id == cid) tgt = 1.f;
        }
        float x = logit[t];
        float g = 0.1f * (sigmoid_f(x) - tgt) / c;
        if (lane == 0) {
            float bce = fmaxf(x, 0.f) - x * tgt + log1pf(expf(-fabsf(x)));
            atomicAdd(&sp[D + 1], 0.1f * bce / c);
            atomicAdd(&sp[D], g);
        }
        long hr = ((long)n * L.lseq + 1 + l) * D;
        for (int d = lane; d < D; d += 32) {
            d_h[hr + d] += g * w[d];
            atomicAdd(&sp[d], g * h[hr + d]);
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < D; i += blockDim.x) if (sp[i] != 0.f) atomicAdd(&dw[i], sp[i]);
    if (threadIdx.x == 0) {
        if (sp[D] != 0.f) atomicAdd(db, sp[D]);
        if (sp[D + 1] != 0.f) atomicAdd(loss, sp[D + 1]);
    }
}

// ---------------------------------------------------------- misc helpers
template <typename TI>
__global__ void k_colsum(float* out, const TI* in, long ld, int rows, int cols,
                         int rows_per_block) {
    int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= cols) return;
    int r0 = blockIdx.y * rows_per_block, r1 = min(rows, r0 + rows_per_block);
    float s = 0.f;
    for (int r = r0; r < r1; r++) s += to_f<TI>(in[(long)r * ld + c]);
    atomicAdd(&out[c], s);
}

// out[c] += sum over groups g, rows r < rows_per_group of
//           src[(g * group_stride + row_off + r) * ld + c]
__global__ void k_colsum_groups(float* out, const float* src, long ld, int ngroups,
                                int group_stride, int row_off, int rows_per_group, int cols,
                                int groups_per_block) {
    int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= cols) return;
    int g0 = blockIdx.y * groups_per_block, g1 = min(ngroups, g0 + groups_per_block);
    float s = 0.f;
    for (int g = g0; g < g1; g++) {
        const float* b = src + ((long)g * group_stride + row_off) * ld + c;
        for (int r = 0; r < rows_per_group; r++) s += b[(long)r * ld];
    }
    atomicAdd(&out[c], s);
}

// out[c] += sum over the rows {g * group_stride + row_off + r : g < ngroups,
// r < rows_per_group} of src[row * ld + c]: warp per row (grid-stride), each
// lane owning 4 consecutive columns of every 128 (float4 loads, NC chunks:
// cols = 128 NC), per-block sums in shared memory, one atomic per column per
// block
template <int NC>
__global__ void k_colsum_rowset(float* out, const float* src, long ld, int ngroups,
                                int group_stride, int row_off, int rows_per_group) {
    __shared__ float part[8][128 * NC];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float4 acc[NC];
    #pragma unroll
    for (int k = 0; k < NC; k++) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    const long nrows = (long)ngroups * rows_per_group;
    for (long i = (long)blockIdx.x * 8 + warp; i < nrows; i += (long)gridDim.x * 8) {
        const int g = (int)(i / rows_per_group), r = (int)(i - (long)g * rows_per_group);
        const float* row = src + ((long)g * group_stride + row_off + r) * ld;
        #pragma unroll
        for (int k = 0; k < NC; k++) acc[k] = add4(acc[k], ld4(row + k * 128 + lane * 4));
    }
    #pragma unroll
    for (int k = 0; k < NC; k++) st4(&part[warp][k * 128 + lane * 4], acc[k]);
    __syncthreads();
    for (int c = threadIdx.x; c < 128 * NC; c += blockDim.x) {
        float v = 0.f;
        #pragma unroll
        for (int w = 0; w < 8; w++) v += part[w][c];
        if (v != 0.f) atomicAdd(&out[c], v);
    }
}

// dst[r, c] += src[r * lds + off + c]
__global__ void k_slice_add(float* dst, const float* src, int rows, int width, long lds,
                            int off) {
    long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i >= (long)rows * width) return;
    int r = (int)(i / width), c = (int)(i % width);
    dst[i] += src[(long)r * lds + off + c];
}

__global__ void k_scale_copy(float* dst, long ldd, const float* src, long lds, int rows,
                             int cols, float scale) {
    long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i >= (long)rows * cols) return;
    int r = (int)(i / cols), c = (int)(i % cols);
    dst[(long)r * ldd + c] = src[(long)r * lds + c] * scale;
}

template <typename T>
__global__ void k_cast(T* dst, long ldd, const float* src, long lds, int rows, int cols) {
    long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i >= (long)rows * cols) return;
    int r = (int)(i / cols), c = (int)(i % cols);
    st(&dst[(long)r * ldd + c], src[(long)r * lds + c]);
}

// ------------------------------------------------------------ PPO loss
// advantage mean / unbiased variance over the minibatch (ppo_var_mean,
// pufferlib.cu:1307-1363), one block, fp64 accumulation.
__global__ void k_adv_stats(float* out, const float* adv, int n) {
    __shared__ double sh[32];
    double s = 0.0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) s += adv[i];
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0; for (int i = 0; i < (int)(blockDim.x >> 5); i++) t += sh[i];
        sh[31] = t / n;
    }
    __syncthreads();
    double mean = sh[31];
    __syncthreads();
    double v = 0.0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) { double d = adv[i] - mean; v += d * d; }
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0; for (int i = 0; i < (int)(blockDim.x >> 5); i++) t += sh[i];
        out[0] = (float)mean;
        out[1] = (float)(t / (n > 1 ? n - 1 : 1));
    }
}

// Fused clipped PPO + clipped value loss + entropy, forward and backward,
// one warp per row (ppo_loss_compute, pufferlib.cu:1010-1248).  Masked
// logits are -1e4.  Writes the gradient w.r.t. the fused decoder output
// [scores | value] and 7 per-block partial stats.
constexpr int PPO_ROWS_PER_BLOCK = 8;
__global__ void k_ppo_loss(const float* dec, int nopt, const float* mask, long mstride,
                           const float* actions, const float* old_logp, const float* adv,
                           const float* values, const float* returns, const float* prio,
                           int horizon, int row0, int nt, int nt_norm, const float* adv_stats,
                           float clip, float vclip, float vf_coef, float ent_coef,
                           float* grad, float* new_logp, float* ratio_out, float* partials) {
    __shared__ float sp[PPO_ROWS_PER_BLOCK][8];
    int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int r = blockIdx.x * PPO_ROWS_PER_BLOCK + wid;
    float st7[7] = {0, 0, 0, 0, 0, 0, 0};
    if (r < nt) {
        const int W = nopt + 1;
        const float inv = 1.f / (float)nt_norm;
        const float* lg = dec + (long)r * W;
        const float* mk = mask + (long)r * mstride;
        int act = (int)actions[r];
        float mx = -INFINITY;
        for (int a = lane; a < nopt; a += 32) {
            float l = mk[a] == 0.f ? -1e4f : lg[a];
            mx = fmaxf(mx, l);
        }
        mx = warp_max(mx);
        float se = 0.f;
        for (int a = lane; a < nopt; a += 32) {
            float l = mk[a] == 0.f ? -1e4f : lg[a];
            se += expf(l - mx);
        }
        se = warp_sum(se);
        float lse = mx + logf(se);
        float ent = 0.f;
        for (int a = lane; a < nopt; a += 32) {
            float l = mk[a] == 0.f ? -1e4f : lg[a];
            float lp = l - lse;
            ent -= expf(lp) * lp;
        }
        ent = warp_sum(ent);
        float act_l = (act >= 0 && act < nopt) ? (mk[act] == 0.f ? -1e4f : lg[act]) : -1e4f;
        float logp = act_l - lse;
        float mean = adv_stats[0], var = adv_stats[1];
        float advn = (adv[r] - mean) / (sqrtf(var) + 1e-8f);
        float w = prio[(row0 + r) / horizon];
        float val = values[r], ret = returns[r], vp = lg[nopt];
        float verr = vp - val;
        float vcl = val + fmaxf(-vclip, fminf(vclip, verr));
        float lu = (vp - ret) * (vp - ret), lc = (vcl - ret) * (vcl - ret);
        float vloss = 0.5f * fmaxf(lu, lc);
        float dv;
        if (lc > lu) dv = (verr >= -vclip && verr <= vclip) ? vcl - ret : 0.f;
        else dv = vp - ret;
        float logratio = logp - old_logp[r];
        float ratio = expf(logratio);
        float rc = fmaxf(1.f - clip, fminf(1.f + clip, ratio));
        float wa = -w * advn;
        float pg1 = wa * ratio, pg2 = wa * rc;
        float pg = fmaxf(pg1, pg2);
        float dr = wa * inv;
        if (pg2 > pg1 && (ratio <= 1.f - clip || ratio >= 1.f + clip)) dr = 0.f;
        float dnlp = dr * ratio;
        float dent = inv * (-ent_coef);
        float* gr = grad + (long)r * W;
        for (int a = lane; a < nopt; a += 32) {
            float g = 0.f;
            if (mk[a] != 0.f) {
                float lp = lg[a] - lse;
                float p = expf(lp);
                g = (a == act ? dnlp : 0.f) - p * dnlp + dent * p * (-ent - lp);
            }
            gr[a] = g;
        }
        if (lane == 0) {
            gr[nopt] = inv * vf_coef * dv;
            new_logp[r] = logp;
            ratio_out[r] = ratio;
        }
        st7[0] = (pg + vf_coef * vloss - ent_coef * ent) * inv;
        st7[1] = pg * inv;
        st7[2] = vloss * inv;
        st7[3] = ent * inv;
        st7[4] = -logratio * inv;
        st7[5] = ((ratio - 1.f) - logratio) * inv;
        st7[6] = (fabsf(ratio - 1.f) > clip ? 1.f : 0.f) * inv;
    }
    if (lane == 0) for (int k = 0; k < 7; k++) sp[wid][k] = st7[k];
    __syncthreads();
    if (threadIdx.x < 7) {
        float s = 0.f;
        for (int w2 = 0; w2 < PPO_ROWS_PER_BLOCK; w2++) s += sp[w2][threadIdx.x];
        partials[(long)blockIdx.x * 7 + threadIdx.x] = s;
    }
}

// deterministic reduction of the block partials (ppo_loss_reduce,
// pufferlib.cu:1254-1284); stats[7] = advantage variance
__global__ void k_ppo_reduce(float* stats, const float* partials, int nblocks,
                             const float* adv_stats, int accumulate) {
    int c = threadIdx.x;
    if (c < 7) {
        double s = 0.0;
        for (int b = 0; b < nblocks; b++) s += partials[(long)b * 7 + c];
        stats[c] = accumulate ? stats[c] + (float)s : (float)s;
    }
    if (c == 7) stats[7] = adv_stats[1];
}

// ------------------------------------------------------------ sampler
// masked online log-sum-exp, inverse-CDF draw, fallback to the last legal
// slot, logprob, value copy (sample_logits, pufferlib.cu:584-718); one warp per row.
__global__ void k_sample(const float* dec, int n, int nopt, const float* mask, long mstride,
                         const float* uni, float* actions, float* logprobs, float* values) {
    int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    int lane = threadIdx.x & 31;
    if (r >= n) return;
    const float* lg = dec + (long)r * (nopt + 1);
    const float* mk = mask + (long)r * mstride;
    float mx = -INFINITY;
    for (int a = lane; a < nopt; a += 32) mx = fmaxf(mx, mk[a] == 0.f ? -1e4f : lg[a]);
    mx = warp_max(mx);
    float se = 0.f;
    for (int a = lane; a < nopt; a += 32) se += expf((mk[a] == 0.f ? -1e4f : lg[a]) - mx);
    se = warp_sum(se);
    float lse = mx + logf(se);
    if (lane == 0) {
        float u = uni[r], cum = 0.f;
        int pick = -1;
        for (int a = 0; a < nopt; a++) {
            float l = mk[a] == 0.f ? -1e4f : lg[a];
            cum += expf(l - lse);
            if (u < cum) { pick = a; break; }
        }
        if (pick < 0) {
            pick = nopt - 1;
            for (int a = nopt - 1; a >= 0; a--) if (mk[a] != 0.f) { pick = a; break; }
        }
        float l = mk[pick] == 0.f ? -1e4f : lg[pick];
        actions[r] = (float)pick;
        logprobs[r] = l - lse;
        values[r] = lg[nopt];
    }
}

// The rollout forward's last step with the sampler fused in (one warp per
// row): the fused output row [scores | value] (scores from the contiguous
// staging buffer, value = dot(v1 row, w2) + b2 in k_rowdot's order), then
// k_sample's draw on those values: masked (-1e4) log-sum-exp, inverse CDF
// on the caller's uniform, fallback to the last legal slot, logprob, value.
// Bit-identical to the unfused output + k_sample.
__global__ void k_out_sample(float* out, const float* staged, int nopt, const float* v1,
                             const float* w2, const float* b2, int K, const float* mask,
                             long mstride, const float* uni, float* actions, float* logprobs,
                             float* values, int n) {
    int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    int lane = threadIdx.x & 31;
    if (r >= n) return;
    const float* sc = staged + (long)r * nopt;
    float* o = out + (long)r * (nopt + 1);
    const float* x = v1 + (long)r * K;
    float v = 0.f;
    for (int k = lane; k < K; k += 32) v += x[k] * w2[k];
    v = warp_sum(v) + b2[0];
    const float* mk = mask + (long)r * mstride;
    float mx = -INFINITY;
    for (int a = lane; a < nopt; a += 32) {
        const float l = sc[a];
        o[a] = l;
        mx = fmaxf(mx, mk[a] == 0.f ? -1e4f : l);
    }
    mx = warp_max(mx);
    float se = 0.f;
    for (int a = lane; a < nopt; a += 32) se += expf((mk[a] == 0.f ? -1e4f : sc[a]) - mx);
    se = warp_sum(se);
    const float lse = mx + logf(se);
    if (lane == 0) {
        o[nopt] = v;
        float u = uni[r], cum = 0.f;
        int pick = -1;
        for (int a = 0; a < nopt; a++) {
            float l = mk[a] == 0.f ? -1e4f : sc[a];
            cum += expf(l - lse);
            if (u < cum) { pick = a; break; }
        }
        if (pick < 0) {
            pick = nopt - 1;
            for (int a = nopt - 1; a >= 0; a--) if (mk[a] != 0.f) { pick = a; break; }
        }
        float l = mk[pick] == 0.f ? -1e4f : sc[pick];
        actions[r] = (float)pick;
        logprobs[r] = l - lse;
        values[r] = v;
    }
}

// ------------------------------------------------------ compact observations
// An observation row in transfer form: the id fields as int16, then the
// float fields as fp32 (ptcg_obs_pack / ptcg_obs_unpack).  Each part is a
// list of strided runs of the fp32 row: run k covers count[k] values at
// row offsets dst[k] + e * stride[k], in the packed order.
constexpr int OBS_RUNS = 8;
struct ObsRuns {
    int n;
    int dst[OBS_RUNS], count[OBS_RUNS], stride[OBS_RUNS];
};
struct ObsPacking {
    ObsRuns ints, floats;
    int obs;                 // fp32 row length
    long row_bytes;          // packed row bytes (16-byte multiple)
    long float_off;          // byte offset of the fp32 part in a packed row
};

// one block per packed row: expand it into the fp32 row layout
__global__ void k_obs_unpack(float* rows, const uint8_t* packed, ObsPacking pk, long n) {
    const long r = blockIdx.x;
    if (r >= n) return;
    const int16_t* iv = (const int16_t*)(packed + r * pk.row_bytes);
    const float* fv = (const float*)(packed + r * pk.row_bytes + pk.float_off);
    float* out = rows + r * pk.obs;
    int base = 0;
    for (int k = 0; k < pk.ints.n; k++) {
        const int c = pk.ints.count[k], d = pk.ints.dst[k], st = pk.ints.stride[k];
        for (int e = threadIdx.x; e < c; e += blockDim.x) out[d + e * st] = (float)iv[base + e];
        base += c;
    }
    base = 0;
    for (int k = 0; k < pk.floats.n; k++) {
        const int c = pk.floats.count[k], d = pk.floats.dst[k], st = pk.floats.stride[k];
        for (int e = threadIdx.x; e < c; e += blockDim.x) out[d + e * st] = fv[base + e];
        base += c;
    }
}

// seat-flipping GAE / V-trace (k_negamax_adv, ptcg_model2.cu:288-311)
__global__ void k_negamax_adv(const float* values, const float* rewards, const float* dones,
                              const float* imp, const float* obs, long obs_size, int seat_col,
                              float* adv, float gamma, float lambda, float rho_clip,
                              float c_clip, int B, int T) {
    int row = blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= B) return;
    long o = (long)row * T;
    const float* ob = obs + (long)row * T * obs_size;
    float last = 0.f;
    for (int t = T - 2; t >= 0; t--) {
        float st_ = ob[(long)t * obs_size + seat_col];
        float sn = ob[(long)(t + 1) * obs_size + seat_col];
        float sign = st_ == sn ? 1.f : -1.f;
        float s = sign * (1.f - dones[o + t + 1]);
        float im = imp[o + t];
        float rho = im < rho_clip ? im : rho_clip;
        float cc = im < c_clip ? im : c_clip;
        float delta = rho * (rewards[o + t + 1] + gamma * values[o + t + 1] * s - values[o + t]);
        last = delta + gamma * lambda * cc * s * last;
        adv[o + t] = last;
    }
}

// ------------------------------------------------------------ Adam
// pass 1: per-block partial sum of squares (fp64 accumulation); g is
// 16-byte aligned (arena tensors start on 16 bytes), n is any length
__global__ void k_sumsq(double* partials, const float* g, long n) {
    __shared__ double sh[32];
    double s = 0.0;
    const float4* g4 = reinterpret_cast<const float4*>(g);
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < (n >> 2);
         i += (long)gridDim.x * blockDim.x) {
        float4 v = g4[i];
        s += (double)v.x * v.x + (double)v.y * v.y + (double)v.z * v.z + (double)v.w * v.w;
    }
    if (blockIdx.x == 0 && threadIdx.x < (n & 3)) {
        double v = g[(n & ~3L) + threadIdx.x];
        s += v * v;
    }
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0; for (int i = 0; i < (int)(blockDim.x >> 5); i++) t += sh[i];
        partials[blockIdx.x] = t;
    }
}

// A weight matrix whose bf16 compute copy the Adam pass refreshes.
struct BfCopy { long off, n; int cols, ldp; bf16* dst; };

// pass 2: every block re-reduces the partials (deterministic), then
// clip coef = min(1, max_norm / (norm + 1e-6)) (clip_grad_norm_), torch Adam:
//   m = b1 m + (1-b1) g; v = b2 v + (1-b2) g^2;
//   p -= (lr / (1-b1^t)) * m / (sqrt(v) / sqrt(1-b2^t) + eps)
// skipped (no state change) when the gate is 0 or the norm is not finite.
__global__ void k_adam(float* p, float* m, float* v, const float* g, long n,
                       const double* partials, int nparts, float lr, float b1, float b2,
                       float eps, float max_norm, const long long* step_dev,
                       const float* gate, float* stats, const BfCopy* copies, int ncopies,
                       const int* chunk_copy, int chunk) {
    __shared__ float s_coef, s_bc1, s_bc2sqrt;
    __shared__ int s_ok;
    __shared__ double s_red[32];
    // every block re-reduces the partials in the same fixed order
    // (deterministic, identical on every block)
    double tp = 0.0;
    for (int i = threadIdx.x; i < nparts; i += blockDim.x) tp += partials[i];
    for (int o = 16; o > 0; o >>= 1) tp += __shfl_xor_sync(0xffffffffu, tp, o);
    if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = tp;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t_step = (double)(step_dev[0] + 1);
        s_bc1 = (float)(1.0 - pow((double)b1, t_step));
        s_bc2sqrt = (float)sqrt(1.0 - pow((double)b2, t_step));
        double t = 0.0;
        for (int i = 0; i < (int)(blockDim.x >> 5); i++) t += s_red[i];
        float norm = (float)sqrt(t);
        int ok = isfinite(norm) && (gate == nullptr || gate[0] != 0.f);
        float coef = max_norm / (norm + 1e-6f);
        s_coef = coef < 1.f ? coef : 1.f;
        s_ok = ok;
        if (blockIdx.x == 0 && stats) { stats[0] = norm; stats[1] = ok ? 1.f : 0.f; }
    }
    __syncthreads();
    if (!s_ok) return;
    float coef = s_coef;
    float step_size = lr / s_bc1;
    float bc2sqrt = s_bc2sqrt;
    float4* p4 = reinterpret_cast<float4*>(p);
    float4* m4 = reinterpret_cast<float4*>(m);
    float4* v4 = reinterpret_cast<float4*>(v);
    const float4* g4 = reinterpret_cast<const float4*>(g);
    // float4 granules: n, chunk and every tensor offset are multiples of 4,
    // so a granule never straddles two tensors
    for (long c0 = (long)blockIdx.x * chunk; c0 < n; c0 += (long)gridDim.x * chunk) {
        // first bf16 copy that ends after the chunk start (copies sorted by off)
        int ci = chunk_copy ? chunk_copy[c0 / chunk] : ncopies;
        long c1 = min(n, c0 + chunk);
        for (long i = c0 + 4 * threadIdx.x; i < c1; i += 4 * blockDim.x) {
            float4 gg = g4[i >> 2], mm = m4[i >> 2], vv = v4[i >> 2], pp = p4[i >> 2];
            float gs[4] = {gg.x, gg.y, gg.z, gg.w}, ms[4] = {mm.x, mm.y, mm.z, mm.w};
            float vs[4] = {vv.x, vv.y, vv.z, vv.w}, ps[4] = {pp.x, pp.y, pp.z, pp.w};
            #pragma unroll
            for (int e = 0; e < 4; e++) {
                float gi = gs[e] * coef;
                ms[e] = b1 * ms[e] + (1.f - b1) * gi;
                vs[e] = b2 * vs[e] + (1.f - b2) * gi * gi;
                ps[e] = ps[e] - step_size * ms[e] / (sqrtf(vs[e]) / bc2sqrt + eps);
            }
            m4[i >> 2] = make_float4(ms[0], ms[1], ms[2], ms[3]);
            v4[i >> 2] = make_float4(vs[0], vs[1], vs[2], vs[3]);
            p4[i >> 2] = make_float4(ps[0], ps[1], ps[2], ps[3]);
            while (ci < ncopies && i >= copies[ci].off + copies[ci].n) ci++;
            if (ci < ncopies && i >= copies[ci].off) {
                const BfCopy& cp = copies[ci];
                long j = i - cp.off;
                if (cp.ldp == cp.cols) {            // contiguous copy: one 8-byte store
                    uint2 q;
                    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&q);
                    h[0] = __floats2bfloat162_rn(ps[0], ps[1]);
                    h[1] = __floats2bfloat162_rn(ps[2], ps[3]);
                    *reinterpret_cast<uint2*>(cp.dst + j) = q;
                } else {                            // padded pitch (rows of cols < ldp)
                    #pragma unroll
                    for (int e = 0; e < 4; e++) {
                        if (j + e >= cp.n) break;
                        int jj = (int)(j + e), r = jj / cp.cols;
                        cp.dst[(long)r * cp.ldp + (jj - r * cp.cols)] = __float2bfloat16_rn(ps[e]);
                    }
                }
            }
        }
    }
}

// fp64 sum of the partials of k_sumsq, in a fixed order, into out[0] (one block)
__global__ void k_sumsq_final(double* out, const double* partials, int nparts) {
    __shared__ double sh[32];
    double t = 0.0;
    for (int i = threadIdx.x; i < nparts; i += blockDim.x) t += partials[i];
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = t;
    __syncthreads();
    if (threadIdx.x == 0) {
        double s = 0.0;
        for (int i = 0; i < (int)(blockDim.x >> 5); i++) s += sh[i];
        out[0] = s;
    }
}

// The Adam update of k_adam over a list of arena segments whose gradients
// sit elsewhere (a rank's reduce-scattered shard): segment y = blockIdx.y
// covers arena floats [seg[3y], seg[3y] + seg[3y+2]) with gradients from
// gsrc + seg[3y+1].  The clip uses the global sum of squares sumsq[0] (all
// ranks' shards).  No bf16 copies here: the caller refreshes them once the
// updated weights are gathered.
__global__ void k_adam_seg(float* p, float* m, float* v, const float* gsrc, const long* seg,
                           const double* sumsq, float lr, float b1, float b2, float eps,
                           float max_norm, const long long* step_dev, const float* gate,
                           float* stats) {
    __shared__ float s_coef, s_step, s_bc2sqrt;
    __shared__ int s_ok;
    if (threadIdx.x == 0) {
        const double t_step = (double)(step_dev[0] + 1);
        const float norm = (float)sqrt(sumsq[0]);
        const int ok = isfinite(norm) && (gate == nullptr || gate[0] != 0.f);
        const float coef = max_norm / (norm + 1e-6f);
        s_coef = coef < 1.f ? coef : 1.f;
        s_step = lr / (float)(1.0 - pow((double)b1, t_step));
        s_bc2sqrt = (float)sqrt(1.0 - pow((double)b2, t_step));
        s_ok = ok;
        if (blockIdx.x == 0 && blockIdx.y == 0 && stats) { stats[0] = norm; stats[1] = ok ? 1.f : 0.f; }
    }
    __syncthreads();
    if (!s_ok) return;
    const long a = seg[3 * blockIdx.y], so = seg[3 * blockIdx.y + 1], len = seg[3 * blockIdx.y + 2];
    const float coef = s_coef, step_size = s_step, bc2sqrt = s_bc2sqrt;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < len;
         i += (long)gridDim.x * blockDim.x) {
        const float gi = gsrc[so + i] * coef;
        const float mi = b1 * m[a + i] + (1.f - b1) * gi;
        const float vi = b2 * v[a + i] + (1.f - b2) * gi * gi;
        m[a + i] = mi;
        v[a + i] = vi;
        p[a + i] = p[a + i] - step_size * mi / (sqrtf(vi) / bc2sqrt + eps);
    }
}

// advance the Adam step counter when the step was applied (after k_adam)
__global__ void k_step_inc(long long* step_dev, const float* stats) {
    if (stats[1] != 0.f) step_dev[0] += 1;
}

// Zero a workspace after a step whose gradient norm was not finite.  Rows
// past a sequence's extent keep whatever an earlier micro-batch left there,
// and the weight-gradient GEMMs multiply them by exact-zero gradients; one
// Inf / NaN kept in such a row would make 0 * Inf = NaN in every later
// weight gradient.  A finite norm makes this a one-load no-op per block.
__global__ void k_zero_if_nonfinite(const float* stats, uint4* base, long n16) {
    if (isfinite(stats[0])) return;
    const uint4 z = make_uint4(0u, 0u, 0u, 0u);
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n16;
         i += (long)gridDim.x * blockDim.x)
        base[i] = z;
}

__global__ void k_gelu_bwd(float* d, const float* pre, long n) {
    long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i < n) d[i] *= pre[i];                                    // saved GELU'
}

// refresh bf16 copies from the master weights (after a load)
__global__ void k_refresh_copies(const float* p, const BfCopy* copies, int ncopies) {
    const BfCopy& cp = copies[blockIdx.y];
    for (long j = blockIdx.x * (long)blockDim.x + threadIdx.x; j < cp.n;
         j += (long)gridDim.x * blockDim.x)
        cp.dst[(j / cp.cols) * cp.ldp + (j % cp.cols)] = __float2bfloat16_rn(p[cp.off + j]);
}

// 64-bit weight checksum: wrapping sums of the raw fp32 bit patterns, one
// weighted by position, so a swap of two values changes it
__global__ void k_checksum(unsigned int* out, const float* p, long n) {
    unsigned long long s1 = 0, s2 = 0;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n;
         i += (long)gridDim.x * blockDim.x) {
        unsigned int b = __float_as_uint(p[i]);
        s1 += b;
        s2 += (unsigned long long)b * (unsigned long long)(i + 1);
    }
    atomicAdd((unsigned long long*)out, s1 ^ (s2 << 1));
}

// ------------------------------------------------- prioritised replay
// (prio_replay_cuda, native/src/pufferlib.cu:1451-1591)
// w[b] = (sum_t |adv[b, t]|)^alpha (0 when not finite); one warp per segment,
// lane-strided partial sums then a shuffle-down tree, as the reference does
__global__ void k_prio_rowsum(float* w, const float* adv, int T, float alpha) {
    int b = blockIdx.x, lane = threadIdx.x;
    float s = 0.f;
    for (int t = lane; t < T; t += 32) s += fabsf(adv[(long)b * T + t]);
    for (int o = 16; o >= 1; o >>= 1) s += __shfl_down_sync(0xffffffffu, s, o);
    if (lane == 0) {
        float p = powf(s, alpha);
        w[b] = (isnan(p) || isinf(p)) ? 0.f : p;
    }
}
// probs = (w + eps) / (sum w + eps), eps = 1e-6 (one block)
__global__ void k_prio_normalize(float* w, int B) {
    __shared__ float sh[32];
    __shared__ float total;
    float s = 0.f;
    for (int i = threadIdx.x; i < B; i += blockDim.x) s += w[i];
    for (int o = 16; o >= 1; o >>= 1) s += __shfl_down_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.f;
        for (int o = 16; o >= 1; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
        if (threadIdx.x == 0) total = v + 1e-6f;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < B; i += blockDim.x) w[i] = (w[i] + 1e-6f) / total;
}
// inclusive running sum in index order (fp32, sequential like the reference)
__global__ void k_prio_cdf(float* cdf, const float* probs, int B) {
    if (threadIdx.x == 0 && blockIdx.x == 0) {
        float c = 0.f;
        for (int i = 0; i < B; i++) { c += probs[i]; cdf[i] = c; }
    }
}
// idx[i] = first b with cdf[b] >= u[i] (clamped to B-1);
// mb_prio[i] = (total_agents * probs[idx[i]])^(-beta)
__global__ void k_prio_sample(int* idx, float* mb_prio, const float* cdf, const float* probs,
                              const float* u, int B, int n, int total_agents, float beta) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float x = u[i];
    int lo = 0, hi = B - 1;
    while (lo < hi) {
        int mid = (lo + hi) / 2;
        if (cdf[mid] < x) lo = mid + 1;
        else hi = mid;
    }
    idx[i] = lo;
    mb_prio[i] = powf(probs[lo] * (float)total_agents, -beta);
}

// dst row i <- src row idx[i] (rows of row_floats, 16-byte aligned when
// row_floats % 4 == 0); gridDim.y = rows
__global__ void k_gather_rows(float* dst, const float* src, const int* idx, long row_floats) {
    long i = blockIdx.y;
    const float* s = src + (long)idx[i] * row_floats;
    float* d = dst + i * row_floats;
    if ((row_floats & 3) == 0) {
        for (long c = (blockIdx.x * (long)blockDim.x + threadIdx.x) * 4; c < row_floats;
             c += (long)gridDim.x * blockDim.x * 4)
            st4(d + c, ld4(s + c));
    } else {
        for (long c = blockIdx.x * (long)blockDim.x + threadIdx.x; c < row_floats;
             c += (long)gridDim.x * blockDim.x)
            d[c] = s[c];
    }
}
// dst row idx[i] <- src row i (index_copy, pufferlib.cu:2147-2160)
__global__ void k_scatter_rows(float* dst, const float* src, const int* idx, long row_floats) {
    long i = blockIdx.y;
    const float* s = src + i * row_floats;
    float* d = dst + (long)idx[i] * row_floats;
    for (long c = blockIdx.x * (long)blockDim.x + threadIdx.x; c < row_floats;
         c += (long)gridDim.x * blockDim.x)
        d[c] = s[c];
}
// returns = values + advantages of the selected segments (copy_values_adv_returns)
__global__ void k_add_rows_flat(float* out, const float* a, const float* b, long n) {
    long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i < n) out[i] = a[i] + b[i];
}

// ---------------------------------------------------------------- Muon
// (muon_step, native/src/muon.cu:209-297; the gate vetoes a step by
// returning before any state or weight is touched, muon.cu:54-60, 89-99)
// grads *= min(1, max_norm / (||g|| + 1e-6)) from the k_sumsq partials
__global__ void k_muon_clip(float* g, long n, const double* partials, int nparts, float max_norm,
                            float* stats) {
    __shared__ double s_red[32];
    __shared__ float s_coef;
    double tp = 0.0;
    for (int i = threadIdx.x; i < nparts; i += blockDim.x) tp += partials[i];
    for (int o = 16; o > 0; o >>= 1) tp += __shfl_xor_sync(0xffffffffu, tp, o);
    if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = tp;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int i = 0; i < (int)(blockDim.x >> 5); i++) t += s_red[i];
        float norm = (float)sqrt(t);
        s_coef = fminf(max_norm / (norm + 1e-6f), 1.f);
        if (blockIdx.x == 0 && stats) stats[0] = norm;
    }
    __syncthreads();
    float c = s_coef;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
        g[i] *= c;
}
// >= 2-D parameters: nesterov with a sum accumulator, m = mu m + g; g += mu m
__global__ void k_muon_nesterov(float* mb, float* g, const float* gate, float mu, long n) {
    if (gate && *gate == 0.f) return;
    long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i < n) {
        float m = mu * mb[i] + g[i];
        mb[i] = m;
        g[i] = g[i] + mu * m;
    }
}
// 1-D parameters: EMA momentum, m = mu m + (1 - mu) g; g += m
__global__ void k_muon_nesterov_ema(float* mb, float* g, const float* gate, float mu, long n) {
    if (gate && *gate == 0.f) return;
    long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i < n) {
        float gi = g[i];
        float m = mu * mb[i] + (1.f - mu) * gi;
        mb[i] = m;
        g[i] = gi + m;
    }
}
// x *= 1 / max(||x||, eps) with the norm from k_sumsq partials (one block)
__global__ void k_muon_normalize(float* x, long n, const double* partials, int nparts, float eps) {
    __shared__ double s_red[32];
    __shared__ float s_inv;
    double tp = 0.0;
    for (int i = threadIdx.x; i < nparts; i += blockDim.x) tp += partials[i];
    for (int o = 16; o > 0; o >>= 1) tp += __shfl_xor_sync(0xffffffffu, tp, o);
    if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = tp;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int i = 0; i < (int)(blockDim.x >> 5); i++) t += s_red[i];
        s_inv = 1.f / fmaxf((float)sqrt(t), eps);
    }
    __syncthreads();
    float inv = s_inv;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
        x[i] *= inv;
}
// y = a x (elementwise)
__global__ void k_scale_to(float* y, const float* x, float a, long n) {
    long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i < n) y[i] = a * x[i];
}
// w = w (1 - lr wd) - lr scale u
__global__ void k_muon_update(float* w, const float* u, float lr, const float* gate, float wd,
                              float scale, long n) {
    if (gate && *gate == 0.f) return;
    float wd_scale = 1.f - lr * wd;
    long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i < n) w[i] = w[i] * wd_scale - lr * scale * u[i];
}
__global__ void k_gate_stat(float* stats, const float* gate) {
    stats[1] = (gate && *gate == 0.f) ? 0.f : 1.f;
}
