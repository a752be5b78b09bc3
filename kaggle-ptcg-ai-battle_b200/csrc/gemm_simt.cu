// SIMT fp32-accumulate GEMM with the fused epilogue of GemmArgs.
// Used for every GEMM in PTCG_FP32 (parity) mode -- fp32 FFMA gives the
// <=1e-4 relative agreement with the torch fp32 reference that tcgen05
// (no true-fp32 kind) cannot -- and, in PTCG_BF16 mode, for the small
// per-sample / per-table GEMMs whose operands stay fp32.
#include "common.cuh"
#include "internal.h"

namespace {

constexpr int BM = 64, BN = 64, BK = 16, NT = 256;

template <typename T>
PTCG_DEV float ld_as_f(const void* p, long i) { return to_f<T>(((const T*)p)[i]); }

PTCG_DEV float ld_dt(const void* p, long i, int dt) {
    return dt == DT_F32 ? ((const float*)p)[i] : __bfloat162float(((const bf16*)p)[i]);
}
PTCG_DEV void st_dt(void* p, long i, int dt, float v) {
    if (dt == DT_F32) ((float*)p)[i] = v;
    else ((bf16*)p)[i] = __float2bfloat16_rn(v);
}

template <typename T>
__global__ void __launch_bounds__(NT) k_gemm_simt(GemmArgs a) {
    __shared__ __align__(16) float As[BK][BM];
    __shared__ __align__(16) float Bs[BK][BN];
    const int tid = threadIdx.x;
    const int tx = tid % 16, ty = tid / 16;
    const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
    const T* A = (const T*)a.A;
    const T* B = (const T*)a.B;
    float acc[4][4];
    #pragma unroll
    for (int i = 0; i < 4; i++)
        #pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = 0.f;

    // split-K (plain f32 accumulate only): blockIdx.z owns K range [kb, ke)
    const int kchunk = (int)(((a.K + gridDim.z - 1) / gridDim.z + BK - 1) / BK) * BK;
    const int kb = blockIdx.z * kchunk;
    const int ke = min(a.K, kb + kchunk);
    for (int k0 = kb; k0 < ke; k0 += BK) {
        #pragma unroll
        for (int e = 0; e < 4; e++) {
            int idx = tid + e * NT;
            int m, k;
            if (a.a_kmajor) { m = idx / BK; k = idx % BK; }
            else { k = idx / BM; m = idx % BM; }
            int gm = m0 + m, gk = k0 + k;
            float v = 0.f;
            if (gm < a.M && gk < ke)
                v = to_f<T>(a.a_kmajor ? A[(long)gm * a.lda + gk] : A[(long)gk * a.lda + gm]);
            As[k][m] = v;
            int n;
            if (a.b_kmajor) { n = idx / BK; k = idx % BK; }
            else { k = idx / BN; n = idx % BN; }
            int gn = n0 + n; gk = k0 + k;
            v = 0.f;
            if (gn < a.N && gk < ke)
                v = to_f<T>(a.b_kmajor ? B[(long)gn * a.ldb + gk] : B[(long)gk * a.ldb + gn]);
            Bs[k][n] = v;
        }
        __syncthreads();
        #pragma unroll
        for (int k = 0; k < BK; k++) {
            float4 av = *(const float4*)&As[k][ty * 4];
            float4 bv = *(const float4*)&Bs[k][tx * 4];
            float ar[4] = {av.x, av.y, av.z, av.w};
            float br[4] = {bv.x, bv.y, bv.z, bv.w};
            #pragma unroll
            for (int i = 0; i < 4; i++)
                #pragma unroll
                for (int j = 0; j < 4; j++) acc[i][j] = fmaf(ar[i], br[j], acc[i][j]);
        }
        __syncthreads();
    }

    float csum[4] = {0.f, 0.f, 0.f, 0.f};
    #pragma unroll
    for (int i = 0; i < 4; i++) {
        int m = m0 + ty * 4 + i;
        if (m >= a.M) continue;
        long orow = a.remap_group > 0
            ? (long)(m / a.remap_group) * a.remap_stride + a.remap_off + (m % a.remap_group)
            : (long)m;
        #pragma unroll
        for (int j = 0; j < 4; j++) {
            int n = n0 + tx * 4 + j;
            if (n >= a.N) continue;
            float v = a.alpha * acc[i][j];
            if (gridDim.z > 1) {             // split-K partial: atomic accumulate
                atomicAdd((float*)a.out + orow * a.ldo + n, v);
                continue;
            }
            if (a.bias) v += a.bias[n];
            if (a.bcast) v += a.bcast[(long)(m / a.bcast_group) * a.ld_bcast + n];
            if (a.act == ACT_GELU) {
                if (a.out2) st_dt(a.out2, (long)m * a.ldo2 + n, a.out2_dtype, gelu_grad_f(v));
                v = gelu_f(v);
            } else if (a.act == ACT_GELU_BWD) {
                v *= ld_dt(a.aux, (long)m * a.ld_aux + n, a.aux_dtype);
            }
            if (a.resid) v += a.resid[orow * a.ld_resid + n];
            long oi = orow * a.ldo + n;
            if (a.accumulate) v += ld_dt(a.out, oi, a.out_dtype);
            st_dt(a.out, oi, a.out_dtype, v);
            if (a.act != ACT_GELU && a.out2) st_dt(a.out2, orow * a.ldo2 + n, a.out2_dtype, v);
            csum[j] += v;
        }
    }
    if (a.colsum && gridDim.z == 1) {
        // per-CTA column partials in shared memory, one global atomic per column
        __syncthreads();
        float* cs = &As[0][0];
        if (tid < BN) cs[tid] = 0.f;
        __syncthreads();
        #pragma unroll
        for (int j = 0; j < 4; j++) atomicAdd(&cs[tx * 4 + j], csum[j]);
        __syncthreads();
        if (tid < BN && n0 + tid < a.N) atomicAdd(&a.colsum[n0 + tid], cs[tid]);
    }
}

}  // namespace

void gemm_simt(const GemmArgs& a, cudaStream_t s) {
    if (a.M <= 0 || a.N <= 0) return;
    dim3 grid(cdiv(a.M, BM), cdiv(a.N, BN));
    // plain f32 accumulation with a long reduction (weight gradients): split K
    bool plain = a.accumulate && a.out_dtype == DT_F32 && !a.bias && !a.bcast &&
                 a.act == ACT_NONE && !a.resid && !a.out2 && a.remap_group == 0 && !a.colsum;
    if (plain && a.K >= 4096) {
        long tiles = (long)grid.x * grid.y;
        long want = (296 + tiles - 1) / tiles;            // ~2 waves of 148 SMs
        long maxs = a.K / 1024;
        grid.z = (unsigned)(want < maxs ? want : maxs);
        if (grid.z < 1) grid.z = 1;
        if (grid.z > 512) grid.z = 512;
    }
    if (a.dtype == DT_F32) ++g_ptcg_launches, k_gemm_simt<float><<<grid, NT, 0, s>>>(a);
    else ++g_ptcg_launches, k_gemm_simt<bf16><<<grid, NT, 0, s>>>(a);
}
