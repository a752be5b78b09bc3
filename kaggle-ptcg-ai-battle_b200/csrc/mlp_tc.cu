// Fused transformer MLP of the rollout forward on the tcgen05 tensor cores:
//   out = res + b2 + GELU(A W1^T + b1) W2^T
// with A = LN2(x) rows (bf16, width 256), W1 [F x 256], W2 [256 x F] (the
// block's FFN1 / FFN2, ptcg/rl/model.py:70-91; the reference runs them as
// two linear layers around a GELU kernel, native/model/ptcg_model3.cu:36-38)
// and the fp32 residual stream.  The F-wide hidden activation never leaves the SM:
// per 128-row tile the hidden units go in chunks of 64 through
//   H_j = A W1_j^T       (TMEM, double-buffered, M = 128, N = 64, K = 256)
//   P_j = GELU(H_j + b1) (epilogue warps, bf16, into shared memory)
//   Y  += P_j W2_j^T     (TMEM accumulator, M = 128, N = 256, K = 64)
// and only Y (+ b2 + residual) is written.  The unfused path writes and
// re-reads the hidden activation (2 x 2 x F bytes a row); the training
// forward keeps that path, since its backward needs the hidden activation.
//
// Roles: a TMA producer lane (A tile once per tile; W1 / W2 chunks through two
// stages, no multicast), an MMA lane, 16 epilogue warps (4 per TMEM lane
// quadrant, each on a quarter of a chunk's columns and of Y's).  GELU and
// its rounding to bf16 are those of the GEMM engine's epilogue, and Y sums
// the chunks in the unfused FFN2's K order.  Every wait is bounded.
//
// Measured on a B200 (c0, 1024 agents, the rollout graph): 3.58 ms per
// forward with this kernel against 2.96 ms with the two GEMMs, so it is off
// by default (ptcg_set_fused_mlp).  Each chunk's H -> GELU -> P -> Y hand-off
// sits on the critical path with only two H / P buffers (the W1 / W2 chunk
// stages take the rest of shared memory), so the 128-row tile's 16 chunks
// run about three times longer than their MMA and GELU work.
#include <algorithm>

#include "common.cuh"
#include "internal.h"
#include "tc_ptx.cuh"

namespace {

using namespace tcx;

constexpr int MT = 128;                    // rows per tile (TMEM lanes)
constexpr int HC = 64;                     // hidden units per chunk
constexpr int DM = 256;                    // model width: A columns and Y columns
constexpr int EPI_WARPS = 16;
constexpr int THREADS = 64 + 32 * EPI_WARPS;
constexpr uint32_t A_BYTES = MT * DM * 2;          // 4 K-atoms of {64 cols, 128 rows}
constexpr uint32_t W1_BYTES = HC * DM * 2;         // 4 K-atoms of {64 cols, 64 rows}
constexpr uint32_t W2_BYTES = DM * HC * 2;         // {64 cols, 256 rows}
constexpr uint32_t W_STAGE = W1_BYTES + W2_BYTES;
constexpr uint32_t P_BYTES = MT * HC * 2;          // {64 cols, 128 rows}
constexpr uint32_t OFF_W = A_BYTES;
constexpr uint32_t OFF_P = OFF_W + 2 * W_STAGE;
constexpr uint32_t OFF_BAR = OFF_P + 2 * P_BYTES;
constexpr size_t SMEM_BYTES = 1024 + OFF_BAR + 256;
constexpr uint32_t T_Y = 0, T_H = 256;             // TMEM columns: Y, then two H buffers

__device__ int g_mlp_tc_error;

struct MlpParams {
    int rows, F;
    long ld_res, ld_out;
    const float* b1;
    const float* b2;
    const float* res;
    float* out;
};

__global__ void __launch_bounds__(THREADS, 1) k_mlp_fwd_tc(
        const __grid_constant__ CUtensorMap a_map, const __grid_constant__ CUtensorMap w1_map,
        const __grid_constant__ CUtensorMap w2_map, const __grid_constant__ MlpParams P) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = (uint64_t*)(smem + OFF_BAR);
    // afull aempty wfull[2] wempty[2] hfull[2] hempty[2] pfull[2] pempty[2] yfull yempty drain
    const uint32_t afull = saddr(bars), aempty = afull + 8;
    const uint32_t wfull0 = afull + 16, wempty0 = afull + 32, hfull0 = afull + 48;
    const uint32_t hempty0 = afull + 64, pfull0 = afull + 80, pempty0 = afull + 96;
    const uint32_t yfull = afull + 112, yempty = afull + 120, drain = afull + 128;
    uint32_t* tmem_slot = (uint32_t*)(bars + 17);
    volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nepi = 32 * EPI_WARPS;

    if (threadIdx.x == 0) {
        bar_init(afull, 1); bar_init(aempty, 1);
        for (int i = 0; i < 2; i++) {
            bar_init(wfull0 + 8 * i, 1); bar_init(wempty0 + 8 * i, 1);
            bar_init(hfull0 + 8 * i, 1); bar_init(hempty0 + 8 * i, nepi);
            bar_init(pfull0 + 8 * i, nepi); bar_init(pempty0 + 8 * i, 1);
        }
        bar_init(yfull, 1); bar_init(yempty, nepi); bar_init(drain, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(saddr(tmem_slot)), "r"(512) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int tiles = (P.rows + MT - 1) / MT;
    const int nchunk = P.F / HC;
    const uint32_t s_a = saddr(smem), s_w = s_a + OFF_W, s_p = s_a + OFF_P;

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            int t = 0, c = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, t++) {
                if (!bar_wait(aempty, (uint32_t)((t & 1) ^ 1), abort_flag, &g_mlp_tc_error, 1)) break;
                bar_expect_tx(afull, A_BYTES);
                #pragma unroll
                for (int k = 0; k < 4; k++) tma_2d(s_a + k * (A_BYTES / 4), &a_map, afull, 64 * k, tile * MT);
                for (int j = 0; j < nchunk; j++, c++) {
                    const int st = c & 1;
                    if (!bar_wait(wempty0 + 8 * st, (uint32_t)(((c >> 1) & 1) ^ 1), abort_flag,
                                  &g_mlp_tc_error, 2)) { ok = false; break; }
                    const uint32_t fb = wfull0 + 8 * st, dst = s_w + st * W_STAGE;
                    bar_expect_tx(fb, W_STAGE);
                    #pragma unroll
                    for (int k = 0; k < 4; k++) tma_2d(dst + k * (W1_BYTES / 4), &w1_map, fb, 64 * k, j * HC);
                    tma_2d(dst + W1_BYTES, &w2_map, fb, j * HC, 0);
                }
            }
            // on an abort, let the copies in flight land before exiting
            if (*abort_flag) {
                if (t > 0) bar_drain(afull, (uint32_t)((t - 1) & 1));
                for (int k = 1; k <= 2 && k <= c; k++)
                    bar_drain(wfull0 + 8 * ((c - k) & 1), (uint32_t)(((c - k) >> 1) & 1));
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA lane
        if (lane == 0) {
            int t = 0, c = 0, h = 0;
            bool ok = true;
            const uint32_t id_h = idesc_bf16(HC, 0, 0), id_y = idesc_bf16(DM, 0, 0);
            // Y += P_jj W2_jj^T (chunk jj of this tile, its H index hh, W stage index cc)
            auto issue_y = [&](int jj, int hh, int cc) -> bool {
                const int pb = hh & 1;
                if (!bar_wait(pfull0 + 8 * pb, (uint32_t)((hh >> 1) & 1), abort_flag, &g_mlp_tc_error, 5))
                    return false;
                if (jj == 0 &&
                    !bar_wait(yempty, (uint32_t)((t & 1) ^ 1), abort_flag, &g_mlp_tc_error, 6))
                    return false;
                tc_fence_after();
                const uint32_t pa = s_p + pb * P_BYTES, wb = s_w + (cc & 1) * W_STAGE + W1_BYTES;
                #pragma unroll
                for (int s = 0; s < 4; s++)
                    mma_bf16(tmem + T_Y, sdesc(pa + 32 * s, 16, 1024, 2), sdesc(wb + 32 * s, 16, 1024, 2),
                             id_y, (jj > 0 || s > 0) ? 1u : 0u);
                mma_commit_to(pempty0 + 8 * pb);            // P buffer read
                mma_commit_to(wempty0 + 8 * (cc & 1));      // W1 / W2 stage of this chunk read
                return true;
            };
            for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, t++) {
                if (!bar_wait(afull, (uint32_t)(t & 1), abort_flag, &g_mlp_tc_error, 3)) break;
                for (int j = 0; j < nchunk && ok; j++, c++, h++) {
                    const int st = c & 1, hb = h & 1;
                    if (!bar_wait(wfull0 + 8 * st, (uint32_t)((c >> 1) & 1), abort_flag, &g_mlp_tc_error, 4) ||
                        !bar_wait(hempty0 + 8 * hb, (uint32_t)(((h >> 1) & 1) ^ 1), abort_flag,
                                  &g_mlp_tc_error, 7)) { ok = false; break; }
                    tc_fence_after();
                    // H_j = A W1_j^T: 4 K-atoms of 64, 4 steps of 16 each
                    const uint32_t w1 = s_w + st * W_STAGE;
                    #pragma unroll
                    for (int k = 0; k < 4; k++)
                        #pragma unroll
                        for (int s = 0; s < 4; s++)
                            mma_bf16(tmem + T_H + HC * hb,
                                     sdesc(s_a + k * (A_BYTES / 4) + 32 * s, 16, 1024, 2),
                                     sdesc(w1 + k * (W1_BYTES / 4) + 32 * s, 16, 1024, 2), id_h,
                                     (k | s) ? 1u : 0u);
                    mma_commit_to(hfull0 + 8 * hb);
                    if (j == nchunk - 1) mma_commit_to(aempty);  // A read once this lands
                    if (j > 0 && !issue_y(j - 1, h - 1, c - 1)) { ok = false; break; }
                }
                if (!ok || !issue_y(nchunk - 1, h - 1, c - 1)) { ok = false; break; }
                mma_commit_to(yfull);
            }
            // no MMA may still be in flight when TMEM is released
            mma_commit_to(drain);
            bar_drain(drain, 0);
        }
        __syncwarp();
    } else {
        // ------------------------------------------------ epilogue warps
        const int quad = warp & 3, u = (warp - 2) >> 2;
        const int row = quad * 32 + lane;
        const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
        int t = 0, h = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, t++) {
            for (int j = 0; j < nchunk; j++, h++) {
                const int hb = h & 1;
                // warp-uniform outcome: tcgen05.ld below is warp-collective
                ok = __all_sync(0xffffffffu,
                                bar_wait(hfull0 + 8 * hb, (uint32_t)((h >> 1) & 1), abort_flag, &g_mlp_tc_error, 8));
                if (!ok) break;
                tc_fence_after();
                float v[16];
                tmem_ld32x32_x16(tmem + lane_off + T_H + HC * hb + 16 * u, v);
                tmem_wait_ld();
                tc_fence_before();
                bar_arrive(hempty0 + 8 * hb);
                const float* bias = P.b1 + j * HC + 16 * u;
                uint32_t q[8];
                #pragma unroll
                for (int i = 0; i < 16; i += 2) {
                    float y0, y1, g0, g1;
                    gelu2(v[i] + __ldg(bias + i), v[i + 1] + __ldg(bias + i + 1), y0, y1, g0, g1);
                    __nv_bfloat162 hq = __floats2bfloat162_rn(y0, y1);
                    q[i >> 1] = *(uint32_t*)&hq;
                }
                // the Y MMA of chunk h - 2 has read this P buffer
                ok = __all_sync(0xffffffffu, bar_wait(pempty0 + 8 * hb, (uint32_t)(((h >> 1) & 1) ^ 1),
                                                      abort_flag, &g_mlp_tc_error, 9));
                if (!ok) break;
                // 128-byte-swizzled K-major rows: granule g of row r at g ^ (r & 7)
                uint8_t* prow = smem + OFF_P + hb * P_BYTES + row * 128;
                *(uint4*)(prow + (((2 * u) ^ (row & 7)) << 4)) = make_uint4(q[0], q[1], q[2], q[3]);
                *(uint4*)(prow + (((2 * u + 1) ^ (row & 7)) << 4)) = make_uint4(q[4], q[5], q[6], q[7]);
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                bar_arrive(pfull0 + 8 * hb);
            }
            if (!ok) break;
            ok = __all_sync(0xffffffffu, bar_wait(yfull, (uint32_t)(t & 1), abort_flag, &g_mlp_tc_error, 10));
            if (!ok) break;
            tc_fence_after();
            const long grow = (long)tile * MT + row;
            #pragma unroll
            for (int part = 0; part < 4; part++) {
                float y[16];
                const int c0 = 64 * u + 16 * part;
                tmem_ld32x32_x16(tmem + lane_off + T_Y + c0, y);
                tmem_wait_ld();
                if (grow < P.rows) {
                    const float4* r4 = (const float4*)(P.res + grow * P.ld_res + c0);
                    float4* o4 = (float4*)(P.out + grow * P.ld_out + c0);
                    #pragma unroll
                    for (int q4 = 0; q4 < 4; q4++) {
                        const float4 r = r4[q4];
                        const float* b = P.b2 + c0 + 4 * q4;
                        o4[q4] = make_float4(y[4 * q4] + __ldg(b) + r.x, y[4 * q4 + 1] + __ldg(b + 1) + r.y,
                                             y[4 * q4 + 2] + __ldg(b + 2) + r.z,
                                             y[4 * q4 + 3] + __ldg(b + 3) + r.w);
                    }
                }
            }
            tc_fence_before();
            bar_arrive(yempty);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
                     :: "r"(tmem), "r"(512) : "memory");
    }
}

}  // namespace

int mlp_tc_error_read_reset() {
    int v = 0, zero = 0;
    cudaMemcpyFromSymbol(&v, g_mlp_tc_error, sizeof(int));
    cudaMemcpyToSymbol(g_mlp_tc_error, &zero, sizeof(int));
    return v;
}

bool mlp_fwd_tc(const void* a, long lda, const void* w1, long ldw1, const float* b1,
                const void* w2, long ldw2, const float* b2, const float* res, long ld_res,
                float* out, long ld_out, int rows, int D, int F, cudaStream_t s) {
    if (D != DM || F < HC || F % HC || rows <= 0 || !b1 || !b2 || !res || !out) return false;
    if (((uintptr_t)a & 15) || ((uintptr_t)w1 & 15) || ((uintptr_t)w2 & 15) || ((uintptr_t)res & 15) ||
        ((uintptr_t)out & 15) || (lda % 8) || (ldw1 % 8) || (ldw2 % 8) || (ld_res % 4) || (ld_out % 4))
        return false;
    CUtensorMap am, w1m, w2m;
    if (!tc_make_map_2d(&am, a, DT_BF16, DM, rows, lda, 64, MT, 128) ||
        !tc_make_map_2d(&w1m, w1, DT_BF16, DM, F, ldw1, 64, HC, 128) ||
        !tc_make_map_2d(&w2m, w2, DT_BF16, F, DM, ldw2, 64, DM, 128))
        return false;
    MlpParams P;
    P.rows = rows; P.F = F;
    P.ld_res = ld_res; P.ld_out = ld_out;
    P.b1 = b1; P.b2 = b2; P.res = res; P.out = out;
    if (cudaFuncSetAttribute(k_mlp_fwd_tc, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)SMEM_BYTES) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    const int tiles = (rows + MT - 1) / MT;
    const int grid = std::min(tiles, tc_num_sms());
    ++g_ptcg_launches, k_mlp_fwd_tc<<<grid, THREADS, SMEM_BYTES, s>>>(am, w1m, w2m, P);
    return true;
}
