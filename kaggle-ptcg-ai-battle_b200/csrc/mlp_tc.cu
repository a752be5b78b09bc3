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
// Roles: two TMA producer lanes (the A tile and the W1 chunks; the W2 chunks:
// their stages free at different times, W1 after its H MMA, W2 after its Y
// MMA; no multicast), an MMA lane that keeps two H MMAs ahead of the Y MMAs
// (four H buffers in TMEM), and 16 epilogue warps (4 per TMEM lane
// quadrant, each on a quarter of a chunk's columns and of Y's).  GELU and
// its rounding to bf16 are those of the GEMM engine's epilogue, and Y sums
// the chunks in the unfused FFN2's K order.  Every wait is bounded.
//
// Measured on a B200 (c0, 1024 agents, the rollout graph): 3.41 ms per
// forward with this kernel against 2.91-3.05 ms with the two GEMMs, with
// either epilogue GELU, so it is off by default (ptcg_set_fused_mlp).  Each
// 128-row tile streams all of W1 and W2 (1 MB at d 256, ffn 1024) through
// L2 into shared memory, more than L2 delivers at the MMA rate.
#include <algorithm>

#include "common.cuh"
#include "internal.h"
#include "tc_ptx.cuh"

namespace {

using namespace tcx;

constexpr int MT = 128;                    // rows per tile (TMEM lanes)
constexpr int HC = 64;                     // hidden units per chunk
constexpr int DM = 256;                    // model width: A columns and Y columns
constexpr int NH = 4;                      // H buffers in TMEM
constexpr int LEAD = 2;                    // H MMAs issued ahead of the Y MMAs
constexpr int EPI_WARPS = 16;
constexpr int EPI0 = 3;                    // first epilogue warp
constexpr int THREADS = 32 * (EPI0 + EPI_WARPS);
constexpr uint32_t A_BYTES = MT * DM * 2;          // 4 K-atoms of {64 cols, 128 rows}
constexpr uint32_t W1_BYTES = HC * DM * 2;         // 4 K-atoms of {64 cols, 64 rows}
constexpr uint32_t W2_BYTES = DM * HC * 2;         // {64 cols, 256 rows}
constexpr uint32_t P_BYTES = MT * HC * 2;          // {64 cols, 128 rows}
constexpr uint32_t OFF_W1 = A_BYTES;
constexpr uint32_t OFF_W2 = OFF_W1 + 2 * W1_BYTES;
constexpr uint32_t OFF_P = OFF_W2 + 2 * W2_BYTES;
constexpr uint32_t OFF_BAR = OFF_P + 2 * P_BYTES;
constexpr size_t SMEM_BYTES = 1024 + OFF_BAR + 256;
constexpr uint32_t T_Y = 0, T_H = 256;             // TMEM columns: Y, then NH H buffers

__device__ int g_mlp_tc_error;

struct MlpParams {
    int rows, F;
    long ld_res, ld_out;
    const float* b1;
    const float* b2;
    const float* res;
    float* out;
};

// barrier slots (8 bytes each) after OFF_BAR
enum : int {
    B_AFULL = 0, B_AEMPTY, B_W1FULL, B_W1EMPTY = B_W1FULL + 2, B_W2FULL = B_W1EMPTY + 2,
    B_W2EMPTY = B_W2FULL + 2, B_HFULL = B_W2EMPTY + 2, B_HEMPTY = B_HFULL + NH,
    B_PFULL = B_HEMPTY + NH, B_PEMPTY = B_PFULL + 2, B_YFULL = B_PEMPTY + 2, B_YEMPTY,
    B_DRAIN, B_COUNT
};

__global__ void __launch_bounds__(THREADS, 1) k_mlp_fwd_tc(
        const __grid_constant__ CUtensorMap a_map, const __grid_constant__ CUtensorMap w1_map,
        const __grid_constant__ CUtensorMap w2_map, const __grid_constant__ MlpParams P) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = (uint64_t*)(smem + OFF_BAR);
    const uint32_t bar0 = saddr(bars);
    auto bar = [&](int i) { return bar0 + 8u * (uint32_t)i; };
    uint32_t* tmem_slot = (uint32_t*)(bars + B_COUNT);
    volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nepi = 32 * EPI_WARPS;

    if (threadIdx.x == 0) {
        bar_init(bar(B_AFULL), 1); bar_init(bar(B_AEMPTY), 1);
        for (int i = 0; i < 2; i++) {
            bar_init(bar(B_W1FULL + i), 1); bar_init(bar(B_W1EMPTY + i), 1);
            bar_init(bar(B_W2FULL + i), 1); bar_init(bar(B_W2EMPTY + i), 1);
            bar_init(bar(B_PFULL + i), nepi); bar_init(bar(B_PEMPTY + i), 1);
        }
        for (int i = 0; i < NH; i++) { bar_init(bar(B_HFULL + i), 1); bar_init(bar(B_HEMPTY + i), nepi); }
        bar_init(bar(B_YFULL), 1); bar_init(bar(B_YEMPTY), nepi); bar_init(bar(B_DRAIN), 1);
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
    const uint32_t s_a = saddr(smem), s_w1 = s_a + OFF_W1, s_w2 = s_a + OFF_W2, s_p = s_a + OFF_P;
    int* err = &g_mlp_tc_error;

    if (warp == 0 || warp == 2) {
        // ------------------------------------------------ TMA producers: warp 0
        // the A tiles and the W1 chunks, warp 2 the W2 chunks (their stages
        // free at different times: W1 after the chunk's H MMA, W2 after its Y)
        if (lane == 0) {
            const bool w1side = warp == 0;
            int t = 0, c = 0, issued_a = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, t++) {
                if (w1side) {
                    if (!bar_wait(bar(B_AEMPTY), (uint32_t)((t & 1) ^ 1), abort_flag, err, 1)) break;
                    bar_expect_tx(bar(B_AFULL), A_BYTES);
                    #pragma unroll
                    for (int k = 0; k < 4; k++)
                        tma_2d(s_a + k * (A_BYTES / 4), &a_map, bar(B_AFULL), 64 * k, tile * MT);
                    issued_a++;
                }
                for (int j = 0; j < nchunk; j++, c++) {
                    const int st = c & 1;
                    const int fullb = w1side ? B_W1FULL : B_W2FULL, emptyb = w1side ? B_W1EMPTY : B_W2EMPTY;
                    if (!bar_wait(bar(emptyb + st), (uint32_t)(((c >> 1) & 1) ^ 1), abort_flag, err, 2)) {
                        ok = false;
                        break;
                    }
                    if (w1side) {
                        bar_expect_tx(bar(fullb + st), W1_BYTES);
                        #pragma unroll
                        for (int k = 0; k < 4; k++)
                            tma_2d(s_w1 + st * W1_BYTES + k * (W1_BYTES / 4), &w1_map, bar(fullb + st),
                                   64 * k, j * HC);
                    } else {
                        bar_expect_tx(bar(fullb + st), W2_BYTES);
                        tma_2d(s_w2 + st * W2_BYTES, &w2_map, bar(fullb + st), j * HC, 0);
                    }
                }
            }
            // on an abort, let the copies in flight land before exiting
            if (*abort_flag) {
                if (issued_a > 0) bar_drain(bar(B_AFULL), (uint32_t)((issued_a - 1) & 1));
                const int fullb = w1side ? B_W1FULL : B_W2FULL;
                for (int k = 1; k <= 2 && k <= c; k++)
                    bar_drain(bar(fullb + ((c - k) & 1)), (uint32_t)(((c - k) >> 1) & 1));
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA lane
        // per tile: H_0 .. H_{LEAD-1}, then for each chunk j: H_{j+LEAD}, Y_j
        if (lane == 0) {
            int t = 0, ch = 0, cy = 0;           // chunks whose H / Y MMAs were issued
            bool ok = true;
            const uint32_t id_h = idesc_bf16(HC, 0, 0), id_y = idesc_bf16(DM, 0, 0);
            auto issue_h = [&](int j, int last) -> bool {
                const int st = ch & 1, hb = ch % NH;
                if (!bar_wait(bar(B_W1FULL + st), (uint32_t)((ch >> 1) & 1), abort_flag, err, 4) ||
                    !bar_wait(bar(B_HEMPTY + hb), (uint32_t)(((ch / NH) & 1) ^ 1), abort_flag, err, 7))
                    return false;
                tc_fence_after();
                const uint32_t w1 = s_w1 + st * W1_BYTES;
                #pragma unroll
                for (int k = 0; k < 4; k++)
                    #pragma unroll
                    for (int s = 0; s < 4; s++)
                        mma_bf16(tmem + T_H + HC * hb, sdesc(s_a + k * (A_BYTES / 4) + 32 * s, 16, 1024, 2),
                                 sdesc(w1 + k * (W1_BYTES / 4) + 32 * s, 16, 1024, 2), id_h,
                                 (k | s) ? 1u : 0u);
                mma_commit_to(bar(B_HFULL + hb));
                mma_commit_to(bar(B_W1EMPTY + st));  // W1 chunk read
                if (last) mma_commit_to(bar(B_AEMPTY));  // A read once this lands
                ch++;
                (void)j;
                return true;
            };
            auto issue_y = [&](int j) -> bool {
                const int pb = cy & 1, st = cy & 1;
                if (!bar_wait(bar(B_PFULL + pb), (uint32_t)((cy >> 1) & 1), abort_flag, err, 5) ||
                    !bar_wait(bar(B_W2FULL + st), (uint32_t)((cy >> 1) & 1), abort_flag, err, 6))
                    return false;
                if (j == 0 && !bar_wait(bar(B_YEMPTY), (uint32_t)((t & 1) ^ 1), abort_flag, err, 3))
                    return false;
                tc_fence_after();
                const uint32_t pa = s_p + pb * P_BYTES, wb = s_w2 + st * W2_BYTES;
                #pragma unroll
                for (int s = 0; s < 4; s++)
                    mma_bf16(tmem + T_Y, sdesc(pa + 32 * s, 16, 1024, 2), sdesc(wb + 32 * s, 16, 1024, 2),
                             id_y, (j > 0 || s > 0) ? 1u : 0u);
                mma_commit_to(bar(B_PEMPTY + pb));   // P buffer read
                mma_commit_to(bar(B_W2EMPTY + st));  // W2 chunk read
                cy++;
                return true;
            };
            for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, t++) {
                if (!bar_wait(bar(B_AFULL), (uint32_t)(t & 1), abort_flag, err, 8)) break;
                for (int j = 0; j < LEAD && j < nchunk && ok; j++) ok = issue_h(j, j == nchunk - 1);
                for (int j = 0; j < nchunk && ok; j++) {
                    if (j + LEAD < nchunk) ok = issue_h(j + LEAD, j + LEAD == nchunk - 1);
                    if (ok) ok = issue_y(j);
                }
                if (ok) mma_commit_to(bar(B_YFULL));
            }
            // no MMA may still be in flight when TMEM is released
            mma_commit_to(bar(B_DRAIN));
            bar_drain(bar(B_DRAIN), 0);
        }
        __syncwarp();
    } else {
        // ------------------------------------------------ epilogue warps
        const int quad = warp & 3, u = (warp - EPI0) >> 2;
        const int row = quad * 32 + lane;
        const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
        int t = 0, g = 0;                         // g: chunks of this CTA so far
        bool ok = true;
        for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, t++) {
            for (int j = 0; j < nchunk; j++, g++) {
                const int hb = g % NH, pb = g & 1;
                // warp-uniform outcome: tcgen05.ld below is warp-collective
                ok = __all_sync(0xffffffffu, bar_wait(bar(B_HFULL + hb), (uint32_t)((g / NH) & 1),
                                                      abort_flag, err, 9));
                if (!ok) break;
                tc_fence_after();
                float v[16];
                tmem_ld32x32_x16(tmem + lane_off + T_H + HC * hb + 16 * u, v);
                tmem_wait_ld();
                tc_fence_before();
                bar_arrive(bar(B_HEMPTY + hb));
                const float* bias = P.b1 + j * HC + 16 * u;
                uint32_t q[8];
                #pragma unroll
                for (int i = 0; i < 16; i += 2) {
                    float y0, y1, g0, g1;
                    gelu2(v[i] + __ldg(bias + i), v[i + 1] + __ldg(bias + i + 1), y0, y1, g0, g1);
                    __nv_bfloat162 hq = __floats2bfloat162_rn(y0, y1);
                    q[i >> 1] = *(uint32_t*)&hq;
                }
                // the Y MMA two chunks back has read this P buffer
                ok = __all_sync(0xffffffffu, bar_wait(bar(B_PEMPTY + pb), (uint32_t)(((g >> 1) & 1) ^ 1),
                                                      abort_flag, err, 10));
                if (!ok) break;
                // 128-byte-swizzled K-major rows: granule k of row r at k ^ (r & 7)
                uint8_t* prow = smem + OFF_P + pb * P_BYTES + row * 128;
                *(uint4*)(prow + (((2 * u) ^ (row & 7)) << 4)) = make_uint4(q[0], q[1], q[2], q[3]);
                *(uint4*)(prow + (((2 * u + 1) ^ (row & 7)) << 4)) = make_uint4(q[4], q[5], q[6], q[7]);
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                bar_arrive(bar(B_PFULL + pb));
            }
            if (!ok) break;
            ok = __all_sync(0xffffffffu, bar_wait(bar(B_YFULL), (uint32_t)(t & 1), abort_flag, err, 11));
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
            bar_arrive(bar(B_YEMPTY));
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
