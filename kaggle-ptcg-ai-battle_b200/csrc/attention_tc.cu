// Masked multi-head attention on the 5th-generation tensor cores (tcgen05 /
// TMEM / TMA), bf16 operands, head width 32, fp32 softmax.  Semantics as the
// other attention paths (attention.cu): torch F.scaled_dot_product_attention
// with a boolean key-padding mask (ptcg/rl/model.py:86-89), scale 1/sqrt(32);
// the forward saves the per-row log-sum-exp; query rows at or past a
// sequence's row extent get zero output and a zero log-sum-exp.
//
// Work item = (sequence, head, 128-row query tile); the CTA (one per SM)
// keeps up to NWG items in flight, one per softmax warpgroup:
//  * the producer warp decodes 32 items at a time (one lane each), zero-fills
//    the query tiles that start past their sequence's extent, and for each
//    live item TMA-loads into a shared-memory stage the Q tile, the keys /
//    values below the extent in 128-row chunks ({32 cols, 128 rows} boxes,
//    64-byte swizzle, no multicast) and the sequence's 64-byte key-mask row
//    (bit j of word c*4 + j/32 = key c*128 + j kept; word 15 = the extent),
//    plus the item's coordinates;
//  * one MMA lane serves the warpgroups round-robin without blocking on any
//    one of them: S = Q K^T of a chunk into the warpgroup's TMEM columns
//    (M = 128 query rows = TMEM lanes, N = keys of the chunk, K = 32 as two
//    kind::f16 instructions) as soon as the stage has landed and the
//    warpgroup released its S columns, and PV = P V (A = P from the
//    warpgroup's shared-memory buffer, K-major 128-byte swizzle; B = V,
//    MN-major 64-byte swizzle, N = 32) once the warpgroup wrote P;
//  * each softmax warpgroup (four warps, one per TMEM lane quadrant, one query
//    row per thread) reads the row's scores with tcgen05.ld, masks them from
//    the key words (whole 32-key blocks at a time where they are all kept),
//    runs an online softmax across chunks in the exp2 domain, writes P (bf16)
//    and accumulates O = O * alpha + PV in registers.
// While one warpgroup's item waits on its MMAs, the others' softmax runs, so
// the tensor pipe, TMA and the four SM sub-partitions overlap.
//
// Every mbarrier wait is bounded by a clock budget: on expiry the CTA records
// an error code (attn_tc_error_read_reset), stops waiting, lets its issued
// copies and MMAs land, frees its TMEM and returns.
#include "common.cuh"
#include "internal.h"
#include "tc_ptx.cuh"

#include <algorithm>

namespace {

constexpr int DH = 32;                 // head width
constexpr int QT = 128;                // query rows per tile (MMA M, TMEM lanes)
constexpr int KC = 128;                // keys per chunk (S accumulator columns)
constexpr int MAXC = 3;                // key chunks per sequence: L <= 384
constexpr uint32_t TILE_BYTES = 128 * DH * 2;   // one {32 cols, 128 rows} bf16 box: 8 KB
constexpr uint32_t P_BYTES = 2 * 128 * 128;     // P: 128 rows x 128 keys bf16, two 64-key blocks
constexpr uint32_t MASK_BYTES = ATTN_KW_WORDS * 4;
constexpr int SMEM_MAX = 227 * 1024;
constexpr float LOG2E = 1.4426950408889634f;

__device__ int g_attn_tc_error;

// ------------------------------------------------------------ PTX helpers
// (the shared ones in tc_ptx.cuh; the wait records this file's error code)
using namespace tcx;
PTCG_DEV bool bar_wait(uint32_t b, uint32_t parity, volatile int* abort_flag, int code) {
    return tcx::bar_wait(b, parity, abort_flag, &g_attn_tc_error, code);
}
PTCG_DEV void tmem_ld32x32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 "
                 "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                 "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                   "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
                   "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]),
                   "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
                   "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
                   "=r"(r[30]), "=r"(r[31])
                 : "r"(taddr));
    #pragma unroll
    for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}
PTCG_DEV void tmem_st32x32(uint32_t taddr, const float (&v)[32]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
                 :: "r"(taddr), "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])), "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31])) : "memory");
}
PTCG_DEV void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// non-blocking probe of a barrier phase (the MMA lane polls several)
PTCG_DEV bool bar_test(uint32_t b, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred P;\n\t"
                 "mbarrier.test_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, P;\n\t}"
                 : "=r"(ok) : "r"(b), "r"(parity) : "memory");
    return ok != 0;
}

// coordinates of a live item, written by the producer next to its tiles
struct Meta { int n, h, qt, ext; };
PTCG_DEV Meta read_meta(const uint8_t* p) {
    const volatile int* v = (const volatile int*)p;
    Meta m;
    m.n = v[0]; m.h = v[1]; m.qt = v[2]; m.ext = v[3];
    return m;
}

struct FwdParams {
    int nseq, L, H, D;
    int nqt;                  // query tiles per (sequence, head)
    int maxc;                 // key chunks a stage has room for: ceil(L / KC)
    int ns;                   // stages
    long ldo;
    bf16* out;
    float* lse;
    const uint32_t* kw;       // [nseq][ATTN_KW_WORDS] key words (extent in the last)
    uint32_t stage_bytes;     // Q tile, maxc K and V chunks, mask row, Meta; 1 KB multiple
    uint32_t mask_off;        // mask row offset within a stage (a multiple of 8 KB)
};

// keys of chunk c, rounded up to the MMA's N granule of 16
PTCG_DEV int chunk_n(int ext, int c) { return min(KC, (ext - c * KC + 15) & ~15); }

PTCG_DEV float max3f(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}
// max of m and the kept entries (bit i of `bits`) of v[0..31]
PTCG_DEV float masked_max32(float m, const float* v, uint32_t bits) {
    if (bits == 0xffffffffu) {
        #pragma unroll
        for (int i = 0; i < 32; i += 2) m = max3f(m, v[i], v[i + 1]);
    } else {
        #pragma unroll
        for (int i = 0; i < 32; i += 2)
            m = max3f(m, ((bits >> i) & 1u) ? v[i] : -INFINITY,
                      ((bits >> (i + 1)) & 1u) ? v[i + 1] : -INFINITY);
    }
    return m;
}
// v[i] <- exp2(v[i] * sc - m) for kept entries, 0 for the others; adds
// them to the two running sums in sum2 (packed fp32 pairs)
PTCG_DEV void exp_block32(float* v, uint32_t bits, unsigned long long sc2,
                          unsigned long long nm2, unsigned long long& sum2) {
    #pragma unroll
    for (int i = 0; i < 32; i += 2) {
        float a, b;
        upk2(fma2(pk2(v[i], v[i + 1]), sc2, nm2), a, b);
        a = ex2_approx(a);
        b = ex2_approx(b);
        if (bits != 0xffffffffu) {
            a = ((bits >> i) & 1u) ? a : 0.f;
            b = ((bits >> (i + 1)) & 1u) ? b : 0.f;
        }
        v[i] = a;
        v[i + 1] = b;
        sum2 = add2(sum2, pk2(a, b));
    }
}
// 32 probabilities of row `row` as bf16 into granules q0 .. q0 + 3 of the
// row's 128-byte line (128-byte swizzle)
PTCG_DEV void store_p32(uint8_t* rp, int row, int q0, const float* v) {
    #pragma unroll
    for (int q = 0; q < 4; q++) {
        uint4 u;
        __nv_bfloat162* hq = (__nv_bfloat162*)&u;
        #pragma unroll
        for (int e = 0; e < 4; e++) hq[e] = __floats2bfloat162_rn(v[8 * q + 2 * e], v[8 * q + 2 * e + 1]);
        *(uint4*)(rp + (((q0 + q) ^ (row & 7)) << 4)) = u;
    }
}

// TMEM columns: S of warpgroup w at w * 128, its PV at 384 + 32 w
PTCG_DEV uint32_t s_col(int w) { return (uint32_t)(w * KC); }
PTCG_DEV uint32_t pv_col(int w) { return (uint32_t)(3 * KC + w * DH); }

template <int NWG>
__global__ void __launch_bounds__(64 + 128 * NWG, 1) k_attn_fwd_tc(
        const __grid_constant__ CUtensorMap qkv_map, const __grid_constant__ CUtensorMap kw_map,
        const __grid_constant__ FwdParams P) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    const int ns = P.ns;
    uint8_t* pbuf = smem + (size_t)ns * P.stage_bytes;               // NWG x P_BYTES
    uint64_t* bars = (uint64_t*)(pbuf + NWG * P_BYTES);
    // full[ns] empty[ns] sfull[NWG] pready[NWG] pvfull[NWG] drain
    uint32_t* tmem_slot = (uint32_t*)(bars + 2 * 4 + 3 * 3 + 1);
    volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
    const uint32_t full0 = saddr(bars), empty0 = saddr(bars + ns);
    const uint32_t sfull0 = saddr(bars + 2 * ns), pready0 = saddr(bars + 2 * ns + NWG);
    const uint32_t pvfull0 = saddr(bars + 2 * ns + 2 * NWG), drain = saddr(bars + 2 * ns + 3 * NWG);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int i = 0; i < ns; i++) { bar_init(full0 + 8 * i, 1); bar_init(empty0 + 8 * i, 1); }
        for (int w = 0; w < NWG; w++) {
            bar_init(sfull0 + 8 * w, 1);
            bar_init(pready0 + 8 * w, 128);
            bar_init(pvfull0 + 8 * w, 1);
        }
        bar_init(drain, 1);
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
    const long items = (long)P.nseq * P.H * P.nqt;
    const int D = P.D, L = P.L;

    if (warp == 0) {
        // ------------------------------------------------ producer warp
        int k = 0;                      // live items issued
        bool ok = true;
        for (long base = blockIdx.x; base < items && ok; base += 32L * gridDim.x) {
            const long it = base + (long)lane * gridDim.x;
            const bool valid = it < items;
            Meta me{0, 0, 0, 0};
            bool live = false;
            if (valid) {
                const int per_seq = P.H * P.nqt;
                me.n = (int)(it / per_seq);
                const int r = (int)(it - (long)me.n * per_seq);
                me.h = r / P.nqt;
                me.qt = r - me.h * P.nqt;
                me.ext = min(max((int)P.kw[(long)me.n * ATTN_KW_WORDS + ATTN_KW_WORDS - 1], 1), L);
                live = me.qt * QT < me.ext;
            }
            // query tiles past the extent: zero output and log-sum-exp
            unsigned zm = __ballot_sync(0xffffffffu, valid && !live);
            while (zm) {
                const int i = __ffs(zm) - 1;
                zm &= zm - 1;
                const int n = __shfl_sync(0xffffffffu, me.n, i);
                const int h = __shfl_sync(0xffffffffu, me.h, i);
                const int qt = __shfl_sync(0xffffffffu, me.qt, i);
                const int r0 = qt * QT, r1 = min(L, r0 + QT);
                for (int e = lane; e < (r1 - r0) * 4; e += 32)
                    *(uint4*)(P.out + ((long)n * L + r0 + (e >> 2)) * P.ldo + h * DH + (e & 3) * 8) =
                        make_uint4(0, 0, 0, 0);
                for (int r = r0 + lane; r < r1; r += 32) P.lse[((long)n * P.H + h) * L + r] = 0.f;
            }
            unsigned am = __ballot_sync(0xffffffffu, live);
            while (am) {
                const int i = __ffs(am) - 1;
                am &= am - 1;
                Meta m;
                m.n = __shfl_sync(0xffffffffu, me.n, i);
                m.h = __shfl_sync(0xffffffffu, me.h, i);
                m.qt = __shfl_sync(0xffffffffu, me.qt, i);
                m.ext = __shfl_sync(0xffffffffu, me.ext, i);
                if (lane == 0) {
                    const int st = k % ns;
                    if (!bar_wait(empty0 + 8 * st, (uint32_t)(((k / ns) & 1) ^ 1), abort_flag, 1)) {
                        ok = false;
                    } else {
                        uint8_t* sp = smem + (size_t)st * P.stage_bytes;
                        *(Meta*)(sp + P.mask_off + MASK_BYTES) = m;
                        const int nkc = (m.ext + KC - 1) / KC;
                        const uint32_t fb = full0 + 8 * st;
                        bar_expect_tx(fb, TILE_BYTES * (1 + 2 * nkc) + MASK_BYTES);
                        const uint32_t sb = saddr(sp);
                        const int row0 = m.n * L;
                        tma_2d(sb, &qkv_map, fb, m.h * DH, row0 + m.qt * QT);
                        for (int c = 0; c < nkc; c++) {
                            tma_2d(sb + TILE_BYTES * (1 + c), &qkv_map, fb, D + m.h * DH, row0 + c * KC);
                            tma_2d(sb + TILE_BYTES * (1 + P.maxc + c), &qkv_map, fb, 2 * D + m.h * DH,
                                   row0 + c * KC);
                        }
                        tma_2d(sb + P.mask_off, &kw_map, fb, 0, m.n);
                    }
                }
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) break;
                k++;
            }
        }
        // one end marker per warpgroup: a stage whose Meta has n = -1
        for (int w = 0; w < NWG && ok; w++) {
            if (lane == 0) {
                const int st = k % ns;
                if (!bar_wait(empty0 + 8 * st, (uint32_t)(((k / ns) & 1) ^ 1), abort_flag, 1)) {
                    ok = false;
                } else {
                    Meta m{-1, 0, 0, 0};
                    *(Meta*)(smem + (size_t)st * P.stage_bytes + P.mask_off + MASK_BYTES) = m;
                    bar_arrive(full0 + 8 * st);
                }
            }
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (ok) k++;
        }
        // on an abort, let the copies still in flight land before exiting
        if (lane == 0 && *abort_flag)
            for (int j = max(0, k - ns); j < k; j++)
                bar_drain(full0 + 8 * (j % ns), (uint32_t)((j / ns) & 1));
    } else if (warp == 1) {
        // ------------------------------------------------ MMA lane
        if (lane == 0) {
            int wk[NWG], wc[NWG], wnkc[NWG], wext[NWG], wg[NWG];
            uint32_t wbase[NWG];
            bool busy[NWG], sdone[NWG];
            #pragma unroll
            for (int w = 0; w < NWG; w++) { busy[w] = sdone[w] = false; wg[w] = 0; wk[w] = wc[w] = wnkc[w] = wext[w] = 0; wbase[w] = 0; }
            int next_k = 0;
            bool more = true;
            long long t_last = clock64();
            const uint32_t pbase = saddr(pbuf);
            while (true) {
                bool prog = false;
                // the next item goes to warpgroup next_k % NWG once that one is free
                if (more) {
                    #pragma unroll
                    for (int w = 0; w < NWG; w++) {
                        if (w != next_k % NWG || busy[w]) continue;
                        const int st = next_k % ns;
                        if (!bar_test(full0 + 8 * st, (uint32_t)((next_k / ns) & 1))) continue;
                        tc_fence_after();
                        uint8_t* sp = smem + (size_t)st * P.stage_bytes;
                        const Meta m = read_meta(sp + P.mask_off + MASK_BYTES);
                        if (m.n < 0) { more = false; continue; }
                        wk[w] = next_k; wc[w] = 0; wext[w] = m.ext;
                        wnkc[w] = (m.ext + KC - 1) / KC;
                        wbase[w] = saddr(sp);
                        busy[w] = true; sdone[w] = false;
                        next_k++;
                        prog = true;
                    }
                }
                #pragma unroll
                for (int w = 0; w < NWG; w++) {
                    if (!busy[w]) continue;
                    if (!sdone[w]) {
                        // S = Q K_c^T (the warpgroup released its S columns
                        // with its last pready)
                        const uint32_t kb = wbase[w] + TILE_BYTES * (1 + wc[w]);
                        const uint32_t id = idesc_bf16(chunk_n(wext[w], wc[w]), 0, 0);
                        #pragma unroll
                        for (int s = 0; s < 2; s++)
                            mma_bf16(tmem + s_col(w), sdesc(wbase[w] + 32 * s, 16, 512, 4),
                                     sdesc(kb + 32 * s, 16, 512, 4), id, s > 0 ? 1u : 0u);
                        mma_commit_to(sfull0 + 8 * w);
                        sdone[w] = true;
                        prog = true;
                    } else if (bar_test(pready0 + 8 * w, (uint32_t)(wg[w] & 1))) {
                        tc_fence_after();
                        // PV = P V_c (the warpgroup read the previous PV
                        // before this pready)
                        const uint32_t vb = wbase[w] + TILE_BYTES * (1 + P.maxc + wc[w]);
                        const uint32_t pw = pbase + w * P_BYTES;
                        const uint32_t id = idesc_bf16(DH, 0, 1);
                        const int ks = chunk_n(wext[w], wc[w]) / 16;
                        for (int s = 0; s < ks; s++)
                            mma_bf16(tmem + pv_col(w),
                                     sdesc(pw + (s >> 2) * 16384 + (s & 3) * 32, 16, 1024, 2),
                                     sdesc(vb + s * 1024, TILE_BYTES, 512, 4), id,
                                     (s > 0 || wc[w] > 0) ? 1u : 0u);
                        mma_commit_to(pvfull0 + 8 * w);
                        wg[w]++;
                        sdone[w] = false;
                        if (++wc[w] == wnkc[w]) {
                            mma_commit_to(empty0 + 8 * (wk[w] % ns));   // stage consumed
                            busy[w] = false;
                        }
                        prog = true;
                    }
                }
                bool any = false;
                #pragma unroll
                for (int w = 0; w < NWG; w++) any = any || busy[w];
                if (!more && !any) break;
                if (prog) {
                    t_last = clock64();
                } else if (__nanosleep(40), *abort_flag) {
                    break;
                } else if (clock64() - t_last > WAIT_BUDGET) {
                    *abort_flag = 1;
                    atomicCAS(&g_attn_tc_error, 0, 2);
                    break;
                }
            }
            // no MMA may still be in flight when TMEM is released
            mma_commit_to(drain);
            bar_drain(drain, 0);
        }
        __syncwarp();
    } else {
        // ------------------------------------------------ softmax warpgroups
        const int w = (warp - 2) >> 2;
        const int quad = warp & 3;
        const int row = quad * 32 + lane;               // query row within the tile = TMEM lane
        const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
        const uint32_t sb = tmem + lane_off + s_col(w);
        const uint32_t pvb = tmem + lane_off + pv_col(w);
        uint8_t* prow = pbuf + w * P_BYTES + row * 128;
        const uint32_t sfull = sfull0 + 8 * w, pready = pready0 + 8 * w, pvfull = pvfull0 + 8 * w;
        const float sc = 0.17677669529663687f * LOG2E; // 1/sqrt(32), exp2 domain
        int g = 0;                                      // chunks of this warpgroup so far
        bool ok = true;
        for (int k = w; ok; k += NWG) {
            const int st = k % ns;
            // warp-uniform outcomes: the tcgen05.ld / wait below are
            // warp-collective, so no lane may leave while the others load
            if (!__all_sync(0xffffffffu, bar_wait(full0 + 8 * st, (uint32_t)((k / ns) & 1), abort_flag, 3)))
                break;
            const uint8_t* sp = smem + (size_t)st * P.stage_bytes;
            const Meta m = read_meta(sp + P.mask_off + MASK_BYTES);
            if (m.n < 0) break;
            const uint32_t* kwp = (const uint32_t*)(sp + P.mask_off);
            const int nkc = (m.ext + KC - 1) / KC;
            float mrow = -INFINITY, l = 0.f;
            for (int c = 0; c < nkc && ok; c++) {
                const int nblk = (chunk_n(m.ext, c) + 31) >> 5;
                ok = __all_sync(0xffffffffu, bar_wait(sfull, (uint32_t)(g & 1), abort_flag, 4));
                if (!ok) break;
                tc_fence_after();
                // pass 1: the chunk's max over kept keys, 64 columns per
                // TMEM round trip (a select, not an add: columns past the
                // chunk's keys hold whatever TMEM held)
                float cm = -INFINITY;
                for (int hb = 0; 2 * hb < nblk; hb++) {
                    const uint32_t b0 = kwp[4 * c + 2 * hb];
                    const uint32_t b1 = 2 * hb + 1 < nblk ? kwp[4 * c + 2 * hb + 1] : 0u;
                    if (!(b0 | b1)) continue;
                    float v[64];
                    tmem_ld32x32(sb + 64 * hb, *(float(*)[32])v);
                    if (b1) tmem_ld32x32(sb + 64 * hb + 32, *(float(*)[32])(v + 32));
                    tmem_wait_ld();
                    cm = masked_max32(cm, v, b0);
                    if (b1) cm = masked_max32(cm, v + 32, b1);
                }
                const float mn = fmaxf(mrow, cm * sc);
                // O accumulates in TMEM (the PV MMAs of later chunks add to
                // it): once the previous chunk's PV landed, rescale O from
                // the previous max to this one; that also frees P
                if (c > 0) {
                    ok = __all_sync(0xffffffffu, bar_wait(pvfull, (uint32_t)((g - 1) & 1), abort_flag, 5));
                    if (!ok) break;
                    tc_fence_after();
                    float ov[DH];
                    tmem_ld32x32(pvb, ov);
                    tmem_wait_ld();
                    const float a = mrow == -INFINITY ? 0.f : ex2_approx(mrow - mn);
                    #pragma unroll
                    for (int d = 0; d < DH; d++) ov[d] *= a;
                    tmem_st32x32(pvb, ov);
                    tmem_wait_st();
                }
                // pass 2: P = exp2(s - max), 0 for masked keys, into the
                // K-major 128-byte-swizzled A operand: key k of row r in
                // 64-key block k / 64, 16-byte granule gi = (k % 64) / 8 at
                // gi ^ (r & 7)
                unsigned long long csum2 = 0ull;        // two fp32 partial sums
                const unsigned long long sc2 = splat2(sc), nm2 = splat2(-mn);
                for (int hb = 0; 2 * hb < nblk; hb++) {
                    const uint32_t b0 = kwp[4 * c + 2 * hb];
                    const bool two = 2 * hb + 1 < nblk;
                    const uint32_t b1 = two ? kwp[4 * c + 2 * hb + 1] : 0u;
                    uint8_t* rp = prow + hb * 16384;
                    if (!(b0 | b1)) {
                        #pragma unroll
                        for (int q = 0; q < 8; q++)
                            if (q < 4 || two)
                                *(uint4*)(rp + ((q ^ (row & 7)) << 4)) = make_uint4(0, 0, 0, 0);
                        continue;
                    }
                    float v[64];
                    tmem_ld32x32(sb + 64 * hb, *(float(*)[32])v);
                    if (b1) tmem_ld32x32(sb + 64 * hb + 32, *(float(*)[32])(v + 32));
                    tmem_wait_ld();
                    exp_block32(v, b0, sc2, nm2, csum2);
                    store_p32(rp, row, 0, v);
                    if (two) {
                        if (b1) {
                            exp_block32(v + 32, b1, sc2, nm2, csum2);
                            store_p32(rp, row, 4, v + 32);
                        } else {
                            #pragma unroll
                            for (int q = 4; q < 8; q++)
                                *(uint4*)(rp + ((q ^ (row & 7)) << 4)) = make_uint4(0, 0, 0, 0);
                        }
                    }
                }
                float cs0, cs1;
                upk2(csum2, cs0, cs1);
                const float csum = cs0 + cs1;
                const float alpha = mrow == -INFINITY ? 0.f : ex2_approx(mrow - mn);
                l = l * alpha + csum;
                mrow = mn;
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                tc_fence_before();
                bar_arrive(pready);                     // P written, S columns free
                g++;
            }
            if (!ok) break;
            // the last chunk's PV
            ok = __all_sync(0xffffffffu, bar_wait(pvfull, (uint32_t)((g - 1) & 1), abort_flag, 6));
            if (!ok) break;
            tc_fence_after();
            float o[DH];
            tmem_ld32x32(pvb, o);
            tmem_wait_ld();
            tc_fence_before();
            const int grow = m.qt * QT + row;           // row within the sequence
            if (grow < L) {
                bf16* orow = P.out + ((long)m.n * L + grow) * P.ldo + m.h * DH;
                float* lrow = P.lse + ((long)m.n * P.H + m.h) * L + grow;
                if (grow < m.ext) {
                    const float inv = 1.f / l;
                    #pragma unroll
                    for (int j = 0; j < 4; j++) {
                        uint4 q;
                        __nv_bfloat162* hq = (__nv_bfloat162*)&q;
                        #pragma unroll
                        for (int e = 0; e < 4; e++)
                            hq[e] = __floats2bfloat162_rn(o[8 * j + 2 * e] * inv, o[8 * j + 2 * e + 1] * inv);
                        ((uint4*)orow)[j] = q;
                    }
                    *lrow = (mrow + __log2f(l)) * 0.6931471805599453f;
                } else {
                    #pragma unroll
                    for (int j = 0; j < 4; j++) ((uint4*)orow)[j] = make_uint4(0, 0, 0, 0);
                    *lrow = 0.f;
                }
            }
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

// per sequence: the kept-key words and the extent, for callers that pass
// only the byte mask and (optionally) the extents
__global__ void k_keep_words(uint32_t* kw, const uint8_t* keep, const int* extent, int nseq, int L) {
    const int n = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (n >= nseq) return;
    const int ext = extent ? min(max(extent[n], 1), L) : L;
    uint32_t mine = 0;
    for (int j = 0; j < ATTN_KW_WORDS - 1; j++) {
        const int key = 32 * j + lane;
        const uint32_t b = __ballot_sync(0xffffffffu, key < ext && keep[(long)n * L + min(key, L - 1)]);
        if (lane == j) mine = b;
    }
    if (lane == ATTN_KW_WORDS - 1) mine = (uint32_t)ext;
    if (lane < ATTN_KW_WORDS) kw[(long)n * ATTN_KW_WORDS + lane] = mine;
}

template <int NWG>
size_t fwd_smem(uint32_t stage_bytes, int ns) {
    return 1024 + (size_t)ns * stage_bytes + (size_t)NWG * P_BYTES + 8 * (2 * 4 + 3 * 3 + 1) + 16;
}

template <int NWG>
bool launch_fwd(const CUtensorMap& qmap, const CUtensorMap& kmap, FwdParams P, long items,
                cudaStream_t s) {
    int ns = 0;
    while (ns < 4 && fwd_smem<NWG>(P.stage_bytes, ns + 1) <= (size_t)SMEM_MAX) ns++;
    // at least one stage per warpgroup: the end markers (one per warpgroup)
    // each need a stage that a live item released
    if (ns < NWG) return false;
    P.ns = ns;
    const size_t smem = fwd_smem<NWG>(P.stage_bytes, ns);
    if (cudaFuncSetAttribute(k_attn_fwd_tc<NWG>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    const int grid = (int)std::min<long>(items, tc_num_sms());
    ++g_ptcg_launches, k_attn_fwd_tc<NWG><<<grid, 64 + 128 * NWG, smem, s>>>(qmap, kmap, P);
    return true;
}

// ===================================================================== backward
// Work item = (sequence, head) whose extent is at most 128 rows: its queries
// and keys are one 128-row tile each (sequences past that are left to the
// mma.sync kernel).  Per item, with the thread of TMEM lane j owning key j:
//   S^T = K Q^T and dP^T = V dO^T (two SS MMAs into the warpgroup's TMEM);
//   P^T = exp2(S^T * sc - lse2) (0 for masked keys and for queries at or past
//   the extent), dS^T = P^T (dP^T - delta), delta = rowsum(dO * O) computed
//   from the staged dO and O tiles;
//   P^T goes back to TMEM (bf16) as the A operand of dV = P^T dO, dS^T to
//   shared memory, read K-major as the A operand of dK = dS^T Q and MN-major
//   as the A operand of dQ = dS K;
//   dQ, dK (scaled by 1/sqrt(32)) and dV rows go to dqkv, their fp32 column
//   sums to the bias gradient.
// Each warpgroup issues its own MMAs (one elected thread after a named
// barrier), so no MMA lane sits between the steps of an item; the producer
// warp keeps the stages (Q, K, V, dO, O tiles, log-sum-exps, key words) ahead.
constexpr int BWD_NWG = 2;
constexpr uint32_t DS_BYTES = 2 * 128 * 128;     // dS^T: 128 keys x 128 queries bf16
constexpr uint32_t BST_LSE = 5 * TILE_BYTES;     // stage: Q K V dO O tiles, then lse
constexpr uint32_t BST_MASK = BST_LSE + 512;
constexpr uint32_t BST_META = BST_MASK + MASK_BYTES;
constexpr uint32_t BST_BYTES = (BST_META + 16 + 1023) & ~1023u;

struct BwdParams {
    int nseq, L, H, D, ns;
    long lddq;
    bf16* dqkv;
    float* dbias;
    const float* lse;
    const uint32_t* kw;
};

PTCG_DEV void mma_bf16_ts(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
                 :: "r"(d), "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc) : "memory");
}
PTCG_DEV void named_sync(int id, int n) { asm volatile("bar.sync %0, %1;" :: "r"(id), "r"(n) : "memory"); }
// named barrier that also ANDs a flag over its threads, so that every thread
// of a warpgroup takes the same branch after a bounded wait
PTCG_DEV bool named_and(int id, int n, bool v) {
    uint32_t r;
    asm volatile("{\n\t.reg .pred p, q;\n\t"
                 "setp.ne.u32 p, %1, 0;\n\t"
                 "bar.red.and.pred q, %2, %3, p;\n\t"
                 "selp.u32 %0, 1, 0, q;\n\t}"
                 : "=r"(r) : "r"((uint32_t)v), "r"(id), "r"(n) : "memory");
    return r != 0;
}
PTCG_DEV void tmem_st32x32_x4(uint32_t taddr, const uint32_t (&v)[4]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1,%2,%3,%4};"
                 :: "r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]) : "memory");
}
PTCG_DEV uint32_t pack_bf2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *(uint32_t*)&h;
}
// lane c of the warp gets the sum over the warp's lanes of x[c] (x is
// destroyed): five butterfly stages, each halving the values a lane keeps
PTCG_DEV float warp_colsum32(float (&x)[32], int lane) {
    #pragma unroll
    for (int k = 16; k >= 1; k >>= 1) {
        const bool up = (lane & k) != 0;
        #pragma unroll
        for (int i = 0; i < k; i++) {
            const float send = up ? x[i] : x[i + k];
            const float keep = up ? x[i + k] : x[i];
            x[i] = keep + __shfl_xor_sync(0xffffffffu, send, k);
        }
    }
    return x[0];
}

__global__ void __launch_bounds__(32 + 128 * BWD_NWG, 1) k_attn_bwd_tc(
        const __grid_constant__ CUtensorMap qkv_map, const __grid_constant__ CUtensorMap do_map,
        const __grid_constant__ CUtensorMap o_map, const __grid_constant__ CUtensorMap kw_map,
        const __grid_constant__ BwdParams P) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    const int ns = P.ns, H = P.H, L = P.L, D = P.D;
    uint8_t* dsbuf = smem + (size_t)ns * BST_BYTES;                   // BWD_NWG x DS_BYTES
    float* rowv = (float*)(dsbuf + BWD_NWG * DS_BYTES);               // per WG: -lse2[128], -delta[128]
    float* acc = rowv + BWD_NWG * 256;                                // [3][H][32] bias-grad sums
    uint64_t* bars = (uint64_t*)(acc + 3 * 16 * 32);
    // full[ns] empty[ns] sfull[NWG] dfull[NWG] drain[NWG]
    uint32_t* tmem_slot = (uint32_t*)(bars + 2 * 4 + 3 * BWD_NWG);
    volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
    const uint32_t full0 = saddr(bars), empty0 = saddr(bars + ns);
    const uint32_t sfull0 = saddr(bars + 2 * ns), dfull0 = saddr(bars + 2 * ns + BWD_NWG);
    const uint32_t drain0 = saddr(bars + 2 * ns + 2 * BWD_NWG);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    for (int i = threadIdx.x; i < 3 * H * 32; i += blockDim.x) acc[i] = 0.f;
    if (threadIdx.x == 0) {
        for (int i = 0; i < ns; i++) { bar_init(full0 + 8 * i, 32); bar_init(empty0 + 8 * i, 1); }
        for (int w = 0; w < BWD_NWG; w++) {
            bar_init(sfull0 + 8 * w, 1); bar_init(dfull0 + 8 * w, 1); bar_init(drain0 + 8 * w, 1);
        }
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
    const long items = (long)P.nseq * H;

    if (warp == 0) {
        // ------------------------------------------------ producer warp
        int k = 0;
        bool ok = true;
        for (long base = blockIdx.x; base < items && ok; base += 32L * gridDim.x) {
            const long it = base + (long)lane * gridDim.x;
            const bool valid = it < items;
            int n = 0, h = 0, ext = 0;
            if (valid) {
                n = (int)(it / H);
                h = (int)(it - (long)n * H);
                ext = min(max((int)P.kw[(long)n * ATTN_KW_WORDS + ATTN_KW_WORDS - 1], 1), L);
            }
            const bool mine = valid && ext <= QT;
            // rows past the tile (L > 128): zero dQ, dK, dV
            unsigned zm = L > QT ? __ballot_sync(0xffffffffu, mine) : 0u;
            while (zm) {
                const int i = __ffs(zm) - 1;
                zm &= zm - 1;
                const int zn = __shfl_sync(0xffffffffu, n, i), zh = __shfl_sync(0xffffffffu, h, i);
                for (int e = lane; e < (L - QT) * 12; e += 32) {
                    const int r = QT + e / 12, part = (e % 12) >> 2;
                    *(uint4*)(P.dqkv + ((long)zn * L + r) * P.lddq + part * D + zh * DH + (e & 3) * 8) =
                        make_uint4(0, 0, 0, 0);
                }
            }
            unsigned am = __ballot_sync(0xffffffffu, mine);
            while (am) {
                const int i = __ffs(am) - 1;
                am &= am - 1;
                const int mn_ = __shfl_sync(0xffffffffu, n, i);
                const int mh = __shfl_sync(0xffffffffu, h, i);
                const int me = __shfl_sync(0xffffffffu, ext, i);
                // this item's log-sum-exps, 4 rows a lane (rows >= L read as 0)
                const float* lrow = P.lse + ((long)mn_ * H + mh) * L;
                float lv[4];
                #pragma unroll
                for (int q = 0; q < 4; q++) lv[q] = 4 * lane + q < min(L, QT) ? lrow[4 * lane + q] : 0.f;
                const int st = k % ns;
                if (lane == 0 &&
                    !bar_wait(empty0 + 8 * st, (uint32_t)(((k / ns) & 1) ^ 1), abort_flag, 11))
                    ok = false;
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) break;
                uint8_t* sp = smem + (size_t)st * BST_BYTES;
                *(float4*)(sp + BST_LSE + 16 * lane) = make_float4(lv[0], lv[1], lv[2], lv[3]);
                if (lane == 0) {
                    int* meta = (int*)(sp + BST_META);
                    meta[0] = mn_; meta[1] = mh; meta[2] = me;
                    const uint32_t fb = full0 + 8 * st;
                    bar_expect_tx(fb, 5 * TILE_BYTES + MASK_BYTES);
                    const uint32_t sb = saddr(sp);
                    const int row0 = mn_ * L;
                    tma_2d(sb, &qkv_map, fb, mh * DH, row0);
                    tma_2d(sb + TILE_BYTES, &qkv_map, fb, D + mh * DH, row0);
                    tma_2d(sb + 2 * TILE_BYTES, &qkv_map, fb, 2 * D + mh * DH, row0);
                    tma_2d(sb + 3 * TILE_BYTES, &do_map, fb, mh * DH, row0);
                    tma_2d(sb + 4 * TILE_BYTES, &o_map, fb, mh * DH, row0);
                    tma_2d(sb + BST_MASK, &kw_map, fb, 0, mn_);
                } else {
                    bar_arrive(full0 + 8 * st);
                }
                k++;
            }
        }
        // one end marker per warpgroup
        for (int w = 0; w < BWD_NWG && ok; w++) {
            const int st = k % ns;
            if (lane == 0 &&
                !bar_wait(empty0 + 8 * st, (uint32_t)(((k / ns) & 1) ^ 1), abort_flag, 11))
                ok = false;
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            if (lane == 0) ((int*)(smem + (size_t)st * BST_BYTES + BST_META))[0] = -1;
            bar_arrive(full0 + 8 * st);
            k++;
        }
        if (lane == 0 && *abort_flag)
            for (int j = max(0, k - ns); j < k; j++)
                bar_drain(full0 + 8 * (j % ns), (uint32_t)((j / ns) & 1));
    } else {
        // ------------------------------------------------ warpgroups
        const int w = (warp - 1) >> 2;
        const int quad = warp & 3;
        const int row = quad * 32 + lane;               // key j (and query j for dQ) = TMEM lane
        const int wtid = threadIdx.x - 32 - 128 * w;    // 0..127 within the warpgroup
        const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
        const uint32_t c0 = (uint32_t)(w * 256);
        const uint32_t t_s = tmem + lane_off + c0;      // S^T, then P^T (bf16) in its first 64 columns
        const uint32_t t_dp = t_s + 128;                // dP^T
        const uint32_t t_dv = t_s + 64, t_dk = t_s + 96, t_dq = t_s + 128;
        uint8_t* ds = dsbuf + w * DS_BYTES;
        uint8_t* dsrow = ds + row * 128;
        float* nl2 = rowv + w * 256;                    // -lse * log2(e) per query
        float* nd = nl2 + 128;                          // -delta per query
        const uint32_t sfull = sfull0 + 8 * w, dfull = dfull0 + 8 * w;
        const int bar_id = 1 + w;
        const float sc = 0.17677669529663687f * LOG2E;
        const float scale = 0.17677669529663687f;
        int g = 0;
        for (int k = w;; k += BWD_NWG) {
            const int st = k % ns;
            if (!named_and(bar_id, 128, bar_wait(full0 + 8 * st, (uint32_t)((k / ns) & 1), abort_flag, 12)))
                break;
            const uint8_t* sp = smem + (size_t)st * BST_BYTES;
            const volatile int* meta = (const volatile int*)(sp + BST_META);
            const int n = meta[0];
            if (n < 0) break;
            const int h = meta[1], ext = meta[2];
            const uint32_t sb = saddr(sp);
            const int nq = (ext + 15) & ~15;            // queries (and keys) the MMAs cover
            const int nblk = (nq + 31) >> 5;
            if (wtid == 0) {
                tc_fence_after();
                const uint32_t id = idesc_bf16(nq, 0, 0);
                #pragma unroll
                for (int s = 0; s < 2; s++) {           // S^T = K Q^T, dP^T = V dO^T
                    mma_bf16(t_s - lane_off, sdesc(sb + TILE_BYTES + 32 * s, 16, 512, 4),
                             sdesc(sb + 32 * s, 16, 512, 4), id, s > 0 ? 1u : 0u);
                    mma_bf16(t_dp - lane_off, sdesc(sb + 2 * TILE_BYTES + 32 * s, 16, 512, 4),
                             sdesc(sb + 3 * TILE_BYTES + 32 * s, 16, 512, 4), id, s > 0 ? 1u : 0u);
                }
                mma_commit_to(sfull);
            }
            // delta_t = dO_t . O_t and -lse2_t for query t = this thread's row
            // (64-byte swizzle: granule q of row t at q ^ ((t >> 1) & 3))
            {
                const uint8_t* dorow = sp + 3 * TILE_BYTES + row * 64;
                const uint8_t* orow = sp + 4 * TILE_BYTES + row * 64;
                float d = 0.f;
                #pragma unroll
                for (int q = 0; q < 4; q++) {
                    const int off = (q ^ ((row >> 1) & 3)) << 4;
                    const uint4 a = *(const uint4*)(dorow + off), b = *(const uint4*)(orow + off);
                    const __nv_bfloat162* ha = (const __nv_bfloat162*)&a;
                    const __nv_bfloat162* hb = (const __nv_bfloat162*)&b;
                    #pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const float2 x = __bfloat1622float2(ha[e]), y = __bfloat1622float2(hb[e]);
                        d = fmaf(x.x, y.x, fmaf(x.y, y.y, d));
                    }
                }
                const bool live = row < ext;
                nd[row] = live ? -d : 0.f;
                nl2[row] = live ? -((const float*)(sp + BST_LSE))[row] * LOG2E : 0.f;
            }
            named_sync(bar_id, 128);
            const uint32_t* kwp = (const uint32_t*)(sp + BST_MASK);
            const bool kept = row < ext && ((kwp[row >> 5] >> (row & 31)) & 1u);
            if (!named_and(bar_id, 128, bar_wait(sfull, (uint32_t)(g & 1), abort_flag, 13))) break;
            tc_fence_after();
            // P^T and dS^T, 32 queries at a time.  tcgen05.ld / wait are
            // warp-collective: a warp loads when any of its keys is kept,
            // and each thread then masks its own row
            const bool wkept = __any_sync(0xffffffffu, kept);
            const unsigned long long sc2 = splat2(sc);
            for (int b = 0; b < nblk; b++) {
                float s[32], dp[32];
                if (wkept) {
                    tmem_ld32x32(t_s + 32 * b, s);
                    tmem_ld32x32(t_dp + 32 * b, dp);
                    tmem_wait_ld();
                }
                // 8 queries at a time: their P^T (4 TMEM columns, bf16
                // pairs) and dS^T (one 16-byte granule of the swizzled row)
                const float* l2 = nl2 + 32 * b;
                const float* dl = nd + 32 * b;
                const int lim = ext - 32 * b;           // queries of this block below the extent
                uint8_t* rp = dsrow + (b >> 1) * 16384;
                #pragma unroll
                for (int q = 0; q < 4; q++) {
                    uint32_t pp[4] = {0u, 0u, 0u, 0u}, dd[4] = {0u, 0u, 0u, 0u};
                    if (kept) {
                        #pragma unroll
                        for (int e = 0; e < 4; e++) {
                            const int i = 8 * q + 2 * e;
                            float p0, p1;
                            upk2(fma2(pk2(s[i], s[i + 1]), sc2, pk2(l2[i], l2[i + 1])), p0, p1);
                            p0 = i < lim ? ex2_approx(p0) : 0.f;
                            p1 = i + 1 < lim ? ex2_approx(p1) : 0.f;
                            float t0, t1;
                            upk2(mul2(pk2(p0, p1), add2(pk2(dp[i], dp[i + 1]), pk2(dl[i], dl[i + 1]))),
                                 t0, t1);
                            // past the extent dP^T columns may hold anything (0 * NaN)
                            t0 = i < lim ? t0 : 0.f;
                            t1 = i + 1 < lim ? t1 : 0.f;
                            pp[e] = pack_bf2(p0, p1);
                            dd[e] = pack_bf2(t0, t1);
                        }
                    }
                    // P^T over S^T columns already read (block b / 2 <= b)
                    tmem_st32x32_x4(t_s + 16 * b + 4 * q, pp);
                    *(uint4*)(rp + ((((b & 1) * 4 + q) ^ (row & 7)) << 4)) =
                        make_uint4(dd[0], dd[1], dd[2], dd[3]);
                }
            }
            tmem_wait_st();
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            tc_fence_before();
            named_sync(bar_id, 128);
            if (wtid == 0) {
                tc_fence_after();
                const uint32_t dsa = saddr(ds);
                const uint32_t id = idesc_bf16(DH, 0, 1);          // B MN-major
                const uint32_t idq = idesc_bf16(DH, 1, 1);         // A and B MN-major
                for (int s = 0; s < nq / 16; s++) {
                    // dV += P^T dO (A = P^T from TMEM, K = queries)
                    mma_bf16_ts(t_dv - lane_off, t_s - lane_off + 8 * s,
                                sdesc(sb + 3 * TILE_BYTES + s * 1024, TILE_BYTES, 512, 4), id,
                                s > 0 ? 1u : 0u);
                    // dK += dS^T Q (A = dS^T K-major, K = queries)
                    mma_bf16(t_dk - lane_off, sdesc(dsa + (s >> 2) * 16384 + (s & 3) * 32, 16, 1024, 2),
                             sdesc(sb + s * 1024, TILE_BYTES, 512, 4), id, s > 0 ? 1u : 0u);
                    // dQ += dS K (A = dS^T read MN-major, K = keys)
                    mma_bf16(t_dq - lane_off, sdesc(dsa + s * 2048, 16384, 1024, 2),
                             sdesc(sb + TILE_BYTES + s * 1024, TILE_BYTES, 512, 4), idq,
                             s > 0 ? 1u : 0u);
                }
                mma_commit_to(dfull);
                mma_commit_to(empty0 + 8 * st);     // the stage is free once these land
            }
            if (!named_and(bar_id, 128, bar_wait(dfull, (uint32_t)(g & 1), abort_flag, 14))) break;
            tc_fence_after();
            g++;
            // rows of dQ (query j), dK and dV (key j); fp32 column sums
            float x[32];
            bf16* drow = P.dqkv + ((long)n * L + row) * P.lddq + h * DH;
            #pragma unroll
            for (int part = 0; part < 3; part++) {
                tmem_ld32x32(part == 0 ? t_dq : part == 1 ? t_dk : t_dv, x);
                tmem_wait_ld();
                if (part < 2) {
                    // dQ rows at or past the extent read dS^T columns this
                    // item did not write (anything, NaN included): a select,
                    // not a multiply by 0 (nothing downstream reads them)
                    const bool zero = part == 0 && row >= ext;
                    #pragma unroll
                    for (int i = 0; i < 32; i++) x[i] = zero ? 0.f : x[i] * scale;
                }
                if (row < L) {
                    #pragma unroll
                    for (int q = 0; q < 4; q++)
                        *(uint4*)(drow + part * D + 8 * q) =
                            make_uint4(pack_bf2(x[8 * q], x[8 * q + 1]), pack_bf2(x[8 * q + 2], x[8 * q + 3]),
                                       pack_bf2(x[8 * q + 4], x[8 * q + 5]), pack_bf2(x[8 * q + 6], x[8 * q + 7]));
                } else {
                    #pragma unroll
                    for (int i = 0; i < 32; i++) x[i] = 0.f;
                }
                if (P.dbias) {
                    const float cs = warp_colsum32(x, lane);
                    atomicAdd(&acc[(part * H + h) * 32 + lane], cs);
                }
            }
            // TMEM read before the next item's MMAs overwrite it
            tc_fence_before();
            named_sync(bar_id, 128);
        }
        // no MMA of this warpgroup may still be in flight when TMEM is freed
        if (wtid == 0) {
            mma_commit_to(drain0 + 8 * w);
            bar_drain(drain0 + 8 * w, 0);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (P.dbias)
        for (int i = threadIdx.x; i < 3 * H * 32; i += blockDim.x) {
            const float v = acc[i];
            if (v != 0.f) atomicAdd(&P.dbias[(i / (H * 32)) * D + (i % (H * 32))], v);
        }
    if (warp == 1) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
                     :: "r"(tmem), "r"(512) : "memory");
    }
}

}  // namespace

int attn_tc_error_read_reset() {
    int v = 0, zero = 0;
    cudaMemcpyFromSymbol(&v, g_attn_tc_error, sizeof(int));
    cudaMemcpyToSymbol(g_attn_tc_error, &zero, sizeof(int));
    return v;
}

void attn_keep_words(uint32_t* kw, const uint8_t* keep, const int* extent, int nseq, int L,
                     cudaStream_t s) {
    if (nseq <= 0) return;
    ++g_ptcg_launches, k_keep_words<<<(nseq + 7) / 8, 256, 0, s>>>(kw, keep, extent, nseq, L);
}

bool attn_fwd_tc(const void* qkv, long ldqkv, const uint32_t* kw, void* out, long ldo,
                 float* lse, int nseq, int L, int H, cudaStream_t s) {
    if (H * DH > 4096 || L > MAXC * KC || L < 1 || nseq <= 0 || !kw) return false;
    if (((uintptr_t)qkv & 15) || ((ldqkv * 2) % 16) || ((uintptr_t)out & 15) || (ldo % 8) ||
        ((uintptr_t)kw & 15))
        return false;
    const int D = H * DH;
    CUtensorMap qmap, kmap;
    if (!tc_make_map_2d(&qmap, qkv, DT_BF16, 3L * D, (long)nseq * L, ldqkv, DH, 128, 64))
        return false;
    if (!tc_make_map_2d(&kmap, kw, DT_F32, ATTN_KW_WORDS, nseq, ATTN_KW_WORDS, ATTN_KW_WORDS, 1, 0))
        return false;
    FwdParams P;
    P.nseq = nseq; P.L = L; P.H = H; P.D = D;
    P.nqt = (L + QT - 1) / QT;
    P.maxc = (L + KC - 1) / KC;
    P.ns = 0;
    P.ldo = ldo;
    P.out = (bf16*)out; P.lse = lse; P.kw = kw;
    P.mask_off = TILE_BYTES * (1 + 2 * P.maxc);
    P.stage_bytes = (P.mask_off + MASK_BYTES + (uint32_t)sizeof(Meta) + 1023) & ~1023u;
    const long items = (long)nseq * H * P.nqt;
    return launch_fwd<3>(qmap, kmap, P, items, s) || launch_fwd<2>(qmap, kmap, P, items, s);
}

bool attn_bwd_tc(const void* qkv, long ldqkv, const uint32_t* kw, const void* out, long ldo,
                 const void* dout, long lddo, const float* lse, void* dqkv, long lddqkv,
                 float* dbias, int nseq, int L, int H, cudaStream_t s) {
    if (H > 16 || L < 1 || nseq <= 0 || !kw) return false;
    if (((uintptr_t)qkv & 15) || ((ldqkv * 2) % 16) || ((uintptr_t)out & 15) || (ldo % 8) ||
        ((uintptr_t)dout & 15) || (lddo % 8) || ((uintptr_t)dqkv & 15) || (lddqkv % 8) ||
        ((uintptr_t)kw & 15))
        return false;
    const int D = H * DH;
    CUtensorMap qmap, dmap, omap, kmap;
    if (!tc_make_map_2d(&qmap, qkv, DT_BF16, 3L * D, (long)nseq * L, ldqkv, DH, 128, 64) ||
        !tc_make_map_2d(&dmap, dout, DT_BF16, D, (long)nseq * L, lddo, DH, 128, 64) ||
        !tc_make_map_2d(&omap, out, DT_BF16, D, (long)nseq * L, ldo, DH, 128, 64) ||
        !tc_make_map_2d(&kmap, kw, DT_F32, ATTN_KW_WORDS, nseq, ATTN_KW_WORDS, ATTN_KW_WORDS, 1, 0))
        return false;
    BwdParams P;
    P.nseq = nseq; P.L = L; P.H = H; P.D = D;
    P.lddq = lddqkv;
    P.dqkv = (bf16*)dqkv; P.dbias = dbias; P.lse = lse; P.kw = kw;
    auto need = [](int ns) {
        return 1024 + (size_t)ns * BST_BYTES + (size_t)BWD_NWG * DS_BYTES + BWD_NWG * 256 * 4 +
               3 * 16 * 32 * 4 + 8 * (2 * 4 + 3 * BWD_NWG) + 16;
    };
    int ns = 0;
    while (ns < 4 && need(ns + 1) <= (size_t)SMEM_MAX) ns++;
    if (ns < BWD_NWG) return false;
    P.ns = ns;
    const size_t smem = need(ns);
    if (cudaFuncSetAttribute(k_attn_bwd_tc, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    const long items = (long)nseq * H;
    const int grid = (int)std::min<long>(items, tc_num_sms());
    ++g_ptcg_launches, k_attn_bwd_tc<<<grid, 32 + 128 * BWD_NWG, smem, s>>>(qmap, dmap, omap, kmap, P);
    return true;
}
