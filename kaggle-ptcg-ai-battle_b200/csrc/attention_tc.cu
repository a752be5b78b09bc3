// Masked multi-head attention on the 5th-generation tensor cores (tcgen05 /
// TMEM / TMA), bf16 operands, head width 32, fp32 softmax.  Semantics as the
// other attention paths (attention.cu): torch F.scaled_dot_product_attention
// with a boolean key-padding mask (ptcg/rl/model.py:86-89), scale 1/sqrt(32);
// the forward saves the per-row log-sum-exp; query rows at or past a
// sequence's row extent get zero output and a zero log-sum-exp.
//
// Work item = (sequence, head, 128-row query tile).  Per item:
//  * one TMA producer lane loads the Q tile [128 x 32] and the sequence's
//    keys / values in chunks of 128 rows ({32 cols, 128 rows} boxes, 64-byte
//    swizzle) into one of two shared-memory stages;
//  * one MMA lane issues S = Q K^T for each key chunk into a TMEM
//    accumulator (M = 128 query rows = TMEM lanes, N = keys of the chunk,
//    K = 32 as two kind::f16 instructions), and, once the softmax has written
//    P for that chunk, PV = P V (A = P from shared memory, K-major 128-byte
//    swizzle; B = V, MN-major 64-byte swizzle, N = 32) into a second TMEM
//    accumulator;
//  * four softmax warps, one per TMEM lane quadrant, so that each thread owns
//    one query row: they read the row's scores with tcgen05.ld, apply the key
//    mask, keep the running max / sum of an online softmax across chunks in
//    the exp2 domain, write P (bf16) into the swizzled A-operand layout, and
//    accumulate O = O * alpha + PV in registers.
// S and PV accumulators are double-buffered, so the next chunk's (or item's)
// S = Q K^T runs while the softmax works on the current one.  Only keys below
// the sequence's row extent are loaded or multiplied (keys past it are
// masked by construction); query tiles starting past it are zero-filled.
//
// Every mbarrier wait is bounded by a clock budget: on expiry the CTA records
// an error code (attn_tc_error_read_reset), stops waiting, lets its issued
// copies and MMAs land, frees its TMEM and returns.
#include "common.cuh"
#include "internal.h"

#include <algorithm>

namespace {

constexpr int DH = 32;                 // head width
constexpr int QT = 128;                // query rows per tile (MMA M, TMEM lanes)
constexpr int KC = 128;                // keys per chunk (S accumulator columns)
constexpr int MAXC = 3;                // key chunks per sequence: L <= 384
constexpr int NSOFT = 4;               // softmax warps, one per TMEM lane quadrant
constexpr int FWD_THREADS = 64 + 32 * NSOFT;
constexpr uint32_t TILE_BYTES = 128 * DH * 2;   // one {32 cols, 128 rows} bf16 box: 8 KB
constexpr uint32_t P_BYTES = 2 * 128 * 128;     // P: 128 rows x 128 keys bf16, two 64-key blocks
constexpr long long WAIT_BUDGET = 4000000000LL; // clock cycles (~2 s)
constexpr float LOG2E = 1.4426950408889634f;

__device__ int g_attn_tc_error;

// ------------------------------------------------------------ PTX helpers
PTCG_DEV uint32_t saddr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
PTCG_DEV void bar_init(uint32_t b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(b), "r"(count));
}
PTCG_DEV void bar_expect_tx(uint32_t b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(b), "r"(bytes)
                 : "memory");
}
PTCG_DEV void bar_arrive(uint32_t b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(b) : "memory");
}
PTCG_DEV bool bar_try(uint32_t b, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred P;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, P;\n\t}"
                 : "=r"(ok) : "r"(b), "r"(parity) : "memory");
    return ok != 0;
}
// bounded wait; false once the CTA's abort flag is set (by this wait on
// expiry, recording `code`, or by another role)
PTCG_DEV bool bar_wait(uint32_t b, uint32_t parity, volatile int* abort_flag, int code) {
    if (*abort_flag) return false;
    const long long t0 = clock64();
    while (!bar_try(b, parity)) {
        if (*abort_flag) return false;
        if (clock64() - t0 > WAIT_BUDGET) {
            *abort_flag = 1;
            atomicCAS(&g_attn_tc_error, 0, code);
            return false;
        }
    }
    return true;
}
// wait for a barrier phase regardless of the abort flag, still bounded (the
// exit path: copies already issued must land before the CTA leaves)
PTCG_DEV void bar_drain(uint32_t b, uint32_t parity) {
    const long long t0 = clock64();
    while (!bar_try(b, parity) && clock64() - t0 < WAIT_BUDGET) {}
}
PTCG_DEV void tma_2d(uint32_t dst, const CUtensorMap* map, uint32_t b, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%3, %4}], [%2];"
                 :: "r"(dst), "l"((uint64_t)map), "r"(b), "r"(x), "r"(y) : "memory");
}
PTCG_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
PTCG_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
PTCG_DEV void mma_bf16(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
                 :: "r"(d), "l"(a), "l"(b), "r"(idesc), "r"(acc) : "memory");
}
PTCG_DEV void mma_commit_to(uint32_t b) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(b) : "memory");
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
PTCG_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// UMMA shared-memory descriptor (sm_100): start, leading / stride byte
// offsets, layout (2 = 128-byte swizzle, 4 = 64-byte swizzle)
PTCG_DEV uint64_t sdesc(uint32_t a, uint32_t lbo, uint32_t sbo, uint32_t layout) {
    uint64_t d = 0;
    d |= (uint64_t)((a >> 4) & 0x3FFF);
    d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)layout << 61;
    return d;
}
// instruction descriptor, kind::f16: fp32 accumulate, bf16 A and B, A / B
// major-ness (1 = MN-major), N, M = 128
__host__ __device__ inline uint32_t idesc_bf16(int n, int a_mn, int b_mn) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) |
           ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}
PTCG_DEV void named_sync(int id, int n) { asm volatile("bar.sync %0, %1;" :: "r"(id), "r"(n) : "memory"); }

struct FwdParams {
    int nseq, L, H, D;
    int nqt;                  // query tiles per (sequence, head)
    int maxc;                 // key chunks staged per item: ceil(L / KC)
    long ldo;
    bf16* out;
    float* lse;
    const uint8_t* keep;
    const int* ext;
    uint32_t stage_bytes;     // Q tile + maxc K chunks + maxc V chunks
};

struct Item {
    int n, h, qt, ext, nkc;
    bool active;
};

PTCG_DEV Item decode(const FwdParams& P, int it) {
    Item t;
    const int per_seq = P.H * P.nqt;
    t.n = it / per_seq;
    const int r = it - t.n * per_seq;
    t.h = r / P.nqt;
    t.qt = r - t.h * P.nqt;
    t.ext = P.ext ? min(max(P.ext[t.n], 1), P.L) : P.L;
    t.active = t.qt * QT < t.ext;
    t.nkc = (t.ext + KC - 1) / KC;
    return t;
}
// keys of chunk c, rounded up to the MMA's N granule of 16
PTCG_DEV int chunk_n(int ext, int c) { return min(KC, (ext - c * KC + 15) & ~15); }

// smem map: [stage 0 | stage 1] (each: Q, K chunks, V chunks), P (two
// 64-key blocks of 128 x 128 B), key bias [MAXC * KC] floats, barriers
__global__ void __launch_bounds__(FWD_THREADS, 1) k_attn_fwd_tc(
        const __grid_constant__ CUtensorMap qkv_map, const __grid_constant__ FwdParams P) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* pbuf = smem + 2 * P.stage_bytes;
    float* kbias = (float*)(pbuf + P_BYTES);
    uint64_t* bars = (uint64_t*)(kbias + MAXC * KC);
    // bars: full[2] empty[2] sfull[2] sempty[2] pfull pvfull[2] pvempty[2] drain
    uint32_t* tmem_slot = (uint32_t*)(bars + 14);
    volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
    const uint32_t full0 = saddr(bars), empty0 = saddr(bars + 2);
    const uint32_t sfull0 = saddr(bars + 4), sempty0 = saddr(bars + 6);
    const uint32_t pfull = saddr(bars + 8), pvfull0 = saddr(bars + 9), pvempty0 = saddr(bars + 11);
    const uint32_t drain = saddr(bars + 13);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; i++) {
            bar_init(full0 + 8 * i, 1); bar_init(empty0 + 8 * i, 1);
            bar_init(sfull0 + 8 * i, 1); bar_init(sempty0 + 8 * i, 32 * NSOFT);
            bar_init(pvfull0 + 8 * i, 1); bar_init(pvempty0 + 8 * i, 32 * NSOFT);
        }
        bar_init(pfull, 32 * NSOFT);
        bar_init(drain, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {
        // S double buffer (2 x 128 columns) + PV double buffer (2 x 32)
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(saddr(tmem_slot)), "r"(512) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int items = P.nseq * P.H * P.nqt;
    const int D = P.D;

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            int stage = 0, issued = 0;
            uint32_t ph = 0;
            for (int it = blockIdx.x; it < items; it += gridDim.x) {
                const Item t = decode(P, it);
                if (!t.active) continue;
                if (!bar_wait(empty0 + 8 * stage, ph ^ 1, abort_flag, 1)) break;
                const uint32_t fb = full0 + 8 * stage;
                bar_expect_tx(fb, TILE_BYTES * (1 + 2 * t.nkc));
                const uint32_t base = saddr(smem + (size_t)stage * P.stage_bytes);
                const int row0 = t.n * P.L;
                tma_2d(base, &qkv_map, fb, t.h * DH, row0 + t.qt * QT);
                for (int c = 0; c < t.nkc; c++) {
                    tma_2d(base + TILE_BYTES * (1 + c), &qkv_map, fb, D + t.h * DH, row0 + c * KC);
                    tma_2d(base + TILE_BYTES * (1 + P.maxc + c), &qkv_map, fb, 2 * D + t.h * DH,
                           row0 + c * KC);
                }
                issued++;
                if (++stage == 2) { stage = 0; ph ^= 1; }
            }
            // on an abort, let the copies of the (at most two) stages still
            // in flight land before the CTA can exit
            if (*abort_flag) {
                for (int k = 1; k <= 2 && k <= issued; k++) {
                    const int idx = issued - k;
                    bar_drain(full0 + 8 * (idx & 1), (uint32_t)((idx >> 1) & 1));
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            int stage = 0;
            uint32_t ph = 0;
            int gc = 0;                         // key chunks processed by this CTA
            bool ok = true;
            const uint32_t pbase = saddr(pbuf);
            for (int it = blockIdx.x; it < items && ok; it += gridDim.x) {
                const Item t = decode(P, it);
                if (!t.active) continue;
                if (!bar_wait(full0 + 8 * stage, ph, abort_flag, 2)) break;
                tc_fence_after();
                const uint32_t base = saddr(smem + (size_t)stage * P.stage_bytes);
                // S = Q K^T for chunk c into S buffer (gc + c) & 1
                auto issue_s = [&](int c) -> bool {
                    const int g = gc + c, b = g & 1;
                    if (!bar_wait(sempty0 + 8 * b, ((g >> 1) & 1) ^ 1, abort_flag, 3)) return false;
                    tc_fence_after();
                    const uint32_t kb = base + TILE_BYTES * (1 + c);
                    const uint32_t id = idesc_bf16(chunk_n(t.ext, c), 0, 0);
                    #pragma unroll
                    for (int s = 0; s < 2; s++)
                        mma_bf16(tmem + b * KC, sdesc(base + 32 * s, 16, 512, 4),
                                 sdesc(kb + 32 * s, 16, 512, 4), id, s > 0 ? 1u : 0u);
                    mma_commit_to(sfull0 + 8 * b);
                    return true;
                };
                if (!issue_s(0)) { ok = false; break; }
                for (int c = 0; c < t.nkc && ok; c++) {
                    if (c + 1 < t.nkc && !issue_s(c + 1)) { ok = false; break; }
                    const int g = gc + c, b = g & 1;
                    // PV = P V once the softmax has written P for this chunk
                    if (!bar_wait(pfull, (uint32_t)(g & 1), abort_flag, 4) ||
                        !bar_wait(pvempty0 + 8 * b, ((g >> 1) & 1) ^ 1, abort_flag, 5)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t vb = base + TILE_BYTES * (1 + P.maxc + c);
                    const uint32_t id = idesc_bf16(DH, 0, 1);
                    const int ks = chunk_n(t.ext, c) / 16;
                    for (int s = 0; s < ks; s++)
                        mma_bf16(tmem + 2 * KC + b * DH,
                                 sdesc(pbase + (s >> 2) * 16384 + (s & 3) * 32, 16, 1024, 2),
                                 sdesc(vb + s * 1024, TILE_BYTES, 512, 4), id, s > 0 ? 1u : 0u);
                    mma_commit_to(pvfull0 + 8 * b);
                }
                if (!ok) break;
                gc += t.nkc;
                mma_commit_to(empty0 + 8 * stage);      // Q / K / V of this stage consumed
                if (++stage == 2) { stage = 0; ph ^= 1; }
            }
            // no MMA may still be in flight when TMEM is released
            mma_commit_to(drain);
            bar_drain(drain, 0);
        }
        __syncwarp();
    } else {
        // ------------------------------------------------ softmax warps
        const int quad = warp & 3;
        const int row = quad * 32 + lane;               // query row within the tile = TMEM lane
        const int tid = threadIdx.x - 64;               // 0..127
        const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
        const float sc = 0.17677669529663687f * LOG2E; // 1/sqrt(32), exp2 domain
        int gc = 0;
        bool ok = true;
        for (int it = blockIdx.x; it < items; it += gridDim.x) {
            const Item t = decode(P, it);
            const int grow = t.qt * QT + row;           // row within the sequence
            bf16* orow = P.out + ((long)t.n * P.L + grow) * P.ldo + t.h * DH;
            float* lrow = P.lse + ((long)t.n * P.H + t.h) * P.L + grow;
            named_sync(1, 32 * NSOFT);                  // the previous item is done with kbias
            if (!t.active) {
                if (grow < P.L) {
                    #pragma unroll
                    for (int j = 0; j < 4; j++) ((uint4*)orow)[j] = make_uint4(0, 0, 0, 0);
                    *lrow = 0.f;
                }
                continue;
            }
            const uint8_t* kp = P.keep + (long)t.n * P.L;
            for (int j = tid; j < t.nkc * KC; j += 32 * NSOFT)
                kbias[j] = (j < t.ext && kp[j]) ? 0.f : -INFINITY;
            named_sync(1, 32 * NSOFT);
            float m = -INFINITY, l = 0.f;
            float o[DH];
            #pragma unroll
            for (int d = 0; d < DH; d++) o[d] = 0.f;
            for (int c = 0; c < t.nkc; c++) {
                const int g = gc + c, b = g & 1;
                const int nc = chunk_n(t.ext, c), nblk = (nc + 31) >> 5;
                const uint32_t sb = tmem + lane_off + b * KC;
                ok = ok && bar_wait(sfull0 + 8 * b, (uint32_t)((g >> 1) & 1), abort_flag, 6);
                // pass 1: the chunk's max over kept keys (masking is a select,
                // not an add: columns past the chunk's keys hold whatever TMEM
                // held, which need not be a finite number)
                float cm = -INFINITY;
                if (ok) {
                    tc_fence_after();
                    for (int j = 0; j < nblk; j++) {
                        float v[32];
                        tmem_ld32x32(sb + 32 * j, v);
                        tmem_wait_ld();
                        #pragma unroll
                        for (int i = 0; i < 32; i++)
                            if (kbias[c * KC + 32 * j + i] == 0.f) cm = fmaxf(cm, v[i] * sc);
                    }
                }
                const float mn = fmaxf(m, cm);
                const float alpha = m == -INFINITY ? 0.f : ex2_approx(m - mn);
                // pass 2: P = exp2(s - max) (0 for masked keys) into the
                // K-major 128-byte-swizzled A operand: key k of row r in
                // 64-key block k / 64, 16-byte granule gi = (k % 64) / 8 at
                // gi ^ (r & 7)
                float csum = 0.f;
                for (int j = 0; j < nblk; j++) {
                    float v[32];
                    if (ok) {
                        tmem_ld32x32(sb + 32 * j, v);
                        tmem_wait_ld();
                    }
                    #pragma unroll
                    for (int i = 0; i < 32; i++) {
                        const bool kept = ok && kbias[c * KC + 32 * j + i] == 0.f;
                        v[i] = kept ? ex2_approx(fmaf(v[i], sc, -mn)) : 0.f;
                        csum += v[i];
                    }
                    uint8_t* rowp = pbuf + (j >> 1) * 16384 + row * 128;
                    #pragma unroll
                    for (int q4 = 0; q4 < 4; q4++) {
                        const int gi = (j & 1) * 4 + q4;
                        uint4 q;
                        __nv_bfloat162* hq = (__nv_bfloat162*)&q;
                        #pragma unroll
                        for (int e = 0; e < 4; e++)
                            hq[e] = __floats2bfloat162_rn(v[8 * q4 + 2 * e], v[8 * q4 + 2 * e + 1]);
                        *(uint4*)(rowp + ((gi ^ (row & 7)) << 4)) = q;
                    }
                }
                tc_fence_before();
                bar_arrive(sempty0 + 8 * b);            // the S buffer may be overwritten
                l = l * alpha + csum;
                m = mn;
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                bar_arrive(pfull);
                float pv[DH];
                ok = ok && bar_wait(pvfull0 + 8 * b, (uint32_t)((g >> 1) & 1), abort_flag, 7);
                if (ok) {
                    tc_fence_after();
                    tmem_ld32x32(tmem + lane_off + 2 * KC + b * DH, pv);
                    tmem_wait_ld();
                } else {
                    #pragma unroll
                    for (int d = 0; d < DH; d++) pv[d] = 0.f;
                }
                tc_fence_before();
                bar_arrive(pvempty0 + 8 * b);
                #pragma unroll
                for (int d = 0; d < DH; d++) o[d] = fmaf(o[d], alpha, pv[d]);
            }
            gc += t.nkc;
            if (!ok || grow >= P.L) continue;
            if (grow < t.ext) {
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
                *lrow = (m + __log2f(l)) * 0.6931471805599453f;
            } else {
                #pragma unroll
                for (int j = 0; j < 4; j++) ((uint4*)orow)[j] = make_uint4(0, 0, 0, 0);
                *lrow = 0.f;
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

}  // namespace

int attn_tc_error_read_reset() {
    int v = 0, zero = 0;
    cudaMemcpyFromSymbol(&v, g_attn_tc_error, sizeof(int));
    cudaMemcpyToSymbol(g_attn_tc_error, &zero, sizeof(int));
    return v;
}

bool attn_fwd_tc(const void* qkv, long ldqkv, const uint8_t* keep, void* out, long ldo,
                 float* lse, int nseq, int L, int H, cudaStream_t s, const int* extent) {
    if (H * DH > 4096 || L > MAXC * KC || L < 1 || nseq <= 0) return false;
    if (((uintptr_t)qkv & 15) || ((ldqkv * 2) % 16) || ((uintptr_t)out & 15) || (ldo % 8))
        return false;
    const int D = H * DH;
    CUtensorMap map;
    if (!tc_make_map_2d(&map, qkv, DT_BF16, 3L * D, (long)nseq * L, ldqkv, DH, 128, 64))
        return false;
    FwdParams P;
    P.nseq = nseq; P.L = L; P.H = H; P.D = D;
    P.nqt = (L + QT - 1) / QT;
    P.maxc = (L + KC - 1) / KC;
    P.ldo = ldo;
    P.out = (bf16*)out; P.lse = lse; P.keep = keep; P.ext = extent;
    P.stage_bytes = TILE_BYTES * (1 + 2 * P.maxc);
    // at least 120 KB, so that one CTA fits per SM: each CTA holds 512 TMEM
    // columns for its lifetime, and a second one would wait on the allocation
    const size_t need = 1024 + 2 * (size_t)P.stage_bytes + P_BYTES + MAXC * KC * 4 + 14 * 8 + 16;
    const size_t smem = std::max<size_t>(need, 120 * 1024);
    cudaFuncSetAttribute(k_attn_fwd_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    const long items = (long)nseq * H * P.nqt;
    const int grid = (int)std::min<long>(items, tc_num_sms());
    ++g_ptcg_launches, k_attn_fwd_tc<<<grid, FWD_THREADS, smem, s>>>(map, P);
    return true;
}
