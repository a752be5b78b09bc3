// tcgen05 / TMEM / TMA GEMM for sm_100a: bf16 operands, fp32 accumulation
// in tensor memory, the fused epilogue of GemmArgs.
//
//   C[M, N] = epilogue( sum_k A(m, k) * B(n, k) )
//
// * CTA tile 128 x BN (BN <= 256, multiple of 16; multiple of 64 when B is
//   MN-major), K block 64 elements (one 128-byte swizzled row).  The
//   fp32-accumulate GEMMs (weight gradients) run 256 x BN tiles: two M = 128
//   MMAs per K step on one B stage, accumulators at TMEM columns 0 and 256.
// * Operands arrive by TMA (cp.async.bulk.tensor, 128B swizzle, no
//   multicast) into a multi-stage shared-memory ring.  K-major operands load
//   one box {64 K, rows}; MN-major operands (the transposed side of dX / dW
//   GEMMs) load boxes {64 MN, 64 K}, so no operand is ever transposed in HBM.
// * One elected thread issues tcgen05.mma.cta_group::1 (kind::f16 for bf16
//   operands, K=16 per instruction; kind::tf32 for fp32 operands, K=8) with
//   M=128, N=BN into a double-buffered TMEM accumulator and releases ring
//   slots with tcgen05.commit.  A 128-byte swizzled row holds 64 bf16 or 32
//   fp32 K-elements, so both kinds share one byte-level smem layout.
// * PTCG_EPI_WARPS epilogue warps for the GELU forward epilogues,
//   PTCG_EPI_WARPS_LIGHT for the rest (16 / 12: four / three per TMEM lane
//   quadrant, each taking every fourth / third 32-column chunk) read the
//   accumulator with
//   tcgen05.ld.32x32b.x32 while the next tile's MMAs run, and apply bias
//   (staged once per CTA in shared memory) / broadcast / GELU and GELU'
//   (packed f32x2 math) / GELU' multiply / row remap / residual /
//   accumulate / fp32 column sums.  Whole 32x32 chunks leave through a
//   swizzled shared staging buffer and a TMA store (the GELU'-multiply
//   epilogue stores from the TMA-filled GELU' slot itself, overwritten in
//   place); the rest through vectorised global stores.  The epilogue, not the MMA, bounds the K = 256
//   GEMMs of this model, so its warp count hides the latency of TMEM loads,
//   operand loads and store fences.
// * Persistent CTAs (one per SM) walk an M-major tile order so that the
//   N-tiles of one A row-block run together and share it through L2; weight
//   gradients (long K) are split over K with fp32 atomic accumulation.
// * Every wait is bounded by a clock budget; on expiry the CTA records an
//   error code in g_tc_error, drains its own in-flight copies and MMAs,
//   frees its TMEM and returns.
#include "common.cuh"
#include "internal.h"

#include <cuda.h>
#include <mutex>
#include <stdlib.h>
#include <string.h>

namespace {

constexpr int BM = 128;
// epilogue warps per CTA (a multiple of 4: NEPI / 4 per TMEM lane quadrant,
// splitting its 32-column chunks).  The GELU forward epilogues are
// instruction-bound and run PTCG_EPI_WARPS warps; the others run
// PTCG_EPI_WARPS_LIGHT, whose larger register budget (the 64K registers
// split over fewer threads) keeps their epilogue free of spills.
constexpr int NUM_EPI = PTCG_EPI_WARPS;
constexpr int NUM_EPI_LIGHT = PTCG_EPI_WARPS_LIGHT;
constexpr int NUM_EPI_AUX = PTCG_EPI_WARPS_AUX;
constexpr int STAGE_BUFS = PTCG_STAGE_BUFS;  // TMA-store staging buffers per epilogue warp
constexpr int STAGE_W = 4096 * STAGE_BUFS;   // staging bytes per epilogue warp
constexpr int BIAS_SMEM_MAX = 4096;          // bias vectors up to this many columns live in smem
static_assert(NUM_EPI % 4 == 0 && NUM_EPI_LIGHT % 4 == 0 && NUM_EPI_AUX % 4 == 0 && STAGE_BUFS >= 1 && STAGE_BUFS <= 2,
              "epilogue layout");
// warp 0 TMA, warp 1 MMA, warps 2.. epilogue
constexpr int threads_for(int nepi) { return 64 + 32 * nepi; }
constexpr long long WAIT_BUDGET = 4000000000LL;   // clock cycles (~2 s)

__device__ int g_tc_error_dev;
// optional per-role cycle counters (ptcg_tc_profile): 0 producer waiting on
// free slots, 1 MMA waiting on loaded slots, 2 MMA waiting on a free TMEM
// buffer, 3 epilogue waiting on a finished accumulator, 4 epilogue working,
// 5 CTA lifetime, 6 tiles, 7 launches
__device__ unsigned long long g_tc_prof[12];   // 8..11 unused
__device__ int g_tc_prof_on;

struct TcParams {
    int M, N, K;
    int bn;                  // CTA tile N
    int b_rows;              // B rows resident per stage (bn, or bn rounded to 64)
    int a_mn, b_mn;          // operand majorness (1 = MN-major)
    int m_tiles, n_tiles, splits, kb_total, kb_per_split;
    int stages;
    uint32_t idesc;
    uint32_t stage_bytes, a_bytes;
    uint32_t tmem_cols, acc_stride;
    int tma_out;             // outputs leave through smem + TMA stores
    uint32_t staging_bytes;  // per-warp TMA-store staging (0 when the epilogue stores in place)
    int bias_smem;           // columns of the bias staged in shared memory (0: read from global)
    int aux_tma;             // the GELU' operand arrives by TMA into two smem slots
    uint32_t aux_bytes;      // bytes of one slot: BM rows x bn bf16, as bn/32 boxes of 8 KB
    int nepi;                // epilogue warps of the instantiation that runs the plan
    int ek;                  // epilogue kind (EPI_*) of that instantiation
    int box_rows;            // rows of one TMA store box: 32, or 8 for a remap in 8-row groups
    int m2;                  // CTA tile of two 128-row halves sharing each B stage (accumulators
                             // at TMEM columns 0 and 256, one TMEM buffer); 0: one 128-row tile
    GemmArgs ep;
};

// ------------------------------------------------------------ PTX wrappers
PTCG_DEV uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
PTCG_DEV void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(bar), "r"(count));
}
PTCG_DEV void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(bar), "r"(bytes) : "memory");
}
PTCG_DEV void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(bar) : "memory");
}
PTCG_DEV bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred P;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, P;\n\t}"
                 : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    return ok != 0;
}
// bounded wait: false (and the abort flag set) when the budget runs out
PTCG_DEV bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int code,
                        long long* waited = nullptr) {
    long long t0 = clock64();
    bool ok = true;
    while (!mbar_try(bar, parity)) {
        if (*abort_flag) { ok = false; break; }
        if (clock64() - t0 > WAIT_BUDGET) {
            *abort_flag = 1;
            atomicCAS(&g_tc_error_dev, 0, code);
            ok = false;
            break;
        }
    }
    if (waited) *waited += clock64() - t0;
    return ok;
}
PTCG_DEV void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%3, %4}], [%2];"
                 :: "r"(dst), "l"((uint64_t)map), "r"(bar), "r"(x), "r"(y) : "memory");
}
PTCG_DEV void tma_store_2d(const CUtensorMap* map, uint32_t src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];"
                 :: "l"((uint64_t)map), "r"(src), "r"(x), "r"(y) : "memory");
}
PTCG_DEV void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
PTCG_DEV void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
PTCG_DEV void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
PTCG_DEV void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
PTCG_DEV void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Stage one warp's 32x32 chunk (lane = row) for a TMA store: fp32 rows of
// 128 B in the 128-byte swizzle (16-byte granule g of row r at g ^ (r & 7)),
// bf16 rows of 64 B in the 64-byte swizzle (granule g at g ^ ((r >> 1) & 3)).
PTCG_DEV void stage32(uint8_t* buf, int lane, int dt, const float (&v)[32]) {
    if (dt == DT_F32) {
        #pragma unroll
        for (int g = 0; g < 8; g++)
            *(float4*)(buf + lane * 128 + ((g ^ (lane & 7)) << 4)) =
                make_float4(v[4 * g], v[4 * g + 1], v[4 * g + 2], v[4 * g + 3]);
    } else {
        #pragma unroll
        for (int g = 0; g < 4; g++) {
            uint4 q;
            __nv_bfloat162* h = (__nv_bfloat162*)&q;
            #pragma unroll
            for (int k = 0; k < 4; k++) h[k] = __floats2bfloat162_rn(v[8 * g + 2 * k], v[8 * g + 2 * k + 1]);
            *(uint4*)(buf + lane * 64 + ((g ^ ((lane >> 1) & 3)) << 4)) = q;
        }
    }
}

PTCG_DEV void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
PTCG_DEV void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
template <int EB>
PTCG_DEV void mma_issue(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
    if (EB == 2)
        asm volatile("{\n\t.reg .pred p;\n\t"
                     "setp.ne.b32 p, %4, 0;\n\t"
                     "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
                     :: "r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc) : "memory");
    else
        asm volatile("{\n\t.reg .pred p;\n\t"
                     "setp.ne.b32 p, %4, 0;\n\t"
                     "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
                     :: "r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc) : "memory");
}
PTCG_DEV void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(bar) : "memory");
}
PTCG_DEV void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
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
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// UMMA shared-memory descriptor, sm_100 version bits.  layout 2 = 128-byte
// swizzle (16-byte granules, 8-row atoms); layout 1 = 128-byte swizzle with
// 32-byte granules and 4-row atoms (the only MN-major layout for 32-bit
// operands; TMA writes it with CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B).
PTCG_DEV uint64_t make_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t layout = 2) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);
    d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
    d |= (uint64_t)1 << 46;                  // descriptor version (sm_100)
    d |= (uint64_t)layout << 61;
    return d;
}


// 32 consecutive values of one row: vectorised when the whole chunk is in
// range and 16-byte aligned, scalar (with zero fill) otherwise
PTCG_DEV void load32(float (&d)[32], const void* p, long base, int dt, int nvalid) {
    if (dt == DT_F32) {
        const float* q = (const float*)p + base;
        if (nvalid == 32 && ((uintptr_t)q & 15) == 0) {
            #pragma unroll
            for (int j = 0; j < 32; j += 4) {
                float4 t = *(const float4*)(q + j);
                d[j] = t.x; d[j + 1] = t.y; d[j + 2] = t.z; d[j + 3] = t.w;
            }
        } else {
            #pragma unroll
            for (int j = 0; j < 32; j++) d[j] = j < nvalid ? q[j] : 0.f;
        }
    } else {
        const bf16* q = (const bf16*)p + base;
        if (nvalid == 32 && ((uintptr_t)q & 15) == 0) {
            #pragma unroll
            for (int j = 0; j < 32; j += 8) {
                uint4 t = *(const uint4*)(q + j);
                const __nv_bfloat162* h = (const __nv_bfloat162*)&t;
                #pragma unroll
                for (int k = 0; k < 4; k++) {
                    float2 f = __bfloat1622float2(h[k]);
                    d[j + 2 * k] = f.x; d[j + 2 * k + 1] = f.y;
                }
            }
        } else {
            #pragma unroll
            for (int j = 0; j < 32; j++) d[j] = j < nvalid ? __bfloat162float(q[j]) : 0.f;
        }
    }
}
PTCG_DEV void store32(void* p, long base, int dt, const float (&v)[32], int nvalid) {
    if (dt == DT_F32) {
        float* q = (float*)p + base;
        if (nvalid == 32 && ((uintptr_t)q & 15) == 0) {
            #pragma unroll
            for (int j = 0; j < 32; j += 4) *(float4*)(q + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        } else {
            #pragma unroll
            for (int j = 0; j < 32; j++) if (j < nvalid) q[j] = v[j];
        }
    } else {
        bf16* q = (bf16*)p + base;
        if (nvalid == 32 && ((uintptr_t)q & 15) == 0) {
            #pragma unroll
            for (int j = 0; j < 32; j += 8) {
                uint4 t;
                __nv_bfloat162* h = (__nv_bfloat162*)&t;
                #pragma unroll
                for (int k = 0; k < 4; k++) h[k] = __floats2bfloat162_rn(v[j + 2 * k], v[j + 2 * k + 1]);
                *(uint4*)(q + j) = t;
            }
        } else {
            #pragma unroll
            for (int j = 0; j < 32; j++) if (j < nvalid) q[j] = __float2bfloat16_rn(v[j]);
        }
    }
}

// lane l ends with sum over the warp's lanes of v[l]  (transpose-reduce)
PTCG_DEV float warp_colsum32(float (&v)[32], int lane) {
    #pragma unroll
    for (int s = 16; s >= 1; s >>= 1) {
        bool up = lane & s;
        #pragma unroll
        for (int i = 0; i < s; i++) {
            float send = up ? v[i] : v[i + s];
            float keep = up ? v[i + s] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, s);
        }
    }
    return v[0];
}

// one operand tile of a ring stage: `rows` MN rows x one 128-byte K row.
// K-major: one box {BK, rows}; MN-major: rows / ATOM boxes {ATOM, BK}
template <int EB>
PTCG_DEV void load_operand(uint32_t dst, const CUtensorMap* map, uint32_t bar, int mn_major,
                           int rows, int mn0, int k0) {
    constexpr int ATOM = 128 / EB;
    constexpr uint32_t BOX = (128 / EB) * 128;
    if (mn_major) {
        for (int j = 0; j < rows / ATOM; j++) tma_load_2d(dst + j * BOX, map, bar, mn0 + ATOM * j, k0);
    } else {
        tma_load_2d(dst, map, bar, k0, mn0);
    }
}

// -------------------------------------------------------------- the kernel
// EB = operand element bytes (2: bf16 / kind::f16, 4: fp32 / kind::tf32)
// epilogue kinds with a specialised chunk loop (compile-time), the rest
// through the generic one
enum { EPI_GENERIC = 0, EPI_GELU_SAVE = 1, EPI_GELU_AUX = 2,
       EPI_PLAIN = 3, EPI_BIAS = 4, EPI_RESID = 5, EPI_BIAS_RESID = 6,  // 3 + bias + 2 resid
       EPI_GELU = 7 };                                                   // bias + GELU, no GELU'

template <int EB, int NEPI, int EK>
__global__ void __launch_bounds__(threads_for(NEPI), 1)
k_gemm_tc(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
          const __grid_constant__ CUtensorMap map_c, const __grid_constant__ CUtensorMap map_c2,
          const __grid_constant__ CUtensorMap map_aux, const __grid_constant__ TcParams P) {
    constexpr int BK = 128 / EB;            // K elements per 128-byte row
    constexpr int KI = 32 / EB;             // K elements per MMA instruction
    constexpr uint32_t BOX = BK * 128;      // bytes of one MN-major box {ATOM, BK}
    // MN-major K-direction atom: 8 rows (bf16, 128B swizzle) or 4 rows
    // (fp32, 128B swizzle with 32-byte base)
    constexpr uint32_t MN_SBO = EB == 2 ? 1024 : 512;
    constexpr uint32_t MN_LAYOUT = EB == 2 ? 2 : 1;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    const int S = P.stages;
    // 256-row tiles exist only in the generic light-epilogue instantiation
    // (the plain fp32-accumulate GEMMs); elsewhere m2 folds to 0
    const int m2 = (EK == EPI_GENERIC && NEPI == NUM_EPI_LIGHT) ? P.m2 : 0;
    constexpr int EPI_GROUPS = NEPI / 4;    // warps sharing a quadrant split its 32-column chunks
    uint8_t* staging = smem + (size_t)S * P.stage_bytes;          // NEPI x STAGE_W, or none
    uint8_t* auxbuf = staging + P.staging_bytes;                  // 2 x aux_bytes
    uint64_t* bars = (uint64_t*)(auxbuf + (P.aux_tma ? 2 * P.aux_bytes : 0));
    // bars: full[S], empty[S], tfull[2], tempty[2], drain[1], afull[2], aempty[2]
    uint32_t* tmem_slot = (uint32_t*)(bars + 2 * S + 9);
    volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
    int* n_issued = (int*)(tmem_slot + 2);     // ring slots filled by TMA
    int* n_consumed = (int*)(tmem_slot + 3);   // ring slots read by the MMA warp
    int* n_aux_issued = (int*)(tmem_slot + 4); // aux tiles requested by the producer
    int* n_aux_done = (int*)(tmem_slot + 5);   // aux tiles the epilogue has waited for
    float* sbias = (float*)(((uintptr_t)(tmem_slot + 8) + 15) & ~(uintptr_t)15);   // [P.bias_smem]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + S);
    const uint32_t tfull0 = smem_u32(bars + 2 * S), tempty0 = smem_u32(bars + 2 * S + 2);
    const uint32_t drain = smem_u32(bars + 2 * S + 4);
    const uint32_t afull0 = smem_u32(bars + 2 * S + 5), aempty0 = smem_u32(bars + 2 * S + 7);

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; i++) { mbar_init(full0 + 8 * i, 1); mbar_init(empty0 + 8 * i, 1); }
        for (int i = 0; i < 2; i++) { mbar_init(tfull0 + 8 * i, 1); mbar_init(tempty0 + 8 * i, NEPI); }
        mbar_init(drain, 1);
        for (int i = 0; i < 2; i++) { mbar_init(afull0 + 8 * i, 1); mbar_init(aempty0 + 8 * i, NEPI); }
        *abort_flag = 0;
        *n_issued = 0;
        *n_consumed = 0;
        *n_aux_issued = 0;
        *n_aux_done = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    for (int i = threadIdx.x; i < P.bias_smem; i += blockDim.x) sbias[i] = P.ep.bias[i];
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(smem_u32(tmem_slot)), "r"(P.tmem_cols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = *tmem_slot;
    const int ntiles = P.m_tiles * P.n_tiles * P.splits;
    const long long t_cta0 = clock64();

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            long long w_empty = 0;
            int plocal = 0;
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, plocal++) {
                int split = t % P.splits;
                int mn = t / P.splits;
                int mt = mn / P.n_tiles, nt = mn % P.n_tiles;
                int kb0 = split * P.kb_per_split;
                int kb1 = min(P.kb_total, kb0 + P.kb_per_split);
                if (P.aux_tma) {
                    // this tile's GELU' block into slot plocal & 1 once the
                    // epilogue has finished the tile two back
                    int slot = plocal & 1;
                    if (!mbar_wait(aempty0 + 8 * slot, ((plocal >> 1) & 1) ^ 1, abort_flag, 5, &w_empty)) {
                        ok = false;
                        break;
                    }
                    uint32_t fb = afull0 + 8 * slot;
                    mbar_expect_tx(fb, P.aux_bytes);
                    uint32_t dst = smem_u32(auxbuf + (size_t)slot * P.aux_bytes);
                    for (int c = 0; c < P.bn / 32; c++)
                        tma_load_2d(dst + c * 8192, &map_aux, fb, nt * P.bn + 32 * c, mt * BM);
                    (*n_aux_issued)++;
                }
                for (int kb = kb0; kb < kb1; kb++) {
                    if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, abort_flag, 1, &w_empty)) { ok = false; break; }
                    uint32_t fb = full0 + 8 * stage;
                    mbar_expect_tx(fb, P.stage_bytes);
                    uint32_t sa = smem_u32(smem + (size_t)stage * P.stage_bytes);
                    int k0 = kb * BK;
                    for (int h = 0; h <= m2; h++)
                        load_operand<EB>(sa + h * BM * 128, &map_a, fb, P.a_mn, BM,
                                         (mt << m2) * BM + h * BM, k0);
                    load_operand<EB>(sa + P.a_bytes, &map_b, fb, P.b_mn, P.b_rows, nt * P.bn, k0);
                    if (++stage == S) { stage = 0; phase ^= 1; }
                    (*n_issued)++;
                }
            }
            if (g_tc_prof_on) atomicAdd(&g_tc_prof[0], (unsigned long long)w_empty);
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int local = 0;
            bool ok = true;
            long long w_full = 0, w_tempty = 0;
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, local++) {
                int split = t % P.splits;
                int kb0 = split * P.kb_per_split;
                int kb1 = min(P.kb_total, kb0 + P.kb_per_split);
                // two TMEM buffers alternate over tiles, or one (both halves) with m2
                int buf = m2 ? 0 : local & 1;
                uint32_t tph = m2 ? local & 1 : (local >> 1) & 1;
                if (!mbar_wait(tempty0 + 8 * buf, tph ^ 1, abort_flag, 2, &w_tempty)) { ok = false; break; }
                fence_after();
                uint32_t dcol = tmem + buf * P.acc_stride;
                for (int kb = kb0; kb < kb1; kb++) {
                    if (!mbar_wait(full0 + 8 * stage, phase, abort_flag, 3, &w_full)) { ok = false; break; }
                    fence_after();
                    uint32_t sa = smem_u32(smem + (size_t)stage * P.stage_bytes);
                    uint32_t sb = sa + P.a_bytes;
                    #pragma unroll
                    for (int s = 0; s < BK / KI; s++) {
                        uint64_t ad = P.a_mn ? make_desc(sa + s * KI * 128, BOX, MN_SBO, MN_LAYOUT)
                                             : make_desc(sa + s * 32, 16, 1024);
                        uint64_t bd = P.b_mn ? make_desc(sb + s * KI * 128, BOX, MN_SBO, MN_LAYOUT)
                                             : make_desc(sb + s * 32, 16, 1024);
                        mma_issue<EB>(dcol, ad, bd, P.idesc, (kb > kb0 || s > 0) ? 1u : 0u);
                        if (m2) {                   // rows 128..255: A half 16 KB on, same B
                            const uint32_t sa2 = sa + BM * 128;
                            uint64_t ad2 = P.a_mn ? make_desc(sa2 + s * KI * 128, BOX, MN_SBO, MN_LAYOUT)
                                                  : make_desc(sa2 + s * 32, 16, 1024);
                            mma_issue<EB>(dcol + 256, ad2, bd, P.idesc, (kb > kb0 || s > 0) ? 1u : 0u);
                        }
                    }
                    mma_commit(empty0 + 8 * stage);
                    if (++stage == S) { stage = 0; phase ^= 1; }
                    (*n_consumed)++;
                }
                if (!ok) break;
                mma_commit(tfull0 + 8 * buf);
            }
            if (g_tc_prof_on) {
                atomicAdd(&g_tc_prof[1], (unsigned long long)w_full);
                atomicAdd(&g_tc_prof[2], (unsigned long long)w_tempty);
                atomicAdd(&g_tc_prof[6], (unsigned long long)local);
            }
            // make sure no MMA is in flight before TMEM is released
            mma_commit(drain);
            long long t0 = clock64();
            while (!mbar_try(drain, 0) && clock64() - t0 < WAIT_BUDGET) {}
        }
        __syncwarp();
    } else {
        // ------------------------------------------------ epilogue warps
        const int quad = warp & 3;           // TMEM lane quadrant this warp may read
        const int grp = (warp - 2) >> 2;     // which of the quadrant's interleaved 32-column chunks
        const int row_in_tile = quad * 32 + lane;
        const GemmArgs& a = P.ep;
        int local = 0;
        int nchunk = 0;
        long long w_tfull = 0, busy = 0;
        for (int t = blockIdx.x; t < ntiles; t += gridDim.x, local++) {
            int split = t % P.splits;
            int mn = t / P.splits;
            int mt = mn / P.n_tiles, nt = mn % P.n_tiles;
            int buf = m2 ? 0 : local & 1;
            uint32_t tph = m2 ? local & 1 : (local >> 1) & 1;
            if (!mbar_wait(tfull0 + 8 * buf, tph, abort_flag, 4, &w_tfull)) break;
            if (P.aux_tma) {
                if (!mbar_wait(afull0 + 8 * buf, tph, abort_flag, 6, &w_tfull)) break;
                if (warp == 2 && lane == 0) *n_aux_done = local + 1;
            }
            long long tb = clock64();
            fence_after();
            for (int h = 0; h <= m2; h++) {
            const int row0 = (mt << m2) * BM + h * BM;   // first row of this 128-row half
            const int m = row0 + row_in_tile;
            const bool row_ok = m < a.M;
            long orow = m;
            if (a.remap_group > 0)
                orow = (long)(m / a.remap_group) * a.remap_stride + a.remap_off + (m % a.remap_group);
            const uint32_t tbase = tmem + (m2 ? h * 256 : buf * P.acc_stride) + ((uint32_t)(quad * 32) << 16);
            for (int c0 = grp * 32; c0 < P.bn; c0 += 32 * EPI_GROUPS) {
                uint32_t r[32];
                tmem_ld32(tbase + c0, r);
                const int n0 = nt * P.bn + c0;
                float v[32];
                #pragma unroll
                for (int j = 0; j < 32; j++) v[j] = __uint_as_float(r[j]);
                if (a.alpha != 1.f) {
                    #pragma unroll
                    for (int j = 0; j < 32; j++) v[j] *= a.alpha;
                }
                int nvalid = a.N - n0;
                if (nvalid > P.bn - c0) nvalid = P.bn - c0;
                if (nvalid > 32) nvalid = 32;
                if (nvalid <= 0) continue;                       // warp-uniform
                if constexpr (EK == EPI_GELU_SAVE || EK == EPI_GELU) {
                    // bias (staged in smem) + GELU, GELU' saved (EPI_GELU_SAVE);
                    // bf16 out (and out2) through the staging buffer and TMA
                    // stores (rows past M are computed on zero-filled operands
                    // and clipped)
                    uint8_t* sbuf = staging + (warp - 2) * STAGE_W + (nchunk % STAGE_BUFS) * 4096;
                    nchunk++;
                    if (lane == 0) {
                        if (STAGE_BUFS == 2) bulk_wait_read1();
                        else bulk_wait_read0();
                    }
                    __syncwarp();
                    if (nvalid == 32) {
                        #pragma unroll
                        for (int j = 0; j < 32; j += 4) {
                            float4 b4 = *(const float4*)(sbias + n0 + j);
                            add_pair(v[j], v[j + 1], b4.x, b4.y);
                            add_pair(v[j + 2], v[j + 3], b4.z, b4.w);
                        }
                    } else {
                        #pragma unroll
                        for (int j = 0; j < 32; j++) if (j < nvalid) v[j] += sbias[n0 + j];
                    }
                    if constexpr (EK == EPI_GELU_SAVE) {
                        float g[32];
                        #pragma unroll
                        for (int j = 0; j < 32; j += 2)
                            gelu2(v[j], v[j + 1], v[j], v[j + 1], g[j], g[j + 1]);
                        stage32(sbuf + 2048, lane, DT_BF16, g);
                    } else {
                        #pragma unroll
                        for (int j = 0; j < 32; j += 2) {
                            float g0, g1;
                            gelu2(v[j], v[j + 1], v[j], v[j + 1], g0, g1);
                        }
                    }
                    stage32(sbuf, lane, a.out_dtype, v);
                    fence_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        const int y = row0 + quad * 32;
                        tma_store_2d(&map_c, smem_u32(sbuf), n0, y);
                        if constexpr (EK == EPI_GELU_SAVE)
                            tma_store_2d(&map_c2, smem_u32(sbuf + 2048), n0, y);
                        bulk_commit();
                    }
                    continue;
                } else if constexpr (EK == EPI_GELU_AUX) {
                    // v *= GELU' (prefetched by TMA into the tile's aux slot);
                    // the bf16 product overwrites this row of the slot in
                    // place (same 64-byte swizzle, so no staging buffer) and
                    // leaves by a TMA store of the warp's 32-row box; the slot
                    // is handed back to the producer once the stores have
                    // read it.  Optional fp32 column sums of the product.
                    uint8_t* box = auxbuf + (size_t)buf * P.aux_bytes + (c0 >> 5) * 8192;
                    uint8_t* ab = box + row_in_tile * 64;
                    const int sw = (row_in_tile >> 1) & 3;
                    #pragma unroll
                    for (int gq = 0; gq < 4; gq++) {
                        uint4* p = (uint4*)(ab + ((gq ^ sw) << 4));
                        uint4 q = *p;
                        __nv_bfloat162* h2 = (__nv_bfloat162*)&q;
                        #pragma unroll
                        for (int k = 0; k < 4; k++) {
                            float2 f = __bfloat1622float2(h2[k]);
                            v[8 * gq + 2 * k] *= f.x;
                            v[8 * gq + 2 * k + 1] *= f.y;
                            h2[k] = __floats2bfloat162_rn(v[8 * gq + 2 * k], v[8 * gq + 2 * k + 1]);
                        }
                        *p = q;
                    }
                    fence_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&map_c, smem_u32(box + quad * 2048), n0, row0 + quad * 32);
                        bulk_commit();
                    }
                    if (a.colsum) {
                        #pragma unroll
                        for (int j = 0; j < 32; j++) if (j >= nvalid || !row_ok) v[j] = 0.f;
                        float cs = warp_colsum32(v, lane);
                        if (lane < nvalid) atomicAdd(&a.colsum[n0 + lane], cs);
                    }
                    continue;
                } else if constexpr (EK >= EPI_PLAIN) {
                    // [bias (smem)] [+ fp32 residual] -> out through staging +
                    // TMA store, optional fp32 column sums
                    constexpr bool HB = (EK - EPI_PLAIN) & 1, HR = (EK - EPI_PLAIN) & 2;
                    uint8_t* sbuf = staging + (warp - 2) * STAGE_W + (nchunk % STAGE_BUFS) * 4096;
                    nchunk++;
                    if (lane == 0) {
                        if (STAGE_BUFS == 2) bulk_wait_read1();
                        else bulk_wait_read0();
                    }
                    __syncwarp();
                    if constexpr (HB) {
                        if (nvalid == 32) {
                            #pragma unroll
                            for (int j = 0; j < 32; j += 4) {
                                float4 b4 = *(const float4*)(sbias + n0 + j);
                                v[j] += b4.x; v[j + 1] += b4.y; v[j + 2] += b4.z; v[j + 3] += b4.w;
                            }
                        } else {
                            #pragma unroll
                            for (int j = 0; j < 32; j++) if (j < nvalid) v[j] += sbias[n0 + j];
                        }
                    }
                    if constexpr (HR) {
                        if (row_ok) {
                            float t[32];
                            load32(t, a.resid, (long)m * a.ld_resid + n0, DT_F32, nvalid);
                            #pragma unroll
                            for (int j = 0; j < 32; j++) v[j] += t[j];
                        }
                    }
                    stage32(sbuf, lane, a.out_dtype, v);
                    fence_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&map_c, smem_u32(sbuf), n0, row0 + quad * 32);
                        bulk_commit();
                    }
                    if (a.colsum) {
                        #pragma unroll
                        for (int j = 0; j < 32; j++) if (j >= nvalid || !row_ok) v[j] = 0.f;
                        float cs = warp_colsum32(v, lane);
                        if (lane < nvalid) atomicAdd(&a.colsum[n0 + lane], cs);
                    }
                    continue;
                }
                if (P.splits > 1) {                              // warp-uniform
                    if (row_ok) {
                        float* o = (float*)a.out + orow * a.ldo + n0;
                        if (nvalid == 32 && ((uintptr_t)o & 15) == 0) {
                            #pragma unroll
                            for (int j = 0; j < 32; j += 4)
                                asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};"
                                             :: "l"(o + j), "f"(v[j]), "f"(v[j + 1]), "f"(v[j + 2]),
                                                "f"(v[j + 3]) : "memory");
                        } else {
                            #pragma unroll
                            for (int j = 0; j < 32; j++) if (j < nvalid) atomicAdd(o + j, v[j]);
                        }
                    }
                    continue;
                }
                // staging: with two buffers the one written now was last used
                // two chunks ago (at most one store group may still read it);
                // with one, the previous store must have finished reading
                uint8_t* sbuf = staging + (warp - 2) * STAGE_W + (nchunk % STAGE_BUFS) * 4096;
                nchunk++;
                if (P.tma_out) {
                    if (lane == 0) {
                        if (STAGE_BUFS == 2) bulk_wait_read1();
                        else bulk_wait_read0();
                    }
                    __syncwarp();
                }
                // fp32 GELU with its fp32 GELU' (TF32 GEMMs): both chunks go
                // through the one staging buffer, GELU' first (stored below)
                const bool f32pair = P.tma_out && a.act == ACT_GELU && a.out2 && a.out_dtype == DT_F32;
                if (row_ok) {
                float t[32];
                if (a.bias) {
                    if (P.bias_smem) {
                        if (nvalid == 32) {
                            #pragma unroll
                            for (int j = 0; j < 32; j += 4) {
                                float4 b4 = *(const float4*)(sbias + n0 + j);
                                v[j] += b4.x; v[j + 1] += b4.y; v[j + 2] += b4.z; v[j + 3] += b4.w;
                            }
                        } else {
                            #pragma unroll
                            for (int j = 0; j < 32; j++) if (j < nvalid) v[j] += sbias[n0 + j];
                        }
                    } else {
                        load32(t, a.bias, n0, DT_F32, nvalid);
                        #pragma unroll
                        for (int j = 0; j < 32; j++) v[j] += t[j];
                    }
                }
                if (a.bcast) {
                    load32(t, a.bcast, (long)(m / a.bcast_group) * a.ld_bcast + n0, DT_F32, nvalid);
                    #pragma unroll
                    for (int j = 0; j < 32; j++) v[j] += t[j];
                }
                if (a.act == ACT_GELU) {
                    if (a.out2) {
                        #pragma unroll
                        for (int j = 0; j < 32; j += 2)        // GELU'(x) saved for backward
                            gelu2(v[j], v[j + 1], v[j], v[j + 1], t[j], t[j + 1]);
                        if (P.tma_out) {
                            if (f32pair) stage32(sbuf, lane, DT_F32, t);
                            else stage32(sbuf + 2048, lane, DT_BF16, t);
                        }
                        else store32(a.out2, (long)m * a.ldo2 + n0, a.out2_dtype, t, nvalid);
                    } else {
                        #pragma unroll
                        for (int j = 0; j < 32; j += 2) {
                            float g0, g1;
                            gelu2(v[j], v[j + 1], v[j], v[j + 1], g0, g1);
                        }
                    }
                } else if (a.act == ACT_GELU_BWD) {
                    if (P.aux_tma) {
                        // row row_in_tile of box c0 / 32 (64-byte rows, 64-byte swizzle)
                        const uint8_t* ab = auxbuf + (size_t)buf * P.aux_bytes + (c0 >> 5) * 8192 +
                                            row_in_tile * 64;
                        #pragma unroll
                        for (int g = 0; g < 4; g++) {
                            uint4 q = *(const uint4*)(ab + ((g ^ ((row_in_tile >> 1) & 3)) << 4));
                            const __nv_bfloat162* h2 = (const __nv_bfloat162*)&q;
                            #pragma unroll
                            for (int k = 0; k < 4; k++) {
                                float2 f = __bfloat1622float2(h2[k]);
                                t[8 * g + 2 * k] = f.x; t[8 * g + 2 * k + 1] = f.y;
                            }
                        }
                    } else {
                        load32(t, a.aux, (long)m * a.ld_aux + n0, a.aux_dtype, nvalid);
                    }
                    #pragma unroll
                    for (int j = 0; j < 32; j++) v[j] *= t[j];
                }
                if (a.resid) {
                    load32(t, a.resid, orow * a.ld_resid + n0, DT_F32, nvalid);
                    #pragma unroll
                    for (int j = 0; j < 32; j++) v[j] += t[j];
                }
                if (a.accumulate) {
                    load32(t, a.out, orow * a.ldo + n0, a.out_dtype, nvalid);
                    #pragma unroll
                    for (int j = 0; j < 32; j++) v[j] += t[j];
                }
                if (P.tma_out) {
                    if (!f32pair) stage32(sbuf, lane, a.out_dtype, v);
                } else {
                    store32(a.out, orow * a.ldo + n0, a.out_dtype, v, nvalid);
                }
                if (!P.tma_out && a.act != ACT_GELU && a.out2)
                    store32(a.out2, orow * a.ldo2 + n0, a.out2_dtype, v, nvalid);
                }   // row_ok
                if (P.tma_out) {
                    if (f32pair) {
                        // GELU' (staged above) out first, then GELU (v) into the same buffer
                        fence_async_smem();
                        __syncwarp();
                        if (lane == 0) {
                            tma_store_2d(&map_c2, smem_u32(sbuf), n0, row0 + quad * 32);
                            bulk_commit();
                            bulk_wait_read0();
                        }
                        __syncwarp();
                        if (row_ok) stage32(sbuf, lane, DT_F32, v);
                    }
                    // rows past M and columns past N are clipped by the TMA unit
                    fence_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        int y = row0 + quad * 32;
                        if (P.box_rows == 8) {                   // four 8-row boxes, each remapped
                            const uint32_t rb = a.out_dtype == DT_F32 ? 128u : 64u;
                            for (int i = 0; i < 4; i++) {
                                const int yi = y + 8 * i;
                                const int yo = (yi / a.remap_group) * a.remap_stride + a.remap_off +
                                               yi % a.remap_group;
                                tma_store_2d(&map_c, smem_u32(sbuf) + i * 8 * rb, n0, yo);
                            }
                        } else {
                            if (a.remap_group > 0)               // the box's first output row
                                y = (y / a.remap_group) * a.remap_stride + a.remap_off + y % a.remap_group;
                            tma_store_2d(&map_c, smem_u32(sbuf), n0, y);
                            if (a.act == ACT_GELU && a.out2 && !f32pair)
                                tma_store_2d(&map_c2, smem_u32(sbuf + 2048), n0, y);
                        }
                        bulk_commit();
                    }
                }
                if (a.colsum) {
                    #pragma unroll
                    for (int j = 0; j < 32; j++) if (j >= nvalid || !row_ok) v[j] = 0.f;
                    float cs = warp_colsum32(v, lane);
                    if (lane < nvalid) atomicAdd(&a.colsum[n0 + lane], cs);
                }
            }
            }   // halves
            (void)split;
            fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(tempty0 + 8 * buf);
                if (P.aux_tma) {
                    // the in-place epilogue's stores read the slot itself
                    if constexpr (EK == EPI_GELU_AUX) bulk_wait_read0();
                    mbar_arrive(aempty0 + 8 * buf);
                }
            }
            busy += clock64() - tb;
        }
        if (P.tma_out && lane == 0) bulk_wait_all();
        if (g_tc_prof_on && lane == 0) {
            atomicAdd(&g_tc_prof[3], (unsigned long long)w_tfull);
            atomicAdd(&g_tc_prof[4], (unsigned long long)busy);
        }
    }
    fence_before();
    __syncthreads();
    fence_after();
    if (threadIdx.x == 0 && *n_consumed < *n_issued) {
        // aborted: wait (bounded) for the copies still in flight into the ring
        for (int i = *n_consumed; i < *n_issued; i++) {
            long long t0 = clock64();
            while (!mbar_try(full0 + 8 * (i % S), (uint32_t)((i / S) & 1)) &&
                   clock64() - t0 < WAIT_BUDGET) {}
        }
    }
    if (threadIdx.x == 0 && *n_aux_done < *n_aux_issued) {
        // the same for GELU' tiles requested but never waited for
        for (int i = *n_aux_done; i < *n_aux_issued; i++) {
            long long t0 = clock64();
            while (!mbar_try(afull0 + 8 * (i & 1), (uint32_t)((i >> 1) & 1)) &&
                   clock64() - t0 < WAIT_BUDGET) {}
        }
    }
    __syncthreads();
    if (threadIdx.x == 0 && g_tc_prof_on) {
        atomicAdd(&g_tc_prof[5], (unsigned long long)(clock64() - t_cta0));
        if (blockIdx.x == 0) atomicAdd(&g_tc_prof[7], 1ull);
    }
    if (warp == 1) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
                     :: "r"(tmem), "r"(P.tmem_cols) : "memory");
    }
}

// ---------------------------------------------------------- host side
typedef CUresult (*EncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                             const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                             const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                             CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeFn g_encode = nullptr;
int g_sms = 0;
bool g_ok = false;
std::once_flag g_once;

void init_once() {
    int dev = 0, major = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev);
    if (major != 10) return;
    // diagnostic engine selector: PTCG_GEMM_ENGINE=simt runs every GEMM on
    // the SIMT kernel (numerical A/B comparisons); the default uses tcgen05
    const char* eng = getenv("PTCG_GEMM_ENGINE");
    if (eng && strcmp(eng, "simt") == 0) return;
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
        return;
    g_encode = (EncodeFn)fn;
    int zero = 0;
    cudaMemcpyToSymbol(g_tc_error_dev, &zero, sizeof(int));
    g_ok = true;
}



}  // namespace

int ptcg_tc_profile_ctl(int enable, unsigned long long* out8) {
    if (out8) cudaMemcpyFromSymbol(out8, g_tc_prof, sizeof(unsigned long long) * 12);
    unsigned long long z[12] = {0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0};
    cudaMemcpyToSymbol(g_tc_prof, z, sizeof z);
    cudaMemcpyToSymbol(g_tc_prof_on, &enable, sizeof(int));
    return 0;
}

int ptcg_tc_error_read_reset() {
    int v = 0, zero = 0;
    cudaMemcpyFromSymbol(&v, g_tc_error_dev, sizeof(int));
    cudaMemcpyToSymbol(g_tc_error_dev, &zero, sizeof(int));
    return v;
}

bool gemm_tc_available() {
    std::call_once(g_once, init_once);
    return g_ok;
}

bool tc_make_map_2d(CUtensorMap* m, const void* ptr, int dtype, long inner, long outer, long ld,
                    int box_in, int box_out, int swizzle_bytes) {
    if (!gemm_tc_available()) return false;
    const int eb = dtype == DT_F32 ? 4 : 2;
    cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
    cuuint64_t strides[1] = {(cuuint64_t)ld * eb};
    cuuint32_t box[2] = {(cuuint32_t)box_in, (cuuint32_t)box_out};
    cuuint32_t es[2] = {1, 1};
    CUtensorMapSwizzle sw = swizzle_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                          : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                          : swizzle_bytes == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                                : CU_TENSOR_MAP_SWIZZLE_NONE;
    CUresult r = g_encode(m, eb == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                          2, const_cast<void*>(ptr), dims, strides, box, es,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

int tc_num_sms() {
    std::call_once(g_once, init_once);
    return g_sms;
}

namespace {

// 2-D tensor map of `eb`-byte elements
bool make_map_eb(CUtensorMap* m, const void* ptr, long inner, long outer, long ld, int box_in,
                 int box_out, int eb, bool mn_major) {
    cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
    cuuint64_t strides[1] = {(cuuint64_t)ld * eb};
    cuuint32_t box[2] = {(cuuint32_t)box_in, (cuuint32_t)box_out};
    cuuint32_t es[2] = {1, 1};
    CUresult r = g_encode(m, eb == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                          2, const_cast<void*>(ptr), dims, strides, box, es,
                          CU_TENSOR_MAP_INTERLEAVE_NONE,
                          (eb == 4 && mn_major) ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
                                                : CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

struct TcPlan {
    TcParams P;
    int eb;
    CUtensorMap ma, mb, mc, mc2, mx;
};

// GELU' operand map for the TMA prefetch: box {32 columns, 128 rows} bf16,
// 64-byte rows in the 64-byte swizzle
bool make_aux_map(CUtensorMap* m, const void* ptr, long n, long rows, long ld) {
    cuuint64_t dims[2] = {(cuuint64_t)n, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    cuuint32_t box[2] = {32, (cuuint32_t)BM};
    cuuint32_t es[2] = {1, 1};
    CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides,
                          box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// output map for TMA stores: box {32 columns, box_rows rows}
bool make_out_map(CUtensorMap* m, void* ptr, long n, long rows, long ld, int dt, int box_rows = 32) {
    int eb = dt == DT_F32 ? 4 : 2;
    cuuint64_t dims[2] = {(cuuint64_t)n, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * eb};
    cuuint32_t box[2] = {32, (cuuint32_t)box_rows};
    cuuint32_t es[2] = {1, 1};
    CUresult r = g_encode(m, dt == DT_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                          2, ptr, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          dt == DT_F32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

bool plan_tc(const GemmArgs& a, TcPlan& pl) {
    if (!gemm_tc_available()) return false;
    int eb;
    if (a.dtype == DT_BF16) eb = 2;
    else if (a.dtype == DT_F32 && a.allow_tf32) eb = 4;
    else return false;
    if (a.M <= 0 || a.N <= 0 || a.K <= 0) return false;
    // TMA: 16-byte aligned base and row pitch
    if (((uintptr_t)a.A & 15) || ((uintptr_t)a.B & 15) || ((a.lda * eb) % 16) || ((a.ldb * eb) % 16))
        return false;
    // small problems stay on the SIMT kernel
    if ((long)a.M * a.N * a.K < (1L << 22)) return false;
    const int BK = 128 / eb, ATOM = 128 / eb;
    TcParams& P = pl.P;
    P.M = a.M; P.N = a.N; P.K = a.K;
    P.a_mn = !a.a_kmajor; P.b_mn = !a.b_kmajor;
    // the GELU' multiply reads its bf16 operand by TMA prefetch (two smem
    // slots of BM x bn): tiles of at most 128 columns leave room for them
    const bool aux_tma = PTCG_AUX_TMA && a.act == ACT_GELU_BWD && a.aux && a.aux_dtype == DT_BF16 &&
                         !((uintptr_t)a.aux & 15) && (a.ld_aux * 2) % 16 == 0 && a.remap_group == 0;
    const int bn_max = aux_tma ? PTCG_AUX_BN_MAX : 256;
    int ntl = (a.N + bn_max - 1) / bn_max;
    int bn = ((a.N + ntl - 1) / ntl + 15) / 16 * 16;
    if (P.b_mn) bn = (bn + ATOM - 1) / ATOM * ATOM;
    if (bn > bn_max) bn = bn_max;
    if (aux_tma && bn % 32) bn = (bn + 31) / 32 * 32;
    P.bn = bn;
    P.b_rows = bn;
    bool plain = a.accumulate && a.out_dtype == DT_F32 && !a.bias && !a.bcast &&
                 a.act == ACT_NONE && !a.resid && !a.out2 && a.remap_group == 0 && !a.colsum;
    // the weight-gradient form (fp32 accumulate, no epilogue operand): CTA
    // tiles of 256 rows, two M = 128 MMAs on each B stage, which cuts the
    // operand bytes each SM pulls through L2 per FLOP by a third
    P.m2 = (PTCG_GEMM_M2 && plain && a.M > BM) ? 1 : 0;   // runs on <EB, NUM_EPI_LIGHT, EPI_GENERIC>
    P.m_tiles = (a.M + (BM << P.m2) - 1) / (BM << P.m2);
    P.n_tiles = (a.N + bn - 1) / bn;
    P.kb_total = (a.K + BK - 1) / BK;
    int tiles = P.m_tiles * P.n_tiles;
    P.splits = 1;
    if (plain && tiles < g_sms && P.kb_total >= 8) {
        // one wave: tiles x splits <= SMs (a split item is a long K range,
        // so even one CTA with a second item doubles the launch)
        int want = g_sms / tiles;
        int maxs = P.kb_total / 4;
        P.splits = want < maxs ? want : maxs;
        if (P.splits < 1) P.splits = 1;
    }
    P.kb_per_split = (P.kb_total + P.splits - 1) / P.splits;
    P.splits = (P.kb_total + P.kb_per_split - 1) / P.kb_per_split;   // no empty splits
    P.a_bytes = (BM * 128) << P.m2;
    P.stage_bytes = P.a_bytes + P.b_rows * 128;
    // outputs through smem + TMA store: plain row mapping, no read-modify-
    // write, whole 32-column chunks per tile, 16-byte aligned pitch
    int oeb = a.out_dtype == DT_F32 ? 4 : 2;
    // a row remap keeps the TMA store when its groups are whole store boxes
    // (each box then lands on consecutive output rows): 32-row boxes, or
    // four 8-row boxes per chunk when the groups are multiples of 8 only;
    // the map then spans the remapped rows
    const bool remap_ok = a.remap_group == 0 ||
        (a.remap_group % 8 == 0 && a.M % a.remap_group == 0 && !a.out2 &&
         a.remap_off + a.remap_group <= a.remap_stride);
    P.box_rows = (a.remap_group > 0 && a.remap_group % 32 != 0) ? 8 : 32;
    P.tma_out = P.splits == 1 && remap_ok && !a.accumulate && (bn % 32) == 0 &&
                !((uintptr_t)a.out & 15) && (a.ldo * oeb) % 16 == 0 &&
                (!a.out2 || (a.act == ACT_GELU && a.out2_dtype == a.out_dtype &&
                             (a.out_dtype == DT_BF16 || !a.resid) &&   // fp32: t holds GELU' to the store
                             !((uintptr_t)a.out2 & 15) && (a.ldo2 * oeb) % 16 == 0));
    P.bias_smem = (PTCG_BIAS_SMEM && a.bias && a.N <= BIAS_SMEM_MAX) ? a.N : 0;
    P.aux_tma = aux_tma && P.splits == 1;
    P.aux_bytes = P.aux_tma ? (uint32_t)(bn / 32) * 8192u : 0u;
    P.nepi = a.act == ACT_GELU ? NUM_EPI : NUM_EPI_LIGHT;
    // specialised epilogues: exactly the argument sets of the FFN1 forward
    // (bias + GELU + saved GELU') and the FFN2 dX (GELU' multiply + FFN1
    // bias column sums) of the transformer blocks in bf16
    const bool simple = eb == 2 && P.tma_out && a.alpha == 1.f && !a.bcast &&
                        !a.accumulate && a.remap_group == 0 && P.splits == 1;
    P.ek = EPI_GENERIC;
    if (simple && a.act == ACT_GELU && a.out2 && P.bias_smem > 0 && !a.colsum && !a.resid)
        P.ek = EPI_GELU_SAVE;
    else if (simple && a.act == ACT_GELU && !a.out2 && P.bias_smem > 0 && !a.colsum && !a.resid)
        P.ek = EPI_GELU;
    else if (simple && a.act == ACT_GELU_BWD && P.aux_tma && !a.bias && !a.out2 && !a.resid &&
             a.out_dtype == DT_BF16 && P.box_rows == 32)
        P.ek = EPI_GELU_AUX;
    else if (simple && a.act == ACT_NONE && !a.out2 && (!a.bias || P.bias_smem > 0))
        P.ek = EPI_PLAIN + (a.bias ? 1 : 0) + (a.resid ? 2 : 0);
    if (P.ek == EPI_GELU_AUX) P.nepi = NUM_EPI_AUX;
    // the GELU'-multiply epilogue stores from the aux slot itself
    P.staging_bytes = (P.tma_out && P.ek != EPI_GELU_AUX) ? (uint32_t)(P.nepi * STAGE_W) : 0u;
    int budget = 232448 - 1024 - 512 - (int)P.staging_bytes - P.bias_smem * 4 - 2 * (int)P.aux_bytes;
    P.stages = budget / P.stage_bytes;
    if (P.stages > 6) P.stages = 6;
    if (P.stages < 2) return false;
    P.acc_stride = (bn <= 128 && !P.m2) ? 128 : 256;
    P.tmem_cols = 2 * P.acc_stride;
    // instruction descriptor: f32 accumulate, A/B format (1 bf16, 2 tf32),
    // majorness, N>>3, M>>4
    uint32_t fmt = eb == 2 ? 1u : 2u;
    P.idesc = (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)P.a_mn << 15) |
              ((uint32_t)P.b_mn << 16) | ((uint32_t)(bn >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
    P.ep = a;
    pl.eb = eb;
    bool ok;
    if (P.a_mn) ok = make_map_eb(&pl.ma, a.A, a.M, a.K, a.lda, ATOM, BK, eb, true);
    else ok = make_map_eb(&pl.ma, a.A, a.K, a.M, a.lda, BK, BM, eb, false);
    if (!ok) return false;
    if (P.b_mn) ok = make_map_eb(&pl.mb, a.B, a.N, a.K, a.ldb, ATOM, BK, eb, true);
    else ok = make_map_eb(&pl.mb, a.B, a.K, a.N, a.ldb, BK, bn, eb, false);
    if (!ok) return false;
    pl.mc = pl.ma; pl.mc2 = pl.ma; pl.mx = pl.ma;
    if (P.aux_tma && !make_aux_map(&pl.mx, a.aux, a.N, a.M, a.ld_aux)) return false;
    if (P.tma_out) {
        const long out_rows = a.remap_group > 0 ? (long)(a.M / a.remap_group) * a.remap_stride : a.M;
        if (!make_out_map(&pl.mc, a.out, a.N, out_rows, a.ldo, a.out_dtype, P.box_rows)) return false;
        if (a.out2 && !make_out_map(&pl.mc2, a.out2, a.N, a.M, a.ldo2, a.out2_dtype)) return false;
    }
    return true;
}

void launch_tc(const TcPlan& pl, cudaStream_t s) {
    const TcParams& P = pl.P;
    size_t smem = 1024 + (size_t)P.stages * P.stage_bytes + (size_t)P.staging_bytes +
                  2 * (size_t)P.aux_bytes + (2 * P.stages + 9) * 8 + 48 + (size_t)P.bias_smem * 4;
    int total = P.m_tiles * P.n_tiles * P.splits;
    int grid = total < g_sms ? total : g_sms;
#define PTCG_TC_LAUNCH(EBV, NV, EKV)                                                         \
    do {                                                                                     \
        cudaFuncSetAttribute(k_gemm_tc<EBV, NV, EKV>,                                        \
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);        \
        ++g_ptcg_launches, k_gemm_tc<EBV, NV, EKV><<<grid, threads_for(NV), smem, s>>>(       \
            pl.ma, pl.mb, pl.mc, pl.mc2, pl.mx, P);                                          \
    } while (0)
    if (P.ek == EPI_GELU_SAVE) PTCG_TC_LAUNCH(2, NUM_EPI, EPI_GELU_SAVE);
    else if (P.ek == EPI_GELU) PTCG_TC_LAUNCH(2, NUM_EPI, EPI_GELU);
    else if (P.ek == EPI_GELU_AUX) PTCG_TC_LAUNCH(2, NUM_EPI_AUX, EPI_GELU_AUX);
    else if (P.ek == EPI_PLAIN) PTCG_TC_LAUNCH(2, NUM_EPI_LIGHT, EPI_PLAIN);
    else if (P.ek == EPI_BIAS) PTCG_TC_LAUNCH(2, NUM_EPI_LIGHT, EPI_BIAS);
    else if (P.ek == EPI_RESID) PTCG_TC_LAUNCH(2, NUM_EPI_LIGHT, EPI_RESID);
    else if (P.ek == EPI_BIAS_RESID) PTCG_TC_LAUNCH(2, NUM_EPI_LIGHT, EPI_BIAS_RESID);
    else if (pl.eb == 2 && P.nepi == NUM_EPI) PTCG_TC_LAUNCH(2, NUM_EPI, EPI_GENERIC);
    else if (pl.eb == 2) PTCG_TC_LAUNCH(2, NUM_EPI_LIGHT, EPI_GENERIC);
    else if (P.nepi == NUM_EPI) PTCG_TC_LAUNCH(4, NUM_EPI, EPI_GENERIC);
    else PTCG_TC_LAUNCH(4, NUM_EPI_LIGHT, EPI_GENERIC);
#undef PTCG_TC_LAUNCH
}

}  // namespace

bool gemm_tc_supported(const GemmArgs& a) {
    TcPlan pl;
    return plan_tc(a, pl);
}

bool gemm_tc(const GemmArgs& a, cudaStream_t s) {
    TcPlan pl;
    if (!plan_tc(a, pl)) return false;
    launch_tc(pl, s);
    return true;
}
