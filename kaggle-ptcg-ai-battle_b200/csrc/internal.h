// Internal launcher interfaces shared by the ptcg_b200 translation units.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

enum { DT_F32 = 0, DT_BF16 = 1 };

// number of kernels this library has launched (every launch site increments it)
extern std::atomic<long long> g_ptcg_launches;
enum { ACT_NONE = 0, ACT_GELU = 1, ACT_GELU_BWD = 2 };

// C[m, n] = epilogue( alpha * sum_k A(m, k) * B(n, k) )
//   A(m,k) = a_kmajor ? A[m*lda + k] : A[k*lda + m]
//   B(n,k) = b_kmajor ? B[n*ldb + k] : B[k*ldb + n]
// epilogue, in order: + bias[n]; + bcast[(m / bcast_group) * ld_bcast + n];
//   act (GELU: out2, if set, receives GELU'(pre-activation) -- the factor
//   the backward needs, so it never re-evaluates erf; GELU_BWD: * aux[m, n],
//   the saved GELU');
//   output row r = remap(m); + resid[r * ld_resid + n]; + out[r, n] if
//   accumulate; store to out (f32 or operand dtype); for act != GELU an out2
//   receives a second copy of the final value.
struct GemmArgs {
    int M = 0, N = 0, K = 0;
    int dtype = DT_F32;                      // operand dtype (A and B)
    const void* A = nullptr; long lda = 0; int a_kmajor = 1;
    const void* B = nullptr; long ldb = 0; int b_kmajor = 1;
    float alpha = 1.f;
    const float* bias = nullptr;
    const float* bcast = nullptr; long ld_bcast = 0; int bcast_group = 1;
    int act = ACT_NONE;
    const void* aux = nullptr; long ld_aux = 0; int aux_dtype = DT_F32;
    int remap_group = 0, remap_stride = 0, remap_off = 0;
    const float* resid = nullptr; long ld_resid = 0;
    void* out = nullptr; long ldo = 0; int out_dtype = DT_F32; int accumulate = 0;
    void* out2 = nullptr; long ldo2 = 0; int out2_dtype = DT_F32;
    // colsum[n] += sum_m (final value) in fp32, before any rounding to the
    // output dtype (bias gradients of the next Linear down)
    float* colsum = nullptr;
    // fp32 operands may run on TF32 tensor cores (10-bit mantissa); 0 = exact fp32
    int allow_tf32 = 0;
};

void gemm_simt(const GemmArgs& a, cudaStream_t s);
// tcgen05 path: returns false if the problem is not supported (caller falls
// back to the SIMT kernel, which is also sm_100a code in this library)
bool gemm_tc(const GemmArgs& a, cudaStream_t s);
bool gemm_tc_supported(const GemmArgs& a);
bool gemm_tc_available();
// 2-D TMA tensor map (inner x outer elements, row pitch ld elements, box
// box_in x box_out, swizzle 0 / 32 / 64 / 128 bytes); false if unavailable
bool tc_make_map_2d(CUtensorMap* m, const void* ptr, int dtype, long inner, long outer, long ld,
                    int box_in, int box_out, int swizzle_bytes);
int tc_num_sms();
// first error code recorded by a tcgen05 kernel since the last call (0 = none)
int ptcg_tc_error_read_reset();
int ptcg_tc_profile_ctl(int enable, unsigned long long* out8);

// per-sequence key words of the tcgen05 attention: word j < 15 holds the
// kept bits of keys 32j .. 32j+31 (none at or past the extent), word 15 the
// extent; ATTN_KW_WORDS uint32 per sequence, rows 64-byte aligned
constexpr int ATTN_KW_WORDS = 16;

// attention over packed qkv rows: qkv [(n*L + l) * ldqkv + {0,D,2D} + h*32 + d]
// extent (nullable, bf16 path): per sequence, the rows anything reads;
// query rows at or past it get zero output and a zero log-sum-exp.
// kw (nullable): the key words of (keep, extent), which the tcgen05 path
// otherwise builds itself
void attn_fwd(int dtype, const void* qkv, long ldqkv, const uint8_t* keep,
              void* out, long ldo, float* lse, int nseq, int L, int H,
              cudaStream_t s, const int* extent = nullptr, const uint32_t* kw = nullptr);
// first query row of each sequence only: q row of sequence n at
// q + n * ldq, keys / values as rows [K | V] of kv (row stride ldkv,
// sequence n at rows n * L ..); out / dout [n * ldo + h*32 + d], lse
// [n * H + h]; the backward writes dq (one row per sequence) and dK / dV of
// every row, and adds the [q | k | v] bias grads to dbias.  H <= 16.
void attn_row0_fwd(int dtype, const void* q, long ldq, const void* kv, long ldkv,
                   const uint8_t* keep, void* out, long ldo, float* lse, int nseq, int L, int H,
                   cudaStream_t s);
void attn_row0_bwd(int dtype, const void* q, long ldq, const void* kv, long ldkv,
                   const uint8_t* keep, const void* out, long ldo, const void* dout, long lddo,
                   const float* lse, void* dq, long lddq, void* dkv, long lddkv, float* dbias,
                   int nseq, int L, int H, cudaStream_t s);
// tcgen05 / TMEM attention (attention_tc.cu), bf16 operands: false when the
// shape or alignment is not supported (the caller runs the mma.sync kernels)
bool attn_fwd_tc(const void* qkv, long ldqkv, const uint32_t* kw, void* out, long ldo,
                 float* lse, int nseq, int L, int H, cudaStream_t s);
// backward of the sequences whose extent is at most 128 rows (one tile);
// their rows past 128 get zero dqkv; the caller runs the mma.sync backward
// for the others
bool attn_bwd_tc(const void* qkv, long ldqkv, const uint32_t* kw, const void* out, long ldo,
                 const void* dout, long lddo, const float* lse, void* dqkv, long lddqkv,
                 float* dbias, int nseq, int L, int H, cudaStream_t s);
// the key words of (keep, extent) (extent nullable: every row) into kw
void attn_keep_words(uint32_t* kw, const uint8_t* keep, const int* extent, int nseq, int L,
                     cudaStream_t s);
// which bf16 attention passes run the tcgen05 kernels instead of the
// mma.sync ones: impl 0 none, 1 both, 2 the backward only (attn_set_impl,
// or PTCG_ATTN_TC=<impl> at load)
bool attn_tc_fwd();
bool attn_tc_bwd();
void attn_set_impl(int impl);
int attn_get_impl();
// first error code recorded by a tcgen05 attention kernel since the last call
int attn_tc_error_read_reset();
// dbias (nullable, 3*H*32 floats): += column sums of dqkv in fp32
void attn_bwd(int dtype, const void* qkv, long ldqkv, const uint8_t* keep,
              const void* out, long ldo, const void* dout, long lddo,
              const float* lse, void* dqkv, long lddqkv, float* dbias, int nseq, int L,
              int H, cudaStream_t s, const int* extent = nullptr, const uint32_t* kw = nullptr);

// ---- native data-parallel exchange (dp_nccl.cu); every int function
// returns 0 on success, else nonzero with the text in dp_last_error()
constexpr int DP_UID_BYTES = 128;
struct DpState;
const char* dp_last_error();
int dp_unique_id(void* out128);
// spans: nspans {arena offset, count} pairs in the order backward finalises
// them; they must tile [0, n_arena).  Collective over the world's ranks.
int dp_create(DpState** out, const void* uid, int rank, int world, int dev, const long* spans,
              int nspans, long n_arena);
void dp_destroy(DpState* d, bool abort);
int dp_bucket(DpState* d, const float* grads, long off, long count, cudaStream_t s);
int dp_join(DpState* d, cudaStream_t s, int* spans_seen);
int dp_nbuckets(DpState* d);
float* dp_shard(DpState* d, long* used, const long** seg, int* nseg, double** sumsq);
int dp_allreduce_sum_f64(DpState* d, double* x, cudaStream_t s);
int dp_gather_params(DpState* d, float* params, cudaStream_t s);
int dp_weights_agree(DpState* d, const unsigned int* ck_dev, long long* minmax_dev,
                     cudaStream_t s);

// ---- fused rollout MLP (mlp_tc.cu): out = res + b2 + GELU(a W1^T + b1) W2^T on
// tcgen05 with the hidden activation kept on chip; false when the shape or
// alignment is not supported (the caller runs the two GEMMs).  D must be 256.
bool mlp_fwd_tc(const void* a, long lda, const void* w1, long ldw1, const float* b1,
                const void* w2, long ldw2, const float* b2, const float* res, long ld_res,
                float* out, long ld_out, int rows, int D, int F, cudaStream_t s);
int mlp_tc_error_read_reset();
