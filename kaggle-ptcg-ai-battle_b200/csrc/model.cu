// ptcg_b200: model state, workspaces, forward / backward orchestration and
// the extern "C" entry points declared in include/ptcg_b200.h.
//
// Dataflow follows ptcg_forward_core / ptcg_backward_core of the reference
// (native/model/ptcg_model3.cu:246-369, ptcg_model4.cu:10-190) and the torch
// model (ptcg/rl/model.py:185-341); the kernels and layouts are this
// library's own:
//  * activations are row-major with leading dimensions padded to 8 elements
//    (16-byte rows for TMA); GEMM operands are bf16 in PTCG_BF16 mode and fp32
//    in PTCG_FP32 mode, the residual stream, LayerNorm statistics, heads and
//    all gradients of the residual stream stay fp32;
//  * attention never materialises probabilities (online softmax, LSE saved);
//  * concat-then-Linear of gathered table rows becomes Linear-per-table-row
//    then gather where the table is small (opt_card / opt_attack);
//  * the static card / attack / skill tables are built once per train step
//    and their gradient is accumulated across micro-batches;
//  * every GELU layer saves GELU'(pre-activation) (the buffers named *pre),
//    so the backward multiplies instead of re-evaluating erf.
#include "kernels.cuh"
#include "ptcg_b200.h"

#include <stdarg.h>
#include <stdio.h>
#include <unistd.h>
#include <string.h>

#include <string>
#include <vector>
#include <algorithm>
#include <mutex>
#include <unordered_map>

std::atomic<long long> g_ptcg_launches{0};
// the rollout forward's fused MLP kernel (ptcg_set_fused_mlp; off: slower
// than the two GEMMs on this part, see mlp_tc.cu)
static std::atomic<int> g_fused_mlp{0};

// ------------------------------------------------------------------ errors
static thread_local char g_err[1024];
static void set_err(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
}
#define CK(x) do { cudaError_t _e = (x); if (_e != cudaSuccess) { \
    set_err("%s failed: %s (%s:%d)", #x, cudaGetErrorString(_e), __FILE__, __LINE__); \
    return PTCG_ECUDA; } } while (0)
#define CKL() CK(cudaGetLastError())
#define REQ(cond, code, ...) do { if (!(cond)) { set_err(__VA_ARGS__); return code; } } while (0)

static const int TPB = 256;
static inline long rup(long x, long a) { return (x + a - 1) / a * a; }

// ------------------------------------------------------------- param table
struct ParamDef { std::string name; long r, c; };

static void blk_defs(std::vector<ParamDef>& v, const std::string& p, int d, int f) {
    v.push_back({p + "ln1_w", d, 0}); v.push_back({p + "ln1_b", d, 0});
    v.push_back({p + "qkv_w", 3L * d, d}); v.push_back({p + "qkv_b", 3L * d, 0});
    v.push_back({p + "proj_w", d, d}); v.push_back({p + "proj_b", d, 0});
    v.push_back({p + "ln2_w", d, 0}); v.push_back({p + "ln2_b", d, 0});
    v.push_back({p + "ffn1_w", f, d}); v.push_back({p + "ffn1_b", f, 0});
    v.push_back({p + "ffn2_w", d, f}); v.push_back({p + "ffn2_b", d, 0});
}

// PT_PARAMS order (native/model/ptcg_model.cu:95-126)
static std::vector<ParamDef> param_defs(const PtcgShape& s) {
    const int d = s.d, dc = 128, da = 64, g = 128;
    const int tok_in = 2 * dc + s.tok_f + 12, q_in = 16 + 2 * d + 136;
    const int score_in = 3 * d + 192, val_in = d + 128;
    std::vector<ParamDef> v = {
        {"card_id_emb", s.n_cards, 64}, {"attack_id_emb", s.n_attacks, 48},
        {"skill_id_emb", s.n_skills, 48},
        {"attack_mlp_w", da, 127}, {"attack_mlp_b", da, 0},
        {"skill_mlp_w", dc, 112}, {"skill_mlp_b", dc, 0},
        {"card_ln_w", 634, 0}, {"card_ln_b", 634, 0},
        {"card_mlp1_w", 256, 634}, {"card_mlp1_b", 256, 0},
        {"card_mlp2_w", dc, 256}, {"card_mlp2_b", dc, 0},
        {"zone_emb", 16, 8}, {"owner_emb", 4, 4},
        {"token_proj_w", d, tok_in}, {"token_proj_b", d, 0},
        {"readout", d, 0},
        {"global1_w", g, 64}, {"global1_b", g, 0}, {"global2_w", g, g}, {"global2_b", g, 0},
        {"sel_type_emb", 29, 8}, {"ctx_emb", 65, 32},
        {"dec1_w", 64, 696}, {"dec1_b", 64, 0}, {"dec2_w", 64, 64}, {"dec2_b", 64, 0},
        {"bcast_w", d, 192}, {"bcast_b", d, 0},
    };
    for (int i = 0; i < s.layers; i++) blk_defs(v, "b" + std::to_string(i) + "_", d, s.ffn);
    std::vector<ParamDef> t2 = {
        {"lnf_w", d, 0}, {"lnf_b", d, 0},
        {"opt_type_emb", 33, 16},
        {"opt_card_w", 64, dc}, {"opt_card_b", 64, 0},
        {"opt_attack_w", 64, da}, {"opt_attack_b", 64, 0},
        {"q1_w", d, q_in}, {"q1_b", d, 0}, {"q2_w", d, d}, {"q2_b", d, 0},
        {"score1_w", 256, score_in}, {"score1_b", 256, 0},
        {"score2_w", 1, 256}, {"score2_b", 1, 0},
        {"value1_w", 256, val_in}, {"value1_b", 256, 0},
        {"value2_w", 1, 256}, {"value2_b", 1, 0},
        {"oracle_proj_w", d, 134}, {"oracle_proj_b", d, 0},
        {"critic_readout", d, 0},
    };
    v.insert(v.end(), t2.begin(), t2.end());
    blk_defs(v, "c0_", d, s.ffn);
    std::vector<ParamDef> t3 = {
        {"oracle_v1_w", 256, val_in}, {"oracle_v1_b", 256, 0},
        {"oracle_v2_w", 1, 256}, {"oracle_v2_b", 1, 0},
        {"aux_hand_w", s.n_cards, val_in}, {"aux_hand_b", s.n_cards, 0},
        {"aux_prize_w", 1, d}, {"aux_prize_b", 1, 0},
    };
    v.insert(v.end(), t3.begin(), t3.end());
    return v;
}

static long numel(const ParamDef& p) { return p.c > 0 ? p.r * p.c : p.r; }

// ------------------------------------------------------------ model state
struct Dims {
    int D, H, FFN, LAYERS, LTOK, LSEQ, NOPT, LCRIT, NC, NA, NS, TOKF;
    int TOK_IN, Q_IN, SCORE_IN, VAL_IN;
    ObsLayout ol;
};

struct W { float* p; float* g; const void* op; long ld; };   // param + GEMM operand

struct BlkW { W ln1w, ln1b, qkvw, qkvb, projw, projb, ln2w, ln2b, f1w, f1b, f2w, f2b; };

struct BlkAct {
    float *x_in, *x_out;
    void *ln1, *qkv, *att, *ln2, *fpre, *fpost;
    void* q0;                           // readout-row blocks: query rows [R, D]; qkv holds [K | V]
    float *mu1, *rs1, *mu2, *rs2, *lse, *xm;
};

struct Work {
    int R = 0, train = 0;
    void* base = nullptr; size_t bytes = 0;
    // per-sample / token buffers
    void* tokcat; uint8_t* keep; uint8_t* ckeep;
    float *g1pre, *g1, *gd, *decin, *d1pre, *d1, *bc;
    std::vector<float*> x;              // trunk states (LAYERS+1 train, 2 rollout)
    std::vector<BlkAct> blk;            // per layer (train) / 1 shared (rollout)
    float* h; float *muf, *rsf;
    void *qin, *q1pre, *q1; void *scin, *s1pre, *s1;
    float *u, *rgd, *wqq, *du, *drgd;   // score1 split: per-sample term, inputs, packed W
    void* otokin; float* xc[2]; BlkAct cblk;
    int* ext;                                 // [R] trunk rows anything reads (k_row_extent)
    uint32_t* kw;                             // [R][ATTN_KW_WORDS] attention key words
    float *ovin, *ov1pre, *ov1; float* out;
    // train-only heads
    float *bvin; void* bvinc; float *bv1pre, *bv1, *blind_v, *hand_lin, *prize_logit;
    // backward scratch
    float *dh, *dgd, *dbvin, *d_v1pre, *dscores, *dscin, *dqin, *dtokcat, *ddecin, *dd1,
          *dg1, *dbc, *dotokin, *dx, *dln, *dx0;
    void* dq0;                          // readout-row block: d query rows [R, D]
    void *dx0c, *dxc, *dhand, *ds1pre, *dq, *dq1, *dotok, *dtokp, *df, *datt, *dqkv;
    float* dgrad;                       // PPO grad for one micro-batch (train_step)
    float* fused;                       // fused [scores | value] of one micro-batch
    float *ppo_scratch, *nlp, *ratio;
};

struct Tab {                            // batch-independent table activations + grads
    float *att_in, *att_pre, *att_tab, *sk_in, *sk_pre, *sk_tab;
    float *a_mean_max_dummy;
    float *card_in, *card_ln, *ln_mu, *ln_rs, *h1pre, *h1, *card_vec, *poc, *poa;
    int8_t *a_arg, *s_arg;
    float *d_cv, *d_att, *d_sk, *d_poc, *d_poa, *d_h1, *d_cardln, *d_cardin, *d_attin, *d_skin;
};

// CUDA-event timing of one GEMM kernel class over a region (bench roofline)
struct KTimer {
    int mode = 0;                       // 0 off, 1 tensor-core GEMM, 2 SIMT GEMM, 3 all GEMMs,
                                        // 4 the Adam kernels of ptcg_adam_step
    std::vector<cudaEvent_t> ev;
    int used = 0;
    double flops = 0.0;
    double bytes = 0.0;                 // algorithmic HBM bytes of the timed launches
    long launches = 0;
    std::vector<int> meta;              // per timed launch: M N K a_kmajor b_kmajor act engine dtype
};

struct PtcgModel {
    PtcgShape s;
    KTimer kt;
    Dims z;
    int prec, dev;
    std::vector<ParamDef> defs;
    std::vector<long> off;
    std::unordered_map<std::string, int> idx;
    long n_arena = 0;
    float *params = nullptr, *grads = nullptr, *am = nullptr, *av = nullptr;
    long long* step_dev = nullptr;
    // bf16 compute copies
    std::vector<BfCopy> copies;
    std::vector<long> copy_ld;          // per param: ld of its copy (0 = none)
    std::vector<bf16*> copy_ptr;
    bf16* wbf = nullptr;
    BfCopy* d_copies = nullptr;
    int* d_chunk_copy = nullptr;
    int adam_chunk = 4096, adam_grid = 0, sumsq_grid = 0;
    double* d_partials = nullptr;
    // Muon scratch (orthogonalisation of the >= 2-D parameters)
    float *mu_gram = nullptr, *mu_gram2 = nullptr, *mu_x = nullptr;
    double* mu_partials = nullptr;
    float* d_misc = nullptr;            // [0..1] adv stats, [2] prize count, [4..19] stats, [32..] adam stats
    unsigned int* d_ck = nullptr;
    // static tables
    float *card_static = nullptr, *att_static = nullptr, *card_text = nullptr,
          *att_text = nullptr, *skill_text = nullptr;
    int *card_attacks = nullptr, *card_skills = nullptr;
    bool tables_ready = false, weights_ready = false;
    // tab holds the static-table activations of the current weights: every
    // call that changes the master weights (optimizer steps, loads, imports,
    // ptcg_refresh_copies) recomputes them, so forwards skip that work
    bool tab_fresh = false;
    Tab tab;
    void* tab_base = nullptr;
    Work roll, trn;
    ptcg_grad_hook hook = nullptr;
    void* hook_user = nullptr;
    DpState* dp = nullptr;              // native data-parallel exchange (ptcg_dp_init)
    bool dp_fail = false;               // a span's reduce-scatter could not be issued
    const float* trn_last_obs = nullptr;
    int trn_last_n = 0;
    int esz() const { return prec == PTCG_BF16 ? 2 : 4; }
    int dt() const { return prec == PTCG_BF16 ? DT_BF16 : DT_F32; }
    W w(const char* name) const {
        auto it = idx.find(name);
        int i = it->second;
        W r;
        r.p = params + off[i];
        r.g = grads + off[i];
        if (prec == PTCG_BF16 && copy_ptr[i]) { r.op = copy_ptr[i]; r.ld = copy_ld[i]; }
        else { r.op = r.p; r.ld = defs[i].c; }
        return r;
    }
    BlkW blk(const std::string& p) const {
        BlkW b;
        b.ln1w = w((p + "ln1_w").c_str()); b.ln1b = w((p + "ln1_b").c_str());
        b.qkvw = w((p + "qkv_w").c_str()); b.qkvb = w((p + "qkv_b").c_str());
        b.projw = w((p + "proj_w").c_str()); b.projb = w((p + "proj_b").c_str());
        b.ln2w = w((p + "ln2_w").c_str()); b.ln2b = w((p + "ln2_b").c_str());
        b.f1w = w((p + "ffn1_w").c_str()); b.f1b = w((p + "ffn1_b").c_str());
        b.f2w = w((p + "ffn2_w").c_str()); b.f2b = w((p + "ffn2_b").c_str());
        return b;
    }
};

// ---------------------------------------------------------------- helpers
static void kt_mark(PtcgModel* M, cudaStream_t s) {
    KTimer& k = M->kt;
    if (k.used >= (int)k.ev.size()) {
        cudaEvent_t e;
        cudaEventCreate(&e);
        k.ev.push_back(e);
    }
    cudaEventRecord(k.ev[k.used++], s);
}

// Algorithmic HBM bytes of one GEMM launch: each operand read once, each
// output written once, plus the epilogue's extra operand streams (saved
// GELU' / residual / read-back of an accumulated output).  Bias and
// broadcast rows are negligible and left out.
static double gemm_bytes(const GemmArgs& a) {
    double eb = a.dtype == DT_BF16 ? 2.0 : 4.0, ob = a.out_dtype == DT_BF16 ? 2.0 : 4.0;
    double mn = (double)a.M * a.N;
    double b = ((double)a.M + a.N) * a.K * eb + mn * ob;
    if (a.out2) b += mn * (a.out2_dtype == DT_BF16 ? 2.0 : 4.0);
    if (a.aux) b += mn * (a.aux_dtype == DT_BF16 ? 2.0 : 4.0);
    if (a.resid) b += mn * 4.0;
    if (a.accumulate) b += mn * ob;
    return b;
}

static void gemm(PtcgModel* M, const GemmArgs& a, cudaStream_t s) {
    bool tc_ok = (a.dtype == DT_BF16 || a.allow_tf32) && gemm_tc_supported(a);
    int cls = tc_ok ? 1 : 2;
    bool timed = M->kt.mode == cls || M->kt.mode == 3;
    if (timed) kt_mark(M, s);
    bool done = tc_ok && gemm_tc(a, s);
    if (!done) gemm_simt(a, s);
    if (timed) {
        kt_mark(M, s);
        M->kt.flops += 2.0 * a.M * a.N * a.K;
        M->kt.bytes += gemm_bytes(a);
        M->kt.launches++;
        int meta[8] = {a.M, a.N, a.K, a.a_kmajor, a.b_kmajor, a.act, cls, a.dtype};
        M->kt.meta.insert(M->kt.meta.end(), meta, meta + 8);
    }
}

// C[M,N] (+)= op(A) op(B)^T helpers for the three GEMM shapes of a Linear
// y = x W^T + b with W [out, in]:
//   fwd : y[M=rows, N=out]   = x[rows, in] . W[out, in]^T
//   dX  : dx[M=rows, N=in]   = dy[rows, out] . W[out, in]
//   dW  : dW[M=out, N=in]   += dy[rows, out]^T . x[rows, in]
static GemmArgs lin_fwd(int dt, int rows, int in, int out, const void* x, long ldx, const W& w,
                        void* y, long ldy, int y_dt) {
    GemmArgs a;
    a.M = rows; a.N = out; a.K = in; a.dtype = dt;
    a.A = x; a.lda = ldx; a.a_kmajor = 1;
    a.B = w.op; a.ldb = w.ld; a.b_kmajor = 1;
    a.out = y; a.ldo = ldy; a.out_dtype = y_dt;
    return a;
}
static GemmArgs lin_dx(int dt, int rows, int in, int out, const void* dy, long lddy, const W& w,
                       void* dx, long lddx, int dx_dt) {
    GemmArgs a;
    a.M = rows; a.N = in; a.K = out; a.dtype = dt;
    a.A = dy; a.lda = lddy; a.a_kmajor = 1;
    a.B = w.op; a.ldb = w.ld; a.b_kmajor = 0;
    a.out = dx; a.ldo = lddx; a.out_dtype = dx_dt;
    return a;
}
static GemmArgs lin_dw(int dt, int rows, int in, int out, const void* dy, long lddy,
                       const void* x, long ldx, float* dw) {
    GemmArgs a;
    a.M = out; a.N = in; a.K = rows; a.dtype = dt;
    a.A = dy; a.lda = lddy; a.a_kmajor = 0;
    a.B = x; a.ldb = ldx; a.b_kmajor = 0;
    a.out = dw; a.ldo = in; a.out_dtype = DT_F32; a.accumulate = 1;
    return a;
}
// fp32-operand GEMM of the small per-sample / per-table layers: TF32 tensor
// cores in bf16 mode (shapes the TMA path cannot take fall back to SIMT),
// the exact SIMT kernel in fp32 parity mode
static void gemm32(PtcgModel* M, GemmArgs a, cudaStream_t s) {
    a.allow_tf32 = M->prec == PTCG_BF16;
    gemm(M, a, s);
}

// view of rows r0.. of a [rows x cols] parameter (operand, master and grad)
static W wrows(const W& w, long r0, long cols, int esz) {
    W r = w;
    r.p = w.p + r0 * cols;
    r.g = w.g + r0 * cols;
    r.op = (const char*)w.op + r0 * w.ld * esz;
    return r;
}
// fp32 operand view of a parameter (per-sample / table GEMMs stay fp32)
static W f32w(const W& w, long cols) { W r = w; r.op = w.p; r.ld = cols; return r; }

template <typename T> static void colsum(float* out, const T* in, long ld, int rows, int cols,
                                         cudaStream_t s) {
    if (rows <= 0) return;
    if (sizeof(T) == 4 && (cols == 128 || cols == 256) && ld % 4 == 0 && !((uintptr_t)in & 15)) {
        // warp per row, float4 columns, block partials (k_colsum_rowset)
        unsigned g = std::min<unsigned>(cdiv(rows, 8), 1184);
        if (cols == 128)
            ++g_ptcg_launches, k_colsum_rowset<1><<<g, 256, 0, s>>>(out, (const float*)in, ld, rows, 1, 0, 1);
        else
            ++g_ptcg_launches, k_colsum_rowset<2><<<g, 256, 0, s>>>(out, (const float*)in, ld, rows, 1, 0, 1);
        return;
    }
    int rpb = 256;
    dim3 g(cdiv(cols, 128), cdiv(rows, rpb));
    ++g_ptcg_launches, k_colsum<T><<<g, 128, 0, s>>>(out, in, ld, rows, cols, rpb);
}

// ext / lseq (nullable / unused): rows of each lseq-row sequence anything
// reads (k_row_extent); the rest are skipped
// the vector LayerNorm kernels (D = 256 or 512) can read the critic's trunk
// rows straight from h and write their input grads straight into d_h
static bool crit_rows_direct(int D) { return D == 256 || D == 512; }

// crit_h (nullable; crit_rows_direct(D)): the rows are critic sequences whose
// trunk rows are read from crit_h (k_ln_fwd CRIT)
static void ln_fwd(int dt, void* y, long ldy, float* mu, float* rs, const float* x, long ldx,
                   const float* w, const float* b, int rows, int D, cudaStream_t s,
                   const int* ext = nullptr, int lseq = 1, const uint8_t* rowkeep = nullptr,
                   const float* crit_h = nullptr, int crit_lseq = 0, int crit_lcrit = 0) {
    unsigned g = cdiv(rows, 8);
    bool vec = D % 128 == 0 && D <= 1024 && ldx % 4 == 0 && ldy % 4 == 0;
    if (crit_h) {
#define LNFC(TO, V) ++g_ptcg_launches, k_ln_fwd<TO, V, true><<<g, 256, 0, s>>>((TO*)y, ldy, mu, rs, x, ldx, \
        w, b, rows, D, ext, lseq, rowkeep, crit_h, crit_lseq, crit_lcrit)
        if (D == 256) { if (dt == DT_F32) LNFC(float, 2); else LNFC(bf16, 2); }
        else { if (dt == DT_F32) LNFC(float, 4); else LNFC(bf16, 4); }
#undef LNFC
        return;
    }
#define LNF(TO, V) ++g_ptcg_launches, k_ln_fwd<TO, V><<<g, 256, 0, s>>>((TO*)y, ldy, mu, rs, x, ldx, w, b, rows, D, ext, lseq, rowkeep)
    if (vec && D == 256) { if (dt == DT_F32) LNF(float, 2); else LNF(bf16, 2); }
    else if (vec && D == 512) { if (dt == DT_F32) LNF(float, 4); else LNF(bf16, 4); }
    else { if (dt == DT_F32) LNF(float, 0); else LNF(bf16, 0); }
#undef LNF
}
// dx (f32, ld D) = LN'(dy) (+ dx), copy to dxc (T) unless dxc == nullptr
// out_cs (nullable): += column sums of the resulting dx.  dy is fp32, or in
// the operand dtype when dy_dt == DT_BF16 (the output of a dX GEMM)
static void ln_bwd(int dt, float* dx, int accumulate, void* dxc, float* dw, float* db,
                   const void* dy, const float* x, const float* w, const float* mu,
                   const float* rs, int rows, int D, cudaStream_t s, float* out_cs = nullptr,
                   int dy_dt = DT_F32, const int* ext = nullptr, int lseq = 1,
                   const uint8_t* rowkeep = nullptr, float* crit_dh = nullptr,
                   int crit_lseq = 0, int crit_lcrit = 0, const float* crit_h = nullptr) {
    int rpb = 64;
    unsigned g = cdiv(rows, rpb);
    size_t sm = 3 * D * sizeof(float);
    if (D % 128 != 0 || D > 512) { ext = nullptr; rowkeep = nullptr; }   // vector kernels only
#define LNB(TC, V, MC, TY) ++g_ptcg_launches, k_ln_bwd<TC, V, MC, TY><<<g, 256, sm, s>>>(dx, D, \
        accumulate, (TC*)dxc, D, dw, db, (const TY*)dy, D, x, D, w, mu, rs, rows, D, rpb, out_cs, \
        ext, lseq, rowkeep)
#define LNB2(TC, V, MC) do { if (dy_dt == DT_BF16) LNB(TC, V, MC, bf16); else LNB(TC, V, MC, float); } while (0)
    bool f = dt == DT_F32 || dxc == nullptr;
    if (crit_dh) {                              // critic rows: crit_rows_direct(D), dy in dt
#define LNBC(TC, V) ++g_ptcg_launches, k_ln_bwd<TC, V, 1, TC, true><<<g, 256, sm, s>>>(dx, D, \
        accumulate, (TC*)dxc, D, dw, db, (const TC*)dy, D, x, D, w, mu, rs, rows, D, rpb, out_cs, \
        ext, lseq, rowkeep, crit_dh, crit_lseq, crit_lcrit, crit_h)
        if (D == 256) { if (f) LNBC(float, 2); else LNBC(bf16, 2); }
        else { if (f) LNBC(float, 4); else LNBC(bf16, 4); }
#undef LNBC
        return;
    }
    if (D == 256) { if (f) LNB2(float, 2, 1); else LNB2(bf16, 2, 1); }
    else if (D == 512) { if (f) LNB2(float, 4, 1); else LNB2(bf16, 4, 1); }
    else if (D <= 256) { if (f) LNB2(float, 0, 8); else LNB2(bf16, 0, 8); }
    else if (D <= 512) { if (f) LNB2(float, 0, 16); else LNB2(bf16, 0, 16); }
    else { if (f) LNB2(float, 0, 32); else LNB2(bf16, 0, 32); }
#undef LNB2
#undef LNB
}

// ---------------------------------------------------------- workspace plan
struct Bump {
    char* base; size_t off; bool measure;
    void* take(size_t bytes) {
        off = (off + 255) & ~(size_t)255;
        void* p = measure ? nullptr : (void*)(base + off);
        off += bytes;
        return p;
    }
    float* f(long n) { return (float*)take((size_t)n * 4); }
};

// rows_out: rows per sequence computed past the attention (L, or 1 for a
// block whose output is read at its first row only)
static void plan_blk(BlkAct& b, Bump& m, int R, int L, int rows_out, const Dims& z, int esz,
                     bool train, bool alloc_x) {
    long NL = (long)R * L, NQ = (long)R * rows_out;
    if (alloc_x) { b.x_in = m.f(NL * z.D); }
    b.ln1 = m.take(NL * z.D * esz);
    b.qkv = m.take(NL * 3 * z.D * esz);
    b.att = m.take(NQ * z.D * esz);
    b.ln2 = m.take(NQ * z.D * esz);
    b.fpre = train ? m.take(NQ * z.FFN * esz) : nullptr;
    b.fpost = m.take(NQ * z.FFN * esz);
    b.mu1 = m.f(NL); b.rs1 = m.f(NL); b.mu2 = m.f(NQ); b.rs2 = m.f(NQ);
    b.q0 = rows_out == 1 ? m.take((long)R * z.D * esz) : nullptr;
    b.lse = m.f(NQ * z.H);
    b.xm = m.f(NQ * z.D);
}

static void plan_work(Work& W, Bump& m, int R, bool train, const Dims& z, int esz,
                      bool bf16mode) {
    W.R = R; W.train = train;
    long NT = (long)R * z.LTOK, NS = (long)R * z.LSEQ, NO = (long)R * z.NOPT,
         NC = (long)R * z.LCRIT;
    W.tokcat = m.take(NT * rup(z.TOK_IN, 8) * esz);
    W.keep = (uint8_t*)m.take(NS);
    W.ext = (int*)m.take((long)R * sizeof(int));
    W.kw = (uint32_t*)m.take((long)R * ATTN_KW_WORDS * sizeof(uint32_t));
    W.ckeep = (uint8_t*)m.take(NC);
    W.g1pre = m.f((long)R * 128); W.g1 = m.f((long)R * 128);
    W.gd = m.f((long)R * 192);
    W.decin = m.f((long)R * 696); W.d1pre = m.f((long)R * 64); W.d1 = m.f((long)R * 64);
    W.bc = m.f((long)R * z.D);
    int nx = train ? z.LAYERS + 1 : 2;
    W.x.assign(nx, nullptr);
    for (int i = 0; i < nx; i++) W.x[i] = m.f(NS * z.D);
    int nb = train ? z.LAYERS : 1;
    W.blk.assign(nb, BlkAct{});
    for (int i = 0; i < nb; i++) plan_blk(W.blk[i], m, R, z.LSEQ, z.LSEQ, z, esz, train, false);
    W.h = m.f(NS * z.D); W.muf = m.f(NS); W.rsf = m.f(NS);
    // option scorer: fp32 operands in both modes (its gradients reduce over
    // options whose inputs share a large per-sample component; bf16 operand
    // rounding would dominate those sums)
    W.qin = m.f(NO * rup(z.Q_IN, 8));
    W.q1pre = train ? m.f(NO * z.D) : nullptr;
    W.q1 = m.f(NO * z.D);
    W.scin = m.f(NO * 2 * z.D);                 // qq = [q | q*r]
    W.u = m.f((long)R * 256);
    W.rgd = m.f((long)R * (z.D + 192));
    W.wqq = m.f(256L * 2 * z.D);
    W.s1pre = train ? m.f(NO * 256) : nullptr;
    W.s1 = m.f(NO * 256);
    W.otokin = m.take((long)R * 56 * 136 * esz);
    // critic block: read at its readout row only -> rows past attention = 1
    W.xc[0] = m.f(NC * z.D); W.xc[1] = m.f((long)R * z.D);
    plan_blk(W.cblk, m, R, z.LCRIT, 1, z, esz, train, false);
    W.ovin = m.f((long)R * z.VAL_IN); W.ov1pre = m.f((long)R * 256); W.ov1 = m.f((long)R * 256);
    W.out = m.f((long)R * (z.NOPT + 1));
    if (!train) return;
    W.bvin = m.f((long)R * z.VAL_IN);
    W.bvinc = bf16mode ? m.take((long)R * z.VAL_IN * esz) : nullptr;
    W.bv1pre = m.f((long)R * 256); W.bv1 = m.f((long)R * 256); W.blind_v = m.f(R);
    W.hand_lin = m.f((long)R * z.NC);
    W.prize_logit = m.f(NT);
    // backward
    W.dh = m.f(NS * z.D);
    W.dgd = m.f((long)R * 192);
    W.dbvin = m.f((long)R * z.VAL_IN);
    W.d_v1pre = m.f((long)R * 256);
    W.dscores = m.f(NO);
    W.dscin = m.f(NO * 2 * z.D);                // d qq
    W.du = m.f((long)R * 256);
    W.drgd = m.f((long)R * (z.D + 192));
    W.dqin = m.f(NO * z.Q_IN);
    W.dtokcat = m.f(NT * z.TOK_IN);
    W.ddecin = m.f((long)R * 696);
    W.dd1 = m.f((long)R * 64);
    W.dg1 = m.f((long)R * 128);
    W.dbc = m.f((long)R * z.D);
    W.dotokin = m.f((long)R * 56 * 136);      // row pitch 136: 16-byte rows for the TMA store
    W.dx = m.f(NC * z.D);
    W.dx0 = m.f((long)R * z.D);
    W.dq0 = m.take((long)R * z.D * esz);
    W.dx0c = bf16mode ? m.take((long)R * z.D * esz) : (void*)W.dx0;
    W.dln = m.f(NC * z.D);
    W.dxc = bf16mode ? m.take(NC * z.D * esz) : (void*)W.dx;
    W.dhand = m.take((long)R * z.NC * esz);
    W.ds1pre = m.f(NO * 256);
    W.dq = m.f(NO * z.D);
    W.dq1 = m.f(NO * z.D);
    W.dotok = m.take((long)R * 56 * z.D * esz);
    W.dtokp = m.take(NT * z.D * esz);
    W.df = m.take(NC * z.FFN * esz);
    W.datt = m.take(NC * z.D * esz);
    W.dqkv = m.take(NC * 3 * z.D * esz);
    W.dgrad = m.f((long)R * (z.NOPT + 1));
    W.fused = m.f((long)R * (z.NOPT + 1));
    W.ppo_scratch = m.f(16 + 7 * ((R + 7) / 8));
    W.nlp = m.f(R); W.ratio = m.f(R);
}

static void plan_tab(Tab& t, Bump& m, const Dims& z) {
    t.att_in = m.f((long)z.NA * 127); t.att_pre = m.f((long)z.NA * 64); t.att_tab = m.f((long)z.NA * 64);
    t.sk_in = m.f((long)z.NS * 112); t.sk_pre = m.f((long)z.NS * 128); t.sk_tab = m.f((long)z.NS * 128);
    t.card_in = m.f((long)z.NC * 634); t.card_ln = m.f((long)z.NC * 634);
    t.ln_mu = m.f(z.NC); t.ln_rs = m.f(z.NC);
    t.h1pre = m.f((long)z.NC * 256); t.h1 = m.f((long)z.NC * 256);
    t.card_vec = m.f((long)z.NC * 128);
    t.poc = m.f((long)z.NC * 64); t.poa = m.f((long)z.NA * 64);
    t.a_arg = (int8_t*)m.take((size_t)z.NC * 64);
    t.s_arg = (int8_t*)m.take((size_t)z.NC * 128);
    t.d_cv = m.f((long)z.NC * 128); t.d_att = m.f((long)z.NA * 64); t.d_sk = m.f((long)z.NS * 128);
    t.d_poc = m.f((long)z.NC * 64); t.d_poa = m.f((long)z.NA * 64);
    t.d_h1 = m.f((long)z.NC * 256); t.d_cardln = m.f((long)z.NC * 634);
    t.d_cardin = m.f((long)z.NC * 634); t.d_attin = m.f((long)z.NA * 127);
    t.d_skin = m.f((long)z.NS * 112);
}

// --------------------------------------------------------------- forward
static void tables_fwd(PtcgModel* M, Tab& t, cudaStream_t s) {
    const Dims& z = M->z;
    Segs g{};
    g.n = 3;
    g.s[0] = {M->w("attack_id_emb").p, 48, 0, 48, 0};
    g.s[1] = {M->att_static, 15, 0, 15, 48};
    g.s[2] = {M->att_text, 64, 0, 64, 63};
    ++g_ptcg_launches, k_concat_rows<<<cdiv((long)z.NA * 127, TPB), TPB, 0, s>>>(t.att_in, 127, z.NA, 127, g);
    GemmArgs a = lin_fwd(DT_F32, z.NA, 127, 64, t.att_in, 127, f32w(M->w("attack_mlp_w"), 127), t.att_tab, 64, DT_F32);
    a.bias = M->w("attack_mlp_b").p; a.act = ACT_GELU; a.out2 = t.att_pre; a.ldo2 = 64;
    gemm32(M, a, s);
    g.n = 2;
    g.s[0] = {M->w("skill_id_emb").p, 48, 0, 48, 0};
    g.s[1] = {M->skill_text, 64, 0, 64, 48};
    ++g_ptcg_launches, k_concat_rows<<<cdiv((long)z.NS * 112, TPB), TPB, 0, s>>>(t.sk_in, 112, z.NS, 112, g);
    a = lin_fwd(DT_F32, z.NS, 112, 128, t.sk_in, 112, f32w(M->w("skill_mlp_w"), 112), t.sk_tab, 128, DT_F32);
    a.bias = M->w("skill_mlp_b").p; a.act = ACT_GELU; a.out2 = t.sk_pre; a.ldo2 = 128;
    gemm32(M, a, s);
    // pools written straight into their card_in columns
    ++g_ptcg_launches, k_pool<<<cdiv((long)z.NC * 64, TPB), TPB, 0, s>>>(t.card_in + 250, t.card_in + 314, 634, t.a_arg,
        t.att_tab, M->card_attacks, z.NC, 4, 64);
    ++g_ptcg_launches, k_pool<<<cdiv((long)z.NC * 128, TPB), TPB, 0, s>>>(t.card_in + 378, t.card_in + 506, 634, t.s_arg,
        t.sk_tab, M->card_skills, z.NC, 2, 128);
    g.n = 3;
    g.s[0] = {M->w("card_id_emb").p, 64, 0, 64, 0};
    g.s[1] = {M->card_static, 58, 0, 58, 64};
    g.s[2] = {M->card_text, 128, 0, 128, 122};
    ++g_ptcg_launches, k_concat_rows<<<cdiv((long)z.NC * 250, TPB), TPB, 0, s>>>(t.card_in, 634, z.NC, 250, g);
    ln_fwd(DT_F32, t.card_ln, 634, t.ln_mu, t.ln_rs, t.card_in, 634, M->w("card_ln_w").p,
           M->w("card_ln_b").p, z.NC, 634, s);
    a = lin_fwd(DT_F32, z.NC, 634, 256, t.card_ln, 634, f32w(M->w("card_mlp1_w"), 634), t.h1, 256, DT_F32);
    a.bias = M->w("card_mlp1_b").p; a.act = ACT_GELU; a.out2 = t.h1pre; a.ldo2 = 256;
    gemm32(M, a, s);
    a = lin_fwd(DT_F32, z.NC, 256, 128, t.h1, 256, f32w(M->w("card_mlp2_w"), 256), t.card_vec, 128, DT_F32);
    a.bias = M->w("card_mlp2_b").p;
    gemm32(M, a, s);
    // option-scorer card / attack projections, per table row
    a = lin_fwd(DT_F32, z.NC, 128, 64, t.card_vec, 128, f32w(M->w("opt_card_w"), 128), t.poc, 64, DT_F32);
    a.bias = M->w("opt_card_b").p;
    gemm32(M, a, s);
    a = lin_fwd(DT_F32, z.NA, 64, 64, t.att_tab, 64, f32w(M->w("opt_attack_w"), 64), t.poa, 64, DT_F32);
    a.bias = M->w("opt_attack_b").p;
    gemm32(M, a, s);
}

// ext (nullable): per sequence, the rows anything reads (k_row_extent)
static void block_fwd(PtcgModel* M, const BlkW& P, BlkAct& b, const uint8_t* keep, int R, int L,
                      bool train, cudaStream_t s, const int* ext = nullptr,
                      const uint32_t* kw = nullptr) {
    const Dims& z = M->z;
    const int dt = M->dt(), D = z.D;
    const int NL = R * L;
    ln_fwd(dt, b.ln1, D, b.mu1, b.rs1, b.x_in, D, P.ln1w.p, P.ln1b.p, NL, D, s, ext, L);
    GemmArgs a = lin_fwd(dt, NL, D, 3 * D, b.ln1, D, P.qkvw, b.qkv, 3 * D, dt);
    a.bias = P.qkvb.p;
    gemm(M, a, s);
    attn_fwd(dt, b.qkv, 3 * D, keep, b.att, D, b.lse, R, L, z.H, s, ext, kw);
    a = lin_fwd(dt, NL, D, D, b.att, D, P.projw, b.xm, D, DT_F32);
    a.bias = P.projb.p; a.resid = b.x_in; a.ld_resid = D;
    gemm(M, a, s);
    ln_fwd(dt, b.ln2, D, b.mu2, b.rs2, b.xm, D, P.ln2w.p, P.ln2b.p, NL, D, s, ext, L);
    // rollout: FFN1 -> GELU -> FFN2 in one kernel, the hidden activation on
    // chip (the backward of a training forward needs it written)
    if (!train && dt == DT_BF16 && g_fused_mlp.load() &&
        mlp_fwd_tc(b.ln2, D, P.f1w.op, P.f1w.ld, P.f1b.p, P.f2w.op, P.f2w.ld, P.f2b.p, b.xm, D,
                   b.x_out, D, NL, D, z.FFN, s))
        return;
    a = lin_fwd(dt, NL, D, z.FFN, b.ln2, D, P.f1w, b.fpost, z.FFN, dt);
    a.bias = P.f1b.p; a.act = ACT_GELU;
    if (train) { a.out2 = b.fpre; a.ldo2 = z.FFN; a.out2_dtype = dt; }
    gemm(M, a, s);
    a = lin_fwd(dt, NL, z.FFN, D, b.fpost, z.FFN, P.f2w, b.x_out, D, DT_F32);
    a.bias = P.f2b.p; a.resid = b.xm; a.ld_resid = D;
    gemm(M, a, s);
}

// The same block evaluated at the first row of each sequence only (its
// output is read there alone): LN1 and QKV over every row (keys / values),
// then single-query attention, proj, LN2 and the FFN on R rows.  x_out and
// the post-attention activations are compact [R, ...].
// h (nullable): the trunk output; when given, the critic's trunk rows are
// read from it (crit_rows_direct(D)) and b.x_in holds rows 0 and LSEQ+1..
static void block_fwd_row0(PtcgModel* M, const BlkW& P, BlkAct& b, const uint8_t* keep, int R,
                           int L, bool train, cudaStream_t s, const float* h = nullptr) {
    const Dims& z = M->z;
    const int dt = M->dt(), D = z.D;
    const int NL = R * L;
    // rows other than the query row and the kept keys are read by nothing
    ln_fwd(dt, b.ln1, D, b.mu1, b.rs1, b.x_in, D, P.ln1w.p, P.ln1b.p, NL, D, s, nullptr, 1, keep,
           h, z.LSEQ, L);
    // keys and values of every row (weight rows D..3D), queries of the
    // readout rows only (weight rows 0..D; A rows at stride L * D)
    GemmArgs a = lin_fwd(dt, NL, D, 2 * D, b.ln1, D, wrows(P.qkvw, D, D, M->esz()), b.qkv, 2 * D, dt);
    a.bias = P.qkvb.p + D;
    gemm(M, a, s);
    a = lin_fwd(dt, R, D, D, b.ln1, (long)L * D, P.qkvw, b.q0, D, dt);
    a.bias = P.qkvb.p;
    gemm(M, a, s);
    attn_row0_fwd(dt, b.q0, D, b.qkv, 2 * D, keep, b.att, D, b.lse, R, L, z.H, s);
    a = lin_fwd(dt, R, D, D, b.att, D, P.projw, b.xm, D, DT_F32);
    a.bias = P.projb.p; a.resid = b.x_in; a.ld_resid = (long)L * D;
    gemm(M, a, s);
    ln_fwd(dt, b.ln2, D, b.mu2, b.rs2, b.xm, D, P.ln2w.p, P.ln2b.p, R, D, s);
    a = lin_fwd(dt, R, D, z.FFN, b.ln2, D, P.f1w, b.fpost, z.FFN, dt);
    a.bias = P.f1b.p; a.act = ACT_GELU;
    if (train) { a.out2 = b.fpre; a.ldo2 = z.FFN; a.out2_dtype = dt; }
    gemm(M, a, s);
    a = lin_fwd(dt, R, z.FFN, D, b.fpost, z.FFN, P.f2w, b.x_out, D, DT_F32);
    a.bias = P.f2b.p; a.resid = b.xm; a.ld_resid = D;
    gemm(M, a, s);
}

// out[c] += column sums over a set of rows (see k_colsum_rowset); the
// vector kernel when the columns are 128 or 256 wide and rows 16-byte aligned
static void colsum_rows(PtcgModel* M, float* out, const float* src, long ld, int ngroups,
                        int group_stride, int row_off, int rows_per_group, int cols,
                        cudaStream_t s) {
    const long nrows = (long)ngroups * rows_per_group;
    if ((cols == 128 || cols == 256) && ld % 4 == 0 && !((uintptr_t)src & 15)) {
        unsigned g = std::min<unsigned>(cdiv(nrows, 8), M->adam_grid);
        if (cols == 128)
            ++g_ptcg_launches, k_colsum_rowset<1><<<g, 256, 0, s>>>(out, src, ld, ngroups, group_stride,
                                                                    row_off, rows_per_group);
        else
            ++g_ptcg_launches, k_colsum_rowset<2><<<g, 256, 0, s>>>(out, src, ld, ngroups, group_stride,
                                                                    row_off, rows_per_group);
        return;
    }
    int gpb = 64;
    dim3 g(cdiv(cols, 128), cdiv(ngroups, gpb));
    ++g_ptcg_launches, k_colsum_groups<<<g, 128, 0, s>>>(out, src, ld, ngroups, group_stride, row_off,
                                                         rows_per_group, cols, gpb);
}

// rows-dot launcher
template <typename TI>
static void rowdot(float* out, long os, const TI* in, long ldi, const float* w, const float* b,
                   int rows, int K, int g, int gs, int go, cudaStream_t s) {
    ++g_ptcg_launches, k_rowdot<TI><<<cdiv(rows, 8), 256, 0, s>>>(out, os, in, ldi, w, b, rows, K, g, gs, go);
}

// the sampler fused into the rollout forward's output step (k_out_sample)
struct SampleArgs {
    const float* mask; long mstride; const float* uni;
    float *actions, *logprobs, *values;
};

static int forward_impl(PtcgModel* M, Work& Wk, Tab& t, const float* obs, int R, float* out,
                        bool train, bool do_tables, cudaStream_t s,
                        const SampleArgs* smp = nullptr) {
    const Dims& z = M->z;
    const int dt = M->dt(), D = z.D, esz = M->esz();
    const ObsLayout& ol = z.ol;
    const int tf32 = M->prec == PTCG_BF16;   // fp32-operand GEMMs may use TF32 in bf16 mode
    if (do_tables) tables_fwd(M, t, s);
    // --- token path
    long ldtok = rup(z.TOK_IN, 8);
    ++g_ptcg_launches, k_x0_readout<<<cdiv((long)R * (z.LSEQ > D ? z.LSEQ : D), TPB), TPB, 0, s>>>(Wk.x[0], Wk.keep,
        M->w("readout").p, obs, ol, R, D);
    ++g_ptcg_launches, k_row_extent<<<cdiv(R, TPB / 32), TPB, 0, s>>>(Wk.ext, Wk.keep, obs, ol, R, Wk.kw);
    if (dt == DT_F32)
        ++g_ptcg_launches, k_tok_cat<float><<<cdiv((long)R * z.LTOK, TPB / 32), TPB, 0, s>>>((float*)Wk.tokcat, ldtok, obs, ol, t.card_vec,
            M->w("zone_emb").p, M->w("owner_emb").p, R, z.TOK_IN, Wk.ext);
    else
        ++g_ptcg_launches, k_tok_cat<bf16><<<cdiv((long)R * z.LTOK, TPB / 32), TPB, 0, s>>>((bf16*)Wk.tokcat, ldtok, obs, ol, t.card_vec,
            M->w("zone_emb").p, M->w("owner_emb").p, R, z.TOK_IN, Wk.ext);
    // --- global / decision encoders (fp32)
    GemmArgs a = lin_fwd(DT_F32, R, 64, 128, obs + ol.glob, ol.obs, f32w(M->w("global1_w"), 64),
                         Wk.g1, 128, DT_F32);
    a.bias = M->w("global1_b").p; a.act = ACT_GELU; a.out2 = Wk.g1pre; a.ldo2 = 128;
    gemm32(M, a, s);
    a = lin_fwd(DT_F32, R, 128, 128, Wk.g1, 128, f32w(M->w("global2_w"), 128), Wk.gd, 192, DT_F32);
    a.bias = M->w("global2_b").p;
    gemm32(M, a, s);
    ++g_ptcg_launches, k_dec_in<<<cdiv((long)R * 696, TPB), TPB, 0, s>>>(Wk.decin, obs, ol, t.card_vec, t.att_tab,
        M->w("sel_type_emb").p, M->w("ctx_emb").p, R);
    a = lin_fwd(DT_F32, R, 696, 64, Wk.decin, 696, f32w(M->w("dec1_w"), 696), Wk.d1, 64, DT_F32);
    a.bias = M->w("dec1_b").p; a.act = ACT_GELU; a.out2 = Wk.d1pre; a.ldo2 = 64;
    gemm32(M, a, s);
    a = lin_fwd(DT_F32, R, 64, 64, Wk.d1, 64, f32w(M->w("dec2_w"), 64), Wk.gd + 128, 192, DT_F32);
    a.bias = M->w("dec2_b").p;
    gemm32(M, a, s);
    a = lin_fwd(DT_F32, R, 192, D, Wk.gd, 192, f32w(M->w("bcast_w"), 192), Wk.bc, D, DT_F32);
    a.bias = M->w("bcast_b").p;
    gemm32(M, a, s);
    // token_proj + broadcast, written into trunk rows 1..LTOK
    a = lin_fwd(dt, R * z.LTOK, z.TOK_IN, D, Wk.tokcat, ldtok, M->w("token_proj_w"), Wk.x[0], D, DT_F32);
    a.bias = M->w("token_proj_b").p;
    a.bcast = Wk.bc; a.ld_bcast = D; a.bcast_group = z.LTOK;
    a.remap_group = z.LTOK; a.remap_stride = z.LSEQ; a.remap_off = 1;
    gemm(M, a, s);
    // --- trunk
    const float* xl = Wk.x[0];
    for (int i = 0; i < z.LAYERS; i++) {
        BlkAct& b = train ? Wk.blk[i] : Wk.blk[0];
        b.x_in = train ? Wk.x[i] : Wk.x[i % 2];
        b.x_out = train ? Wk.x[i + 1] : Wk.x[(i + 1) % 2];
        block_fwd(M, M->blk("b" + std::to_string(i) + "_"), b, Wk.keep, R, z.LSEQ, train, s, Wk.ext,
                  Wk.kw);
        xl = b.x_out;
    }
    ln_fwd(DT_F32, Wk.h, D, Wk.muf, Wk.rsf, xl, D, M->w("lnf_w").p, M->w("lnf_b").p, R * z.LSEQ, D, s,
           Wk.ext, z.LSEQ);
    // --- option scorer
    long NO = (long)R * z.NOPT;
    long ldq = rup(z.Q_IN, 8);
    ++g_ptcg_launches, k_q_in<<<cdiv(NO, TPB / 32), TPB, 0, s>>>((float*)Wk.qin, ldq, obs, ol, Wk.h, D,
        M->w("opt_type_emb").p, t.poc, t.poa, R, z.Q_IN);
    a = lin_fwd(DT_F32, (int)NO, z.Q_IN, D, Wk.qin, ldq, f32w(M->w("q1_w"), z.Q_IN), Wk.q1, D, DT_F32);
    a.bias = M->w("q1_b").p; a.act = ACT_GELU; a.allow_tf32 = tf32;
    if (train) { a.out2 = Wk.q1pre; a.ldo2 = D; }
    gemm(M, a, s);
    // score1(cat[q, r, g, d, q*r]) (model.py:270-273) evaluated as
    //   [q | q*r] Wqq^T + bcast_n([r | g | d] Wrgd^T + b):
    // the per-sample columns r, g, d go through one GEMM per sample instead
    // of NOPT copies per sample
    float* qq = (float*)Wk.scin;
    a = lin_fwd(DT_F32, (int)NO, D, D, Wk.q1, D, f32w(M->w("q2_w"), D), qq, 2 * D, DT_F32);
    a.bias = M->w("q2_b").p; a.allow_tf32 = tf32;
    gemm(M, a, s);
    ++g_ptcg_launches, k_qr_fill<<<cdiv(NO, TPB / 32), TPB, 0, s>>>(qq, D, Wk.h, z.LSEQ, z.NOPT, NO);
    ++g_ptcg_launches, k_rgd_fill<<<cdiv((long)R * (D + 192), TPB), TPB, 0, s>>>(Wk.rgd, Wk.h, z.LSEQ, Wk.gd,
        D, R);
    W ws1 = f32w(M->w("score1_w"), z.SCORE_IN);
    W wrgd = ws1; wrgd.op = ws1.p + D;           // columns [D, 2D + 192)
    a = lin_fwd(DT_F32, R, D + 192, 256, Wk.rgd, D + 192, wrgd, Wk.u, 256, DT_F32);
    a.bias = M->w("score1_b").p; a.allow_tf32 = tf32;
    gemm(M, a, s);
    ++g_ptcg_launches, k_pack_wqq<<<cdiv(256L * 2 * D, TPB), TPB, 0, s>>>(Wk.wqq, ws1.p, D, z.SCORE_IN, 256);
    W wqq = ws1; wqq.op = Wk.wqq; wqq.ld = 2 * D;
    a = lin_fwd(DT_F32, (int)NO, 2 * D, 256, qq, 2 * D, wqq, Wk.s1, 256, DT_F32);
    a.bcast = Wk.u; a.ld_bcast = 256; a.bcast_group = z.NOPT;
    a.act = ACT_GELU; a.allow_tf32 = tf32;
    if (train) { a.out2 = Wk.s1pre; a.ldo2 = 256; }
    gemm(M, a, s);
    // score2 -> out[n, j]  (out row stride NOPT+1): rows r = n*NOPT + j map to
    // n*(NOPT+1) + j, i.e. group NOPT of output stride NOPT+1
    {
        int rows = (int)NO;
        unsigned g = cdiv(rows, 8);
        ++g_ptcg_launches, k_rowdot<float><<<g, 256, 0, s>>>(Wk.out, 1, (const float*)Wk.s1, 256,
            M->w("score2_w").p, M->w("score2_b").p, rows, 256, 0, 0, 0);
    }
    // (scores are staged contiguous (R*NOPT) at the head of Wk.out and
    //  expanded to the fused layout at the end)
    // --- oracle critic top
    long ldo_t = rup(134, 8);
    long no = (long)R * 56;                     // oracle tokens, one warp each
    if (dt == DT_F32)
        ++g_ptcg_launches, k_otok_in<float><<<cdiv(no, TPB / 32), TPB, 0, s>>>((float*)Wk.otokin, ldo_t, Wk.ckeep, obs, ol,
            t.card_vec, Wk.keep, R);
    else
        ++g_ptcg_launches, k_otok_in<bf16><<<cdiv(no, TPB / 32), TPB, 0, s>>>((bf16*)Wk.otokin, ldo_t, Wk.ckeep, obs, ol,
            t.card_vec, Wk.keep, R);
    // critic rows 0 and 1..LSEQ; with crit_rows_direct(D) the trunk rows are
    // read from h by the critic's LN1 and only row 0 is written
    const bool crit_direct = crit_rows_direct(D);
    const int xc_rows = crit_direct ? 0 : z.LSEQ;
    ++g_ptcg_launches, k_xc_fill<<<cdiv((long)R * (1 + xc_rows), TPB / 32), TPB, 0, s>>>(Wk.xc[0], Wk.h,
        M->w("critic_readout").p, xc_rows, z.LCRIT, D, R, Wk.ext);
    a = lin_fwd(dt, R * 56, 134, D, Wk.otokin, ldo_t, M->w("oracle_proj_w"), Wk.xc[0], D, DT_F32);
    a.bias = M->w("oracle_proj_b").p;
    a.remap_group = 56; a.remap_stride = z.LCRIT; a.remap_off = 1 + z.LSEQ;
    gemm(M, a, s);
    Wk.cblk.x_in = Wk.xc[0]; Wk.cblk.x_out = Wk.xc[1];
    block_fwd_row0(M, M->blk("c0_"), Wk.cblk, Wk.ckeep, R, z.LCRIT, train, s,
                   crit_direct ? Wk.h : nullptr);
    ++g_ptcg_launches, k_val_in<float><<<cdiv((long)R * z.VAL_IN, TPB), TPB, 0, s>>>(Wk.ovin, nullptr, 0, Wk.xc[1],
        1, D, Wk.gd, R);
    a = lin_fwd(DT_F32, R, z.VAL_IN, 256, Wk.ovin, z.VAL_IN, f32w(M->w("oracle_v1_w"), z.VAL_IN),
                Wk.ov1, 256, DT_F32);
    a.bias = M->w("oracle_v1_b").p; a.act = ACT_GELU; a.out2 = Wk.ov1pre; a.ldo2 = 256;
    gemm32(M, a, s);
    // fused output [scores | value]: expand staged scores, then the value
    // column -- with the sampler in the same kernel when one is requested
    if (smp) {
        ++g_ptcg_launches, k_out_sample<<<cdiv(R, TPB / 32), TPB, 0, s>>>(out, Wk.out, z.NOPT, Wk.ov1,
            M->w("oracle_v2_w").p, M->w("oracle_v2_b").p, 256,
            smp->mask ? smp->mask : obs + ol.mask, smp->mask ? smp->mstride : ol.obs, smp->uni,
            smp->actions, smp->logprobs, smp->values, R);
        return 0;
    }
    ++g_ptcg_launches, k_scale_copy<<<cdiv(NO, TPB), TPB, 0, s>>>(out, z.NOPT + 1, Wk.out, z.NOPT, R, z.NOPT, 1.f);
    rowdot<float>(out + z.NOPT, z.NOPT + 1, Wk.ov1, 256, M->w("oracle_v2_w").p,
                  M->w("oracle_v2_b").p, R, 256, 0, 0, 0, s);
    if (!train) return 0;
    // --- train-only heads: blind V, opp-hand counts, prize logits
    if (dt == DT_F32)
        ++g_ptcg_launches, k_val_in<float><<<cdiv((long)R * z.VAL_IN, TPB), TPB, 0, s>>>(Wk.bvin, nullptr, 0, Wk.h,
            z.LSEQ, D, Wk.gd, R);
    else
        ++g_ptcg_launches, k_val_in<bf16><<<cdiv((long)R * z.VAL_IN, TPB), TPB, 0, s>>>(Wk.bvin, (bf16*)Wk.bvinc,
            z.VAL_IN, Wk.h, z.LSEQ, D, Wk.gd, R);
    a = lin_fwd(DT_F32, R, z.VAL_IN, 256, Wk.bvin, z.VAL_IN, f32w(M->w("value1_w"), z.VAL_IN),
                Wk.bv1, 256, DT_F32);
    a.bias = M->w("value1_b").p; a.act = ACT_GELU; a.out2 = Wk.bv1pre; a.ldo2 = 256;
    gemm32(M, a, s);
    rowdot<float>(Wk.blind_v, 1, Wk.bv1, 256, M->w("value2_w").p, M->w("value2_b").p, R, 256,
                  0, 0, 0, s);
    a = lin_fwd(dt, R, z.VAL_IN, z.NC, dt == DT_F32 ? (const void*)Wk.bvin : Wk.bvinc, z.VAL_IN,
                M->w("aux_hand_w"), Wk.hand_lin, z.NC, DT_F32);
    a.bias = M->w("aux_hand_b").p;
    gemm(M, a, s);
    rowdot<float>(Wk.prize_logit, 1, Wk.h, D, M->w("aux_prize_w").p, M->w("aux_prize_b").p,
                  R * z.LTOK, D, z.LTOK, z.LSEQ, 1, s);
    (void)esz;
    return 0;
}

// --------------------------------------------------------------- backward
// A span of the grad arena is final: with the native data-parallel exchange
// on, start its reduce-scatter; else hand it to the caller's hook.
static void fire_hook(PtcgModel* M, const char* first, const char* last_excl, cudaStream_t s) {
    if (!M->hook && !M->dp) return;
    long a = M->off[M->idx[first]];
    long b = last_excl ? M->off[M->idx[last_excl]] : M->n_arena;
    if (b <= a) return;
    if (M->dp) {
        if (dp_bucket(M->dp, M->grads, a, b - a, s)) {
            set_err("data-parallel reduce-scatter: %s", dp_last_error());
            M->dp_fail = true;
        }
    } else {
        M->hook(M->hook_user, a, b - a, (void*)s);
    }
}

// The spans fire_hook reports in one step, in firing order: ln_f and the
// heads after it, each block from the last to the first, the encoders, then
// the tables ({offset, count} pairs).
static std::vector<long> hook_spans(const PtcgModel* M) {
    auto o = [&](const std::string& n) { return M->off[M->idx.at(n)]; };
    std::vector<long> v;
    auto add = [&](long a, long b) { if (b > a) { v.push_back(a); v.push_back(b - a); } };
    const int L = M->z.LAYERS;
    add(o("lnf_w"), M->n_arena);
    for (int i = L - 1; i >= 0; i--)
        add(o("b" + std::to_string(i) + "_ln1_w"),
            i == L - 1 ? o("lnf_w") : o("b" + std::to_string(i + 1) + "_ln1_w"));
    add(o("zone_emb"), o("b0_ln1_w"));
    add(o("card_id_emb"), o("zone_emb"));
    return v;
}

// On entry dx holds d(x_out) and the FFN2 bias grad of this block is
// already accumulated (by the LayerNorm backward that produced dx); the LN1
// backward at the end adds the column sums of d(x_in) to lower_f2b, the
// FFN2 bias grad of the block below (nullptr for the first block).
static void block_bwd(PtcgModel* M, const BlkW& P, BlkAct& b, const uint8_t* keep, Work& Wk,
                      int R, int L, float* lower_f2b, cudaStream_t s) {
    const Dims& z = M->z;
    const int dt = M->dt(), D = z.D, F = z.FFN;
    const int NL = R * L;
    const bool bf = dt == DT_BF16;
    float* dx = Wk.dx;                 // f32, holds d(x_out) on entry
    void* dxc = Wk.dxc;                // operand-dtype copy of dx
    // FFN2
    gemm(M, lin_dw(dt, NL, F, D, dxc, D, b.fpost, F, P.f2w.g), s);
    GemmArgs a = lin_dx(dt, NL, F, D, dxc, D, P.f2w, Wk.df, F, dt);
    a.act = ACT_GELU_BWD; a.aux = b.fpre; a.ld_aux = F; a.aux_dtype = dt;
    a.colsum = P.f1b.g;                 // FFN1 bias grad, fp32 before rounding
    gemm(M, a, s);
    // FFN1
    gemm(M, lin_dw(dt, NL, D, F, Wk.df, F, b.ln2, D, P.f1w.g), s);
    // d(LN2 output) in the operand dtype (bf16 mode: half the bytes of the
    // GEMM's output and of the LayerNorm backward's input)
    gemm(M, lin_dx(dt, NL, D, F, Wk.df, F, P.f1w, Wk.dln, D, dt), s);
    // LN2: dx <- d(x_mid) = dx + LN2'(dln)
    // (+ proj bias grad = column sums of d(x_mid))
    ln_bwd(dt, dx, 1, bf ? dxc : nullptr, P.ln2w.g, P.ln2b.g, Wk.dln, b.xm, P.ln2w.p, b.mu2,
           b.rs2, NL, D, s, P.projb.g, dt, Wk.ext, L);
    // proj
    gemm(M, lin_dw(dt, NL, D, D, dxc, D, b.att, D, P.projw.g), s);
    gemm(M, lin_dx(dt, NL, D, D, dxc, D, P.projw, Wk.datt, D, dt), s);
    // attention
    attn_bwd(dt, b.qkv, 3 * D, keep, b.att, D, Wk.datt, D, b.lse, Wk.dqkv, 3 * D, P.qkvb.g,
             R, L, z.H, s, Wk.ext, Wk.kw);
    // QKV
    gemm(M, lin_dw(dt, NL, D, 3 * D, Wk.dqkv, 3 * D, b.ln1, D, P.qkvw.g), s);
    gemm(M, lin_dx(dt, NL, D, 3 * D, Wk.dqkv, 3 * D, P.qkvw, Wk.dln, D, dt), s);
    // LN1: dx <- d(x_in) = dx + LN1'(dln)
    ln_bwd(dt, dx, 1, bf ? dxc : nullptr, P.ln1w.g, P.ln1b.g, Wk.dln, b.x_in, P.ln1w.p, b.mu1,
           b.rs1, NL, D, s, lower_f2b, dt, Wk.ext, L);
}

// Backward of block_fwd_row0.  On entry Wk.dx0 (f32) / Wk.dx0c (operand
// dtype) hold d(x_out) [R, D]; on exit Wk.dx [R * L, D] holds d(x_in).
static void block_bwd_row0(PtcgModel* M, const BlkW& P, BlkAct& b, const uint8_t* keep, Work& Wk,
                           int R, int L, cudaStream_t s) {
    const Dims& z = M->z;
    const int dt = M->dt(), D = z.D, F = z.FFN;
    const int NL = R * L;
    const bool bf = dt == DT_BF16;
    float* dx0 = Wk.dx0;
    void* dx0c = Wk.dx0c;
    // FFN2
    colsum<float>(P.f2b.g, dx0, D, R, D, s);
    gemm(M, lin_dw(dt, R, F, D, dx0c, D, b.fpost, F, P.f2w.g), s);
    GemmArgs a = lin_dx(dt, R, F, D, dx0c, D, P.f2w, Wk.df, F, dt);
    a.act = ACT_GELU_BWD; a.aux = b.fpre; a.ld_aux = F; a.aux_dtype = dt;
    a.colsum = P.f1b.g;
    gemm(M, a, s);
    // FFN1
    gemm(M, lin_dw(dt, R, D, F, Wk.df, F, b.ln2, D, P.f1w.g), s);
    gemm(M, lin_dx(dt, R, D, F, Wk.df, F, P.f1w, Wk.dln, D, DT_F32), s);
    ln_bwd(dt, dx0, 1, bf ? dx0c : nullptr, P.ln2w.g, P.ln2b.g, Wk.dln, b.xm, P.ln2w.p, b.mu2,
           b.rs2, R, D, s, P.projb.g);
    // proj
    gemm(M, lin_dw(dt, R, D, D, dx0c, D, b.att, D, P.projw.g), s);
    gemm(M, lin_dx(dt, R, D, D, dx0c, D, P.projw, Wk.datt, D, dt), s);
    // attention: dQ of the readout rows, dK / dV at every key
    attn_row0_bwd(dt, b.q0, D, b.qkv, 2 * D, keep, b.att, D, Wk.datt, D, b.lse, Wk.dq0, D,
                  Wk.dqkv, 2 * D, P.qkvb.g, R, L, z.H, s);
    // QKV weight grads: query rows from the readout rows, key / value rows
    // from every row
    W wkv = wrows(P.qkvw, D, D, M->esz());
    gemm(M, lin_dw(dt, R, D, D, Wk.dq0, D, b.ln1, (long)L * D, P.qkvw.g), s);
    gemm(M, lin_dw(dt, NL, D, 2 * D, Wk.dqkv, 2 * D, b.ln1, D, wkv.g), s);
    // d(LN1 out) = dKV Wkv at every row, + dQ Wq at the readout rows
    gemm(M, lin_dx(dt, NL, D, 2 * D, Wk.dqkv, 2 * D, wkv, Wk.dln, D, dt), s);
    {
        GemmArgs a = lin_dx(dt, R, D, D, Wk.dq0, D, P.qkvw, Wk.dln, (long)L * D, dt);
        a.accumulate = 1;
        gemm(M, a, s);
    }
    // d(x_in) = LN1'(dln) + the residual grad at row 0.  With the vector
    // kernel the trunk rows 1..LSEQ go straight to d_h (its first writer)
    // and the oracle-token rows also to d_otok, the oracle_proj GEMMs'
    // operand; otherwise k_xc_bwd splits Wk.dx afterwards
    const bool direct = crit_rows_direct(D);
    ln_bwd(dt, Wk.dx, 0, direct ? Wk.dotok : nullptr, P.ln1w.g, P.ln1b.g, Wk.dln, b.x_in, P.ln1w.p,
           b.mu1, b.rs1, NL, D, s, nullptr, dt, nullptr, 1, keep, direct ? Wk.dh : nullptr,
           M->z.LSEQ, L, direct ? Wk.h : nullptr);
    ++g_ptcg_launches, k_add_rows<<<cdiv((long)R * D, TPB), TPB, 0, s>>>(Wk.dx, (long)L * D, dx0, R, D);
}

static void tables_bwd(PtcgModel* M, cudaStream_t s) {
    const Dims& z = M->z;
    Tab& t = M->tab;
    // card_mlp2
    colsum<float>(M->w("card_mlp2_b").g, t.d_cv, 128, z.NC, 128, s);
    gemm32(M, lin_dw(DT_F32, z.NC, 256, 128, t.d_cv, 128, t.h1, 256, M->w("card_mlp2_w").g), s);
    GemmArgs a = lin_dx(DT_F32, z.NC, 256, 128, t.d_cv, 128, f32w(M->w("card_mlp2_w"), 256),
                        t.d_h1, 256, DT_F32);
    a.act = ACT_GELU_BWD; a.aux = t.h1pre; a.ld_aux = 256; a.aux_dtype = DT_F32;
    gemm32(M, a, s);
    // card_mlp1
    colsum<float>(M->w("card_mlp1_b").g, t.d_h1, 256, z.NC, 256, s);
    gemm32(M, lin_dw(DT_F32, z.NC, 634, 256, t.d_h1, 256, t.card_ln, 634, M->w("card_mlp1_w").g), s);
    gemm32(M, lin_dx(DT_F32, z.NC, 634, 256, t.d_h1, 256, f32w(M->w("card_mlp1_w"), 634),
                     t.d_cardln, 634, DT_F32), s);
    // card LayerNorm (input card_in, ld 634) -> d_cardin
    {
        int rpb = 64;
        ++g_ptcg_launches, k_ln_bwd<float, 0, 20><<<cdiv(z.NC, rpb), 256, 3 * 634 * sizeof(float), s>>>(t.d_cardin, 634, 0,
            nullptr, 634, M->w("card_ln_w").g, M->w("card_ln_b").g, t.d_cardln, 634, t.card_in, 634,
            M->w("card_ln_w").p, t.ln_mu, t.ln_rs, z.NC, 634, rpb, nullptr);
    }
    ++g_ptcg_launches, k_slice_add<<<cdiv((long)z.NC * 64, TPB), TPB, 0, s>>>(M->w("card_id_emb").g, t.d_cardin,
        z.NC, 64, 634, 0);
    ++g_ptcg_launches, k_pool_bwd<<<cdiv((long)z.NC * 64, TPB), TPB, 0, s>>>(t.d_att, t.d_cardin, 634, 250, 314,
        t.a_arg, M->card_attacks, z.NC, 4, 64);
    ++g_ptcg_launches, k_pool_bwd<<<cdiv((long)z.NC * 128, TPB), TPB, 0, s>>>(t.d_sk, t.d_cardin, 634, 378, 506,
        t.s_arg, M->card_skills, z.NC, 2, 128);
    // attack mlp
    ++g_ptcg_launches, k_gelu_bwd<<<cdiv((long)z.NA * 64, TPB), TPB, 0, s>>>(t.d_att, t.att_pre, (long)z.NA * 64);
    colsum<float>(M->w("attack_mlp_b").g, t.d_att, 64, z.NA, 64, s);
    gemm32(M, lin_dw(DT_F32, z.NA, 127, 64, t.d_att, 64, t.att_in, 127, M->w("attack_mlp_w").g), s);
    gemm32(M, lin_dx(DT_F32, z.NA, 127, 64, t.d_att, 64, f32w(M->w("attack_mlp_w"), 127),
                     t.d_attin, 127, DT_F32), s);
    ++g_ptcg_launches, k_slice_add<<<cdiv((long)z.NA * 48, TPB), TPB, 0, s>>>(M->w("attack_id_emb").g, t.d_attin,
        z.NA, 48, 127, 0);
    // skill mlp
    ++g_ptcg_launches, k_gelu_bwd<<<cdiv((long)z.NS * 128, TPB), TPB, 0, s>>>(t.d_sk, t.sk_pre, (long)z.NS * 128);
    colsum<float>(M->w("skill_mlp_b").g, t.d_sk, 128, z.NS, 128, s);
    gemm32(M, lin_dw(DT_F32, z.NS, 112, 128, t.d_sk, 128, t.sk_in, 112, M->w("skill_mlp_w").g), s);
    gemm32(M, lin_dx(DT_F32, z.NS, 112, 128, t.d_sk, 128, f32w(M->w("skill_mlp_w"), 112),
                     t.d_skin, 112, DT_F32), s);
    ++g_ptcg_launches, k_slice_add<<<cdiv((long)z.NS * 48, TPB), TPB, 0, s>>>(M->w("skill_id_emb").g, t.d_skin,
        z.NS, 48, 112, 0);
}

static void zero_table_grads(PtcgModel* M, cudaStream_t s) {
    const Dims& z = M->z;
    Tab& t = M->tab;
    cudaMemsetAsync(t.d_cv, 0, (size_t)z.NC * 128 * 4, s);
    cudaMemsetAsync(t.d_att, 0, (size_t)z.NA * 64 * 4, s);
    cudaMemsetAsync(t.d_sk, 0, (size_t)z.NS * 128 * 4, s);
}

// aux_norm_rows: rows of the whole minibatch; prize_cnt_dev: device count of
// MY_UNSEEN tokens in the whole minibatch (or nullptr + prize_cnt_host)
static int backward_impl(PtcgModel* M, Work& Wk, const float* obs, const float* grad,
                         const float* returns, int R, int norm_rows, const float* prize_cnt_dev,
                         float prize_cnt_host, float* aux_loss, bool last, cudaStream_t s) {
    const Dims& z = M->z;
    const int dt = M->dt(), D = z.D;
    const bool bf = dt == DT_BF16;
    const int tf32 = bf;
    const ObsLayout& ol = z.ol;
    Tab& t = M->tab;
    long NS = (long)R * z.LSEQ, NO = (long)R * z.NOPT;
    cudaMemsetAsync(Wk.dgd, 0, (size_t)R * 192 * 4, s);
    cudaMemsetAsync(t.d_poc, 0, (size_t)z.NC * 64 * 4, s);
    cudaMemsetAsync(t.d_poa, 0, (size_t)z.NA * 64 * 4, s);
    // The oracle value head and the critic block go first: the critic input
    // grad is the first writer of d_h (every row stored), so d_h needs no
    // zeroing; the heads after it add into d_h
    // ---- oracle value head (PPO value grad = grad[:, NOPT])
    {
        int rpb = 64;
        ++g_ptcg_launches, k_rowdot_bwd<float, float><<<cdiv(R, rpb), 256, (256 + 1) * sizeof(float), s>>>(
            Wk.d_v1pre, 256, Wk.ov1pre, 256, Wk.ov1, 256, M->w("oracle_v2_w").p,
            M->w("oracle_v2_w").g, M->w("oracle_v2_b").g, grad + z.NOPT, z.NOPT + 1, nullptr, 0.f,
            R, 256, rpb, nullptr, M->w("oracle_v1_b").g);
    }
    gemm32(M, lin_dw(DT_F32, R, z.VAL_IN, 256, Wk.d_v1pre, 256, Wk.ovin, z.VAL_IN,
                     M->w("oracle_v1_w").g), s);
    gemm32(M, lin_dx(DT_F32, R, z.VAL_IN, 256, Wk.d_v1pre, 256, f32w(M->w("oracle_v1_w"), z.VAL_IN),
                     Wk.dbvin, z.VAL_IN, DT_F32), s);
    ++g_ptcg_launches, k_val_in_bwd<<<cdiv((long)R * z.VAL_IN, TPB), TPB, 0, s>>>(Wk.dx0, 1, D, Wk.dgd, Wk.dbvin, R, 0);
    if (bf) ++g_ptcg_launches, k_cast<bf16><<<cdiv((long)R * D, TPB), TPB, 0, s>>>((bf16*)Wk.dx0c, D, Wk.dx0, D, R, D);
    // ---- critic block (evaluated at its readout row)
    block_bwd_row0(M, M->blk("c0_"), Wk.cblk, Wk.ckeep, Wk, R, z.LCRIT, s);
    {   // critic input grad: row 0 -> critic_readout (column sum over samples),
        // rows 1..LSEQ -> d_h (stored), rows 1+LSEQ.. -> d_otok (compact)
        colsum_rows(M, M->w("critic_readout").g, Wk.dx, D, R, z.LCRIT, 0, 1, D, s);
        unsigned gb = cdiv((long)R * (z.LCRIT - 1), TPB / 32);
        if (crit_rows_direct(D)) {}                 // done by the critic LN1 backward
        else if (bf)
            ++g_ptcg_launches, k_xc_bwd<bf16><<<gb, TPB, 0, s>>>((bf16*)Wk.dotok, Wk.dh, Wk.dx, z.LSEQ, z.LCRIT, D, R, Wk.ext);
        else
            ++g_ptcg_launches, k_xc_bwd<float><<<gb, TPB, 0, s>>>((float*)Wk.dotok, Wk.dh, Wk.dx, z.LSEQ, z.LCRIT, D, R, Wk.ext);
    }
    // ---- aux: opponent-hand counts
    float hscale = 0.1f / ((float)norm_rows * (float)z.NC);
    if (bf)
        ++g_ptcg_launches, k_hand_grad<bf16><<<R, 256, z.NC * sizeof(float), s>>>((bf16*)Wk.dhand, z.NC, Wk.hand_lin,
            z.NC, obs, ol, hscale, aux_loss + 1);
    else
        ++g_ptcg_launches, k_hand_grad<float><<<R, 256, z.NC * sizeof(float), s>>>((float*)Wk.dhand, z.NC, Wk.hand_lin,
            z.NC, obs, ol, hscale, aux_loss + 1);
    W wh = M->w("aux_hand_w");
    colsum<float>(M->w("aux_hand_b").g, Wk.hand_lin, z.NC, R, z.NC, s);   // fp32 grad copy
    gemm(M, lin_dw(dt, R, z.VAL_IN, z.NC, Wk.dhand, z.NC, bf ? Wk.bvinc : (void*)Wk.bvin,
                   z.VAL_IN, wh.g), s);
    gemm(M, lin_dx(dt, R, z.VAL_IN, z.NC, Wk.dhand, z.NC, wh, Wk.dbvin, z.VAL_IN, DT_F32), s);
    // ---- aux: blind V (0.5 * mean (v - R)^2)
    {
        int rpb = 64;
        ++g_ptcg_launches, k_rowdot_bwd<float, float><<<cdiv(R, rpb), 256, (256 + 1) * sizeof(float), s>>>(
            Wk.d_v1pre, 256, Wk.bv1pre, 256, Wk.bv1, 256, M->w("value2_w").p, M->w("value2_w").g,
            M->w("value2_b").g, Wk.blind_v, 1, returns, 1.0f / (float)norm_rows, R, 256, rpb,
            aux_loss + 0, M->w("value1_b").g);
    }
    gemm32(M, lin_dw(DT_F32, R, z.VAL_IN, 256, Wk.d_v1pre, 256, Wk.bvin, z.VAL_IN,
                     M->w("value1_w").g), s);
    {
        GemmArgs a = lin_dx(DT_F32, R, z.VAL_IN, 256, Wk.d_v1pre, 256,
                            f32w(M->w("value1_w"), z.VAL_IN), Wk.dbvin, z.VAL_IN, DT_F32);
        a.accumulate = 1;
        gemm32(M, a, s);
    }
    ++g_ptcg_launches, k_val_in_bwd<<<cdiv((long)R * z.VAL_IN, TPB), TPB, 0, s>>>(Wk.dh, z.LSEQ, D, Wk.dgd, Wk.dbvin, R, 1);
    // ---- aux: prize BCE over MY_UNSEEN tokens
    ++g_ptcg_launches, k_prize_bwd<<<std::min<unsigned>(cdiv((long)R * z.LTOK, 8), M->adam_grid), 256, (D + 2) * sizeof(float), s>>>(Wk.dh, M->w("aux_prize_w").g,
        M->w("aux_prize_b").g, Wk.prize_logit, Wk.h, M->w("aux_prize_w").p, obs, ol, prize_cnt_dev,
        prize_cnt_host, D, R, aux_loss + 2);
    W wo = M->w("oracle_proj_w");
    {   // oracle_proj bias grad: fp32 sum of the critic-input grad rows 1+LSEQ..
        colsum_rows(M, M->w("oracle_proj_b").g, Wk.dx, D, R, z.LCRIT, 1 + z.LSEQ, 56, D, s);
    }
    gemm(M, lin_dw(dt, R * 56, 134, D, Wk.dotok, D, Wk.otokin, rup(134, 8), wo.g), s);
    gemm(M, lin_dx(dt, R * 56, 134, D, Wk.dotok, D, wo, Wk.dotokin, 136, DT_F32), s);
    ++g_ptcg_launches, k_otok_bwd<<<cdiv((long)R * 56 * 32, TPB), TPB, 0, s>>>(t.d_cv, Wk.dotokin, 136, obs, ol, R);
    // ---- option scorer (d scores = grad[:, :NOPT])
    ++g_ptcg_launches, k_scale_copy<<<cdiv(NO, TPB), TPB, 0, s>>>(Wk.dscores, z.NOPT, grad, z.NOPT + 1, R, z.NOPT, 1.f);
    {
        // one sample per block: the block sums of d s1pre are d u (the
        // per-sample broadcast term of score1)
        int rpb = z.NOPT;
        unsigned g = cdiv(NO, rpb);
        ++g_ptcg_launches, k_rowdot_bwd_v4<<<g, 256, 0, s>>>((float*)Wk.ds1pre, 256,
                (const float*)Wk.s1pre, 256, (const float*)Wk.s1, 256, M->w("score2_w").p,
                M->w("score2_w").g, M->w("score2_b").g, Wk.dscores, 1, (int)NO, 256, rpb,
                M->w("score1_b").g, Wk.du);
    }
    W ws1 = f32w(M->w("score1_w"), z.SCORE_IN);
    const float* qq = (const float*)Wk.scin;
    {
        // [q | q*r] part -> score1_w columns [0, D) and [2D + 192, 3D + 192)
        GemmArgs a = lin_dw(DT_F32, (int)NO, D, 256, Wk.ds1pre, 256, qq, 2 * D, ws1.g);
        a.ldo = z.SCORE_IN; a.allow_tf32 = tf32;
        gemm(M, a, s);
        a = lin_dw(DT_F32, (int)NO, D, 256, Wk.ds1pre, 256, qq + D, 2 * D, ws1.g + 2 * D + 192);
        a.ldo = z.SCORE_IN; a.allow_tf32 = tf32;
        gemm(M, a, s);
        // per-sample part -> columns [D, 2D + 192)
        a = lin_dw(DT_F32, R, D + 192, 256, Wk.du, 256, Wk.rgd, D + 192, ws1.g + D);
        a.ldo = z.SCORE_IN; a.allow_tf32 = tf32;
        gemm(M, a, s);
        W wqq = ws1; wqq.op = Wk.wqq; wqq.ld = 2 * D;
        a = lin_dx(DT_F32, (int)NO, 2 * D, 256, Wk.ds1pre, 256, wqq, Wk.dscin, 2 * D, DT_F32);
        a.allow_tf32 = tf32;
        gemm(M, a, s);
        W wrgd = ws1; wrgd.op = ws1.p + D;
        a = lin_dx(DT_F32, R, D + 192, 256, Wk.du, 256, wrgd, Wk.drgd, D + 192, DT_F32);
        a.allow_tf32 = tf32;
        gemm(M, a, s);
    }
    ++g_ptcg_launches, k_qq_bwd<float><<<R, 256, 0, s>>>((float*)Wk.dq, D, Wk.dh, Wk.dgd, (const float*)Wk.dscin,
            qq, Wk.drgd, Wk.h, D, z.LSEQ, z.NOPT, M->w("q2_b").g);
    W wq2 = f32w(M->w("q2_w"), D), wq1 = f32w(M->w("q1_w"), z.Q_IN);
    {
        GemmArgs a = lin_dw(DT_F32, (int)NO, D, D, Wk.dq, D, Wk.q1, D, wq2.g);
        a.allow_tf32 = tf32;
        gemm(M, a, s);
        a = lin_dx(DT_F32, (int)NO, D, D, Wk.dq, D, wq2, Wk.dq1, D, DT_F32);
        a.act = ACT_GELU_BWD; a.aux = Wk.q1pre; a.ld_aux = D; a.aux_dtype = DT_F32;
        a.colsum = M->w("q1_b").g; a.allow_tf32 = tf32;
        gemm(M, a, s);
    }
    long ldq = rup(z.Q_IN, 8);
    {
        GemmArgs a = lin_dw(DT_F32, (int)NO, z.Q_IN, D, Wk.dq1, D, Wk.qin, ldq, wq1.g);
        a.allow_tf32 = tf32;
        gemm(M, a, s);
        a = lin_dx(DT_F32, (int)NO, z.Q_IN, D, Wk.dq1, D, wq1, Wk.dqin, z.Q_IN, DT_F32);
        a.allow_tf32 = tf32;
        gemm(M, a, s);
    }
    ++g_ptcg_launches, k_q_in_bwd<<<cdiv(NO, TPB / 32), TPB, 0, s>>>(M->w("opt_type_emb").g, Wk.dh, t.d_poc,
        t.d_poa, Wk.dqin, z.Q_IN, obs, ol, D, R, z.Q_IN);
    // opt_card / opt_attack per-table-row projections -> table grads
    colsum<float>(M->w("opt_card_b").g, t.d_poc, 64, z.NC, 64, s);
    gemm32(M, lin_dw(DT_F32, z.NC, 128, 64, t.d_poc, 64, t.card_vec, 128, M->w("opt_card_w").g), s);
    {
        GemmArgs a = lin_dx(DT_F32, z.NC, 128, 64, t.d_poc, 64, f32w(M->w("opt_card_w"), 128),
                            t.d_cv, 128, DT_F32);
        a.accumulate = 1;
        gemm32(M, a, s);
    }
    colsum<float>(M->w("opt_attack_b").g, t.d_poa, 64, z.NA, 64, s);
    gemm32(M, lin_dw(DT_F32, z.NA, 64, 64, t.d_poa, 64, t.att_tab, 64, M->w("opt_attack_w").g), s);
    {
        GemmArgs a = lin_dx(DT_F32, z.NA, 64, 64, t.d_poa, 64, f32w(M->w("opt_attack_w"), 64),
                            t.d_att, 64, DT_F32);
        a.accumulate = 1;
        gemm32(M, a, s);
    }
    // ---- ln_f
    // (+ the last block's FFN2 bias grad = column sums of d(x_L))
    ln_bwd(dt, Wk.dx, 0, bf ? Wk.dxc : nullptr, M->w("lnf_w").g, M->w("lnf_b").g, Wk.dh,
           Wk.x[z.LAYERS], M->w("lnf_w").p, Wk.muf, Wk.rsf, (int)NS, D, s,
           M->w(("b" + std::to_string(z.LAYERS - 1) + "_ffn2_b").c_str()).g, DT_F32, Wk.ext, z.LSEQ);
    if (last) fire_hook(M, "lnf_w", nullptr, s);
    // ---- trunk
    for (int i = z.LAYERS - 1; i >= 0; i--) {
        std::string p = "b" + std::to_string(i) + "_";
        block_bwd(M, M->blk(p), Wk.blk[i], Wk.keep, Wk, R, z.LSEQ,
                  i > 0 ? M->w(("b" + std::to_string(i - 1) + "_ffn2_b").c_str()).g : nullptr, s);
        if (last) fire_hook(M, (p + "ln1_w").c_str(),
                            i == z.LAYERS - 1 ? "lnf_w" : ("b" + std::to_string(i + 1) + "_ln1_w").c_str(), s);
    }
    // ---- x0 split, token projection, broadcast
    {   // readout grad: column sum of row 0 over samples
        colsum_rows(M, M->w("readout").g, Wk.dx, D, R, z.LSEQ, 0, 1, D, s);
    }
    if (bf)
        ++g_ptcg_launches, k_x0_bwd<bf16><<<R, 256, 0, s>>>((bf16*)Wk.dtokp, Wk.dbc, Wk.dx, z.LTOK, D, Wk.ext);
    else
        ++g_ptcg_launches, k_x0_bwd<float><<<R, 256, 0, s>>>((float*)Wk.dtokp, Wk.dbc, Wk.dx, z.LTOK, D, Wk.ext);
    W wt = M->w("token_proj_w");
    long ldtok = rup(z.TOK_IN, 8);
    colsum<float>(M->w("token_proj_b").g, Wk.dbc, D, R, D, s);
    gemm(M, lin_dw(dt, R * z.LTOK, z.TOK_IN, D, Wk.dtokp, D, Wk.tokcat, ldtok, wt.g), s);
    gemm(M, lin_dx(dt, R * z.LTOK, z.TOK_IN, D, Wk.dtokp, D, wt, Wk.dtokcat, z.TOK_IN, DT_F32), s);
    ++g_ptcg_launches, k_tok_cat_bwd<<<std::min<unsigned>(cdiv((long)R * z.LTOK, TPB / 32), M->adam_grid), TPB, 0, s>>>(t.d_cv, M->w("zone_emb").g,
        M->w("owner_emb").g, Wk.dtokcat, z.TOK_IN, obs, ol, R, z.TOK_IN, Wk.ext);
    colsum<float>(M->w("bcast_b").g, Wk.dbc, D, R, D, s);
    gemm32(M, lin_dw(DT_F32, R, 192, D, Wk.dbc, D, Wk.gd, 192, M->w("bcast_w").g), s);
    {
        GemmArgs a = lin_dx(DT_F32, R, 192, D, Wk.dbc, D, f32w(M->w("bcast_w"), 192), Wk.dgd, 192, DT_F32);
        a.accumulate = 1;
        gemm32(M, a, s);
    }
    // ---- decision encoder
    colsum<float>(M->w("dec2_b").g, Wk.dgd + 128, 192, R, 64, s);
    gemm32(M, lin_dw(DT_F32, R, 64, 64, Wk.dgd + 128, 192, Wk.d1, 64, M->w("dec2_w").g), s);
    {
        GemmArgs a = lin_dx(DT_F32, R, 64, 64, Wk.dgd + 128, 192, f32w(M->w("dec2_w"), 64), Wk.dd1,
                            64, DT_F32);
        a.act = ACT_GELU_BWD; a.aux = Wk.d1pre; a.ld_aux = 64; a.aux_dtype = DT_F32;
        gemm32(M, a, s);
    }
    colsum<float>(M->w("dec1_b").g, Wk.dd1, 64, R, 64, s);
    gemm32(M, lin_dw(DT_F32, R, 696, 64, Wk.dd1, 64, Wk.decin, 696, M->w("dec1_w").g), s);
    gemm32(M, lin_dx(DT_F32, R, 696, 64, Wk.dd1, 64, f32w(M->w("dec1_w"), 696), Wk.ddecin, 696,
                     DT_F32), s);
    ++g_ptcg_launches, k_dec_in_bwd<<<cdiv((long)R * 696, TPB), TPB, 0, s>>>(t.d_cv, t.d_att, M->w("sel_type_emb").g,
        M->w("ctx_emb").g, Wk.ddecin, obs, ol, R);
    // ---- global encoder
    colsum<float>(M->w("global2_b").g, Wk.dgd, 192, R, 128, s);
    gemm32(M, lin_dw(DT_F32, R, 128, 128, Wk.dgd, 192, Wk.g1, 128, M->w("global2_w").g), s);
    {
        GemmArgs a = lin_dx(DT_F32, R, 128, 128, Wk.dgd, 192, f32w(M->w("global2_w"), 128), Wk.dg1,
                            128, DT_F32);
        a.act = ACT_GELU_BWD; a.aux = Wk.g1pre; a.ld_aux = 128; a.aux_dtype = DT_F32;
        gemm32(M, a, s);
    }
    colsum<float>(M->w("global1_b").g, Wk.dg1, 128, R, 128, s);
    gemm32(M, lin_dw(DT_F32, R, 64, 128, Wk.dg1, 128, obs + ol.glob, ol.obs, M->w("global1_w").g), s);
    if (last) fire_hook(M, "zone_emb", "b0_ln1_w", s);
    return 0;
}

// ================================================================= C-ABI
extern "C" {

const char* ptcg_last_error(void) { return g_err; }
int ptcg_abi_version(void) { return PTCG_B200_ABI_VERSION; }

static int check_shape(const PtcgShape* s) {
    REQ(s, PTCG_EINVAL, "null shape");
    REQ(s->d > 0 && s->heads > 0 && s->d % s->heads == 0 && s->d / s->heads == 32, PTCG_EINVAL,
        "head width d/heads must be 32 (d=%d heads=%d)", s->d, s->heads);
    REQ(s->heads <= 16, PTCG_EINVAL, "heads must be <= 16 (d <= 512), got %d", s->heads);
    REQ(s->d % 8 == 0 && s->ffn % 8 == 0 && s->ffn > 0 && s->layers >= 1, PTCG_EINVAL,
        "d and ffn must be multiples of 8, layers >= 1");
    REQ(s->ltok >= 1 && s->ltok <= 256 && s->nopt >= 1 && s->nopt <= 1024 && s->tok_f >= 0,
        PTCG_EINVAL, "ltok must be in [1, 256], nopt in [1, 1024]");
    REQ(s->n_cards >= 2 && s->n_attacks >= 1 && s->n_skills >= 1, PTCG_EINVAL, "bad vocab sizes");
    return PTCG_OK;
}

static ObsLayout make_layout(const PtcgShape& s) {
    ObsLayout L;
    L.toki = 0;
    L.tokf = L.toki + s.ltok * 5;
    L.opti = L.tokf + s.ltok * s.tok_f;
    L.optf = L.opti + s.nopt * 6;
    L.mask = L.optf + s.nopt * 8;
    L.glob = L.mask + s.nopt;
    L.deci = L.glob + 64;
    L.decf = L.deci + 8;
    L.orc = L.decf + 16;
    L.obs = L.orc + 136;
    L.ltok = s.ltok; L.lseq = s.ltok + 1; L.nopt = s.nopt; L.tok_f = s.tok_f;
    L.nc = s.n_cards; L.na = s.n_attacks; L.ns = s.n_skills;
    return L;
}

long ptcg_obs_size(const PtcgShape* s) {
    if (check_shape(s)) return -1;
    return make_layout(*s).obs;
}

// The transfer form of an observation row: the fields that hold ids (token
// and option ints, the option mask, the decision ints, the oracle block's
// card ids) as int16, every other field as fp32, in row order within each
// part.  Oracle block (buffers.py): 24 hand (id, count) pairs, 24 split
// (id, count, count) triples, 8 prize (id, count) pairs.
static ObsPacking obs_packing(const PtcgShape& s) {
    const ObsLayout L = make_layout(s);
    ObsPacking p{};
    auto add = [](ObsRuns& r, int dst, int count, int stride) {
        r.dst[r.n] = dst; r.count[r.n] = count; r.stride[r.n] = stride; r.n++;
    };
    add(p.ints, L.toki, s.ltok * 5, 1);
    add(p.ints, L.opti, s.nopt * 6, 1);
    add(p.ints, L.mask, s.nopt, 1);
    add(p.ints, L.deci, 8, 1);
    add(p.ints, L.orc, 24, 2);
    add(p.ints, L.orc + 48, 24, 3);
    add(p.ints, L.orc + 120, 8, 2);
    add(p.floats, L.tokf, s.ltok * s.tok_f, 1);
    add(p.floats, L.optf, s.nopt * 8, 1);
    add(p.floats, L.glob, 64, 1);
    add(p.floats, L.decf, 16, 1);
    add(p.floats, L.orc + 1, 24, 2);
    add(p.floats, L.orc + 49, 24, 3);
    add(p.floats, L.orc + 50, 24, 3);
    add(p.floats, L.orc + 121, 8, 2);
    long ni = 0, nf = 0;
    for (int k = 0; k < p.ints.n; k++) ni += p.ints.count[k];
    for (int k = 0; k < p.floats.n; k++) nf += p.floats.count[k];
    p.obs = L.obs;
    p.float_off = (ni * 2 + 15) / 16 * 16;
    p.row_bytes = (p.float_off + nf * 4 + 15) / 16 * 16;
    return p;
}

long ptcg_obs_packed_bytes(const PtcgShape* s) {
    if (check_shape(s)) return -1;
    return obs_packing(*s).row_bytes;
}

int ptcg_obs_pack(const PtcgShape* s, const float* rows, long n, void* packed, long* bad_index) {
    if (check_shape(s)) return PTCG_EINVAL;
    REQ(rows && packed && n >= 0, PTCG_EINVAL, "bad arguments");
    const ObsPacking p = obs_packing(*s);
    for (long r = 0; r < n; r++) {
        const float* in = rows + r * p.obs;
        uint8_t* row = (uint8_t*)packed + r * p.row_bytes;
        int16_t* iv = (int16_t*)row;
        float* fv = (float*)(row + p.float_off);
        long b = 0;
        for (int k = 0; k < p.ints.n; k++)
            for (int e = 0; e < p.ints.count[k]; e++) {
                const long col = p.ints.dst[k] + (long)e * p.ints.stride[k];
                const float x = in[col];
                if (!(x == truncf(x) && x >= -32768.f && x <= 32767.f)) {
                    if (bad_index) *bad_index = r * p.obs + col;
                    set_err("obs row %ld column %ld holds %g: not an integer in the int16 range "
                            "of the compact form", r, col, (double)x);
                    return PTCG_EINVAL;
                }
                iv[b++] = (int16_t)x;
            }
        for (long i = b * 2; i < p.float_off; i++) row[i] = 0;
        b = 0;
        for (int k = 0; k < p.floats.n; k++)
            for (int e = 0; e < p.floats.count[k]; e++)
                fv[b++] = in[p.floats.dst[k] + (long)e * p.floats.stride[k]];
        for (long i = p.float_off + b * 4; i < p.row_bytes; i++) row[i] = 0;
    }
    return PTCG_OK;
}

int ptcg_obs_unpack(const PtcgShape* s, const void* packed, long n, float* rows, void* stream) {
    if (check_shape(s)) return PTCG_EINVAL;
    REQ(packed && rows && n >= 0, PTCG_EINVAL, "bad arguments");
    REQ(((uintptr_t)packed & 15) == 0, PTCG_EINVAL, "packed rows must be 16-byte aligned");
    if (n == 0) return PTCG_OK;
    const ObsPacking p = obs_packing(*s);
    REQ(n <= 0x7fffffffL, PTCG_ERANGE, "too many rows");
    ++g_ptcg_launches, k_obs_unpack<<<(unsigned)n, 256, 0, (cudaStream_t)stream>>>(
        rows, (const uint8_t*)packed, p, n);
    CKL();
    return PTCG_OK;
}

long ptcg_seat_column(const PtcgShape* s) {
    if (check_shape(s)) return -1;
    return make_layout(*s).glob + 31;              // global_f[31], GlobF.ACTOR_SEAT
}

int ptcg_num_params(const PtcgShape* s) {
    if (check_shape(s)) return -1;
    return (int)param_defs(*s).size();
}

int ptcg_param_info(const PtcgShape* s, int i, const char** name, long* rows, long* cols) {
    int e = check_shape(s);
    if (e) return e;
    static thread_local std::vector<ParamDef> defs;
    defs = param_defs(*s);
    REQ(i >= 0 && i < (int)defs.size(), PTCG_EINVAL, "param index %d out of range", i);
    // names are stable string literals per (process, index): keep a copy
    static std::unordered_map<std::string, std::string> interned;
    auto it = interned.find(defs[i].name);
    if (it == interned.end()) it = interned.emplace(defs[i].name, defs[i].name).first;
    if (name) *name = it->second.c_str();
    if (rows) *rows = defs[i].r;
    if (cols) *cols = defs[i].c;
    return PTCG_OK;
}

long ptcg_param_total(const PtcgShape* s) {
    if (check_shape(s)) return -1;
    long n = 0;
    for (auto& p : param_defs(*s)) n += numel(p);
    return n;
}

int ptcg_create(const PtcgShape* s, int precision, int device, PtcgModel** out) {
    int e = check_shape(s);
    if (e) return e;
    REQ(out, PTCG_EINVAL, "null out");
    REQ(precision == PTCG_FP32 || precision == PTCG_BF16, PTCG_EINVAL, "bad precision %d", precision);
    int ndev = 0;
    CK(cudaGetDeviceCount(&ndev));
    REQ(device >= 0 && device < ndev, PTCG_EINVAL, "device %d not present (%d devices)", device, ndev);
    CK(cudaSetDevice(device));
    PtcgModel* M = new PtcgModel();
    M->s = *s; M->prec = precision; M->dev = device;
    Dims& z = M->z;
    z.D = s->d; z.H = s->heads; z.FFN = s->ffn; z.LAYERS = s->layers; z.LTOK = s->ltok;
    z.LSEQ = s->ltok + 1; z.NOPT = s->nopt; z.LCRIT = 1 + z.LSEQ + 56; z.NC = s->n_cards;
    z.NA = s->n_attacks; z.NS = s->n_skills; z.TOKF = s->tok_f;
    z.TOK_IN = 256 + s->tok_f + 12; z.Q_IN = 16 + 2 * s->d + 136; z.SCORE_IN = 3 * s->d + 192;
    z.VAL_IN = s->d + 128;
    z.ol = make_layout(*s);
    M->defs = param_defs(*s);
    long off = 0;
    for (size_t i = 0; i < M->defs.size(); i++) {
        M->idx[M->defs[i].name] = (int)i;
        M->off.push_back(off);
        off += rup(numel(M->defs[i]), 4);          // 16-byte aligned per tensor
    }
    M->n_arena = off;
    size_t ab = (size_t)off * 4;
    CK(cudaMalloc(&M->params, ab)); CK(cudaMalloc(&M->grads, ab));
    CK(cudaMalloc(&M->am, ab)); CK(cudaMalloc(&M->av, ab));
    CK(cudaMemset(M->params, 0, ab)); CK(cudaMemset(M->grads, 0, ab));
    CK(cudaMemset(M->am, 0, ab)); CK(cudaMemset(M->av, 0, ab));
    CK(cudaMalloc(&M->step_dev, sizeof(long long)));
    CK(cudaMemset(M->step_dev, 0, sizeof(long long)));
    // bf16 compute copies of the matrices that feed tensor-core GEMMs
    M->copy_ld.assign(M->defs.size(), 0);
    M->copy_ptr.assign(M->defs.size(), nullptr);
    if (precision == PTCG_BF16) {
        std::vector<int> which;
        for (size_t i = 0; i < M->defs.size(); i++) {
            const std::string& n = M->defs[i].name;
            bool blockmat = (n.size() > 3 && (n[0] == 'b' || n[0] == 'c') && n[1] >= '0' && n[1] <= '9' &&
                             (n.find("qkv_w") != std::string::npos || n.find("proj_w") != std::string::npos ||
                              n.find("ffn1_w") != std::string::npos || n.find("ffn2_w") != std::string::npos));
            if (blockmat || n == "token_proj_w" || n == "oracle_proj_w" || n == "aux_hand_w")
                which.push_back((int)i);
        }
        long tot = 0;
        for (int i : which) tot += M->defs[i].r * rup(M->defs[i].c, 8);
        CK(cudaMalloc(&M->wbf, (size_t)tot * 2));
        CK(cudaMemset(M->wbf, 0, (size_t)tot * 2));
        long o = 0;
        for (int i : which) {
            long ld = rup(M->defs[i].c, 8);
            BfCopy c;
            c.off = M->off[i]; c.n = numel(M->defs[i]); c.cols = (int)M->defs[i].c; c.ldp = (int)ld;
            c.dst = M->wbf + o;
            M->copies.push_back(c);
            M->copy_ld[i] = ld; M->copy_ptr[i] = M->wbf + o;
            o += M->defs[i].r * ld;
        }
        CK(cudaMalloc(&M->d_copies, sizeof(BfCopy) * M->copies.size()));
        CK(cudaMemcpy(M->d_copies, M->copies.data(), sizeof(BfCopy) * M->copies.size(),
                      cudaMemcpyHostToDevice));
        long nchunks = (M->n_arena + M->adam_chunk - 1) / M->adam_chunk;
        std::vector<int> cc(nchunks);
        size_t ci = 0;
        for (long c = 0; c < nchunks; c++) {
            long c0 = c * M->adam_chunk;
            while (ci < M->copies.size() && c0 >= M->copies[ci].off + M->copies[ci].n) ci++;
            cc[c] = (int)ci;
        }
        CK(cudaMalloc(&M->d_chunk_copy, sizeof(int) * nchunks));
        CK(cudaMemcpy(M->d_chunk_copy, cc.data(), sizeof(int) * nchunks, cudaMemcpyHostToDevice));
    }
    cudaDeviceProp prop;
    CK(cudaGetDeviceProperties(&prop, device));
    // one wave of resident blocks for both optimizer passes
    int per_sm = 0;
    CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_adam, 256, 0));
    M->adam_grid = prop.multiProcessorCount * (per_sm > 0 ? per_sm : 1);
    CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_sumsq, 256, 0));
    M->sumsq_grid = prop.multiProcessorCount * (per_sm > 0 ? per_sm : 1);
    CK(cudaMalloc(&M->d_partials, sizeof(double) * M->sumsq_grid));
    {   // Muon scratch: gram pair [maxM^2] and the iterate [maxM x maxN]
        long mm = 0, mn = 0;
        for (auto& d : M->defs)
            if (d.c > 0) { mm = std::max(mm, std::min(d.r, d.c)); mn = std::max(mn, std::max(d.r, d.c)); }
        if (mm > 0) {
            CK(cudaMalloc(&M->mu_gram, sizeof(float) * mm * mm));
            CK(cudaMalloc(&M->mu_gram2, sizeof(float) * mm * mm));
            CK(cudaMalloc(&M->mu_x, sizeof(float) * mm * mn));
        }
        CK(cudaMalloc(&M->mu_partials, sizeof(double) * M->sumsq_grid));
    }
    CK(cudaMalloc(&M->d_misc, sizeof(float) * 64));
    CK(cudaMemset(M->d_misc, 0, sizeof(float) * 64));
    CK(cudaMalloc(&M->d_ck, 16));
    // table activations
    Bump b{nullptr, 0, true};
    plan_tab(M->tab, b, z);
    CK(cudaMalloc(&M->tab_base, b.off));
    CK(cudaMemset(M->tab_base, 0, b.off));
    Bump b2{(char*)M->tab_base, 0, false};
    plan_tab(M->tab, b2, z);
    *out = M;
    return PTCG_OK;
}

static void free_work(Work& w) { if (w.base) cudaFree(w.base); w = Work(); }

int ptcg_destroy(PtcgModel* M) {
    if (!M) return PTCG_OK;
    cudaSetDevice(M->dev);
    cudaDeviceSynchronize();
    dp_destroy(M->dp, false);
    M->dp = nullptr;
    free_work(M->roll); free_work(M->trn);
    void* ptrs[] = {M->params, M->grads, M->am, M->av, M->step_dev, M->wbf, M->d_copies,
                    M->d_chunk_copy, M->d_partials, M->d_misc, M->d_ck, M->card_static,
                    M->att_static, M->card_text, M->att_text, M->skill_text, M->card_attacks,
                    M->card_skills, M->tab_base, M->mu_gram, M->mu_gram2, M->mu_x,
                    M->mu_partials};
    for (void* p : ptrs) if (p) cudaFree(p);
    delete M;
    return PTCG_OK;
}

static void refresh_tables(PtcgModel* M, cudaStream_t s);

int ptcg_set_tables(PtcgModel* M, const float* card_static, const int* card_attacks,
                    const int* card_skills, const float* att_static, const float* card_text,
                    const float* att_text, const float* skill_text) {
    REQ(M && card_static && card_attacks && card_skills && att_static && card_text && att_text &&
        skill_text, PTCG_EINVAL, "null table pointer");
    CK(cudaSetDevice(M->dev));
    const Dims& z = M->z;
    for (int k = 0; k < (long)z.NC * 4; k++)
        REQ(card_attacks[k] >= 0 && card_attacks[k] < z.NA, PTCG_EINVAL,
            "card_attacks[%d]=%d outside [0, %d)", k, card_attacks[k], z.NA);
    for (int k = 0; k < (long)z.NC * 2; k++)
        REQ(card_skills[k] >= 0 && card_skills[k] < z.NS, PTCG_EINVAL,
            "card_skills[%d]=%d outside [0, %d)", k, card_skills[k], z.NS);
#define UP(dst, src, n, T) do { if (!M->dst) CK(cudaMalloc(&M->dst, (size_t)(n) * sizeof(T))); \
    CK(cudaMemcpy(M->dst, src, (size_t)(n) * sizeof(T), cudaMemcpyHostToDevice)); } while (0)
    UP(card_static, card_static, (long)z.NC * 58, float);
    UP(card_attacks, card_attacks, (long)z.NC * 4, int);
    UP(card_skills, card_skills, (long)z.NC * 2, int);
    UP(att_static, att_static, (long)z.NA * 15, float);
    UP(card_text, card_text, (long)z.NC * 128, float);
    UP(att_text, att_text, (long)z.NA * 64, float);
    UP(skill_text, skill_text, (long)z.NS * 64, float);
#undef UP
    M->tables_ready = true;
    M->tab_fresh = false;
    if (M->weights_ready) {
        refresh_tables(M, 0);
        CKL();
        CK(cudaDeviceSynchronize());
    }
    return PTCG_OK;
}

// The static-table activations (tables_fwd) of the current master weights,
// into M->tab.  Batch-independent: recomputed when the weights change, not
// per forward.
static void refresh_tables(PtcgModel* M, cudaStream_t s) {
    if (!M->tables_ready) { M->tab_fresh = false; return; }
    tables_fwd(M, M->tab, s);
    M->tab_fresh = true;
}

// After the master weights changed: the bf16 compute copies and the table
// activations
static int refresh_copies(PtcgModel* M, cudaStream_t s) {
    if (!M->copies.empty()) {
        dim3 g(64, (unsigned)M->copies.size());
        ++g_ptcg_launches, k_refresh_copies<<<g, 256, 0, s>>>(M->params, M->d_copies, (int)M->copies.size());
    }
    refresh_tables(M, s);
    CKL();
    return PTCG_OK;
}

int ptcg_load_weights(PtcgModel* M, const float* packed, long n) {
    REQ(M && packed, PTCG_EINVAL, "null argument");
    long tot = 0;
    for (auto& p : M->defs) tot += numel(p);
    REQ(n == tot, PTCG_EINVAL, "blob has %ld floats, expected %ld", n, tot);
    CK(cudaSetDevice(M->dev));
    long o = 0;
    for (size_t i = 0; i < M->defs.size(); i++) {
        long k = numel(M->defs[i]);
        CK(cudaMemcpy(M->params + M->off[i], packed + o, k * 4, cudaMemcpyHostToDevice));
        o += k;
    }
    int e = refresh_copies(M, 0);
    if (e) return e;
    CK(cudaDeviceSynchronize());
    M->weights_ready = true;
    return PTCG_OK;
}

int ptcg_save_weights(PtcgModel* M, float* packed, long n) {
    REQ(M && packed, PTCG_EINVAL, "null argument");
    long tot = 0;
    for (auto& p : M->defs) tot += numel(p);
    REQ(n == tot, PTCG_EINVAL, "buffer has %ld floats, expected %ld", n, tot);
    CK(cudaSetDevice(M->dev));
    CK(cudaDeviceSynchronize());
    long o = 0;
    for (size_t i = 0; i < M->defs.size(); i++) {
        long k = numel(M->defs[i]);
        CK(cudaMemcpy(packed + o, M->params + M->off[i], k * 4, cudaMemcpyDeviceToHost));
        o += k;
    }
    return PTCG_OK;
}

// ---- on-disk formats (native/src/bindings.cu:202-367)
static long packed_total(const PtcgModel* M) {
    long tot = 0;
    for (auto& p : M->defs) tot += numel(p);
    return tot;
}
// device arena (16-byte aligned per tensor) <-> packed PT_PARAMS order
static int arena_to_packed(PtcgModel* M, const float* arena, std::vector<float>& out) {
    out.assign(packed_total(M), 0.f);
    long o = 0;
    for (size_t i = 0; i < M->defs.size(); i++) {
        long k = numel(M->defs[i]);
        CK(cudaMemcpy(out.data() + o, arena + M->off[i], k * 4, cudaMemcpyDeviceToHost));
        o += k;
    }
    return PTCG_OK;
}
static int packed_to_arena(PtcgModel* M, const float* packed, float* arena) {
    long o = 0;
    for (size_t i = 0; i < M->defs.size(); i++) {
        long k = numel(M->defs[i]);
        CK(cudaMemcpy(arena + M->off[i], packed + o, k * 4, cudaMemcpyHostToDevice));
        o += k;
    }
    return PTCG_OK;
}
// write whole buffers to path + ".tmp", flush, fsync, rename onto path
static int write_atomic(const char* path, const std::vector<std::pair<const void*, size_t>>& parts) {
    std::string tmp = std::string(path) + ".tmp";
    FILE* f = fopen(tmp.c_str(), "wb");
    REQ(f, PTCG_EINVAL, "cannot open %s for writing", tmp.c_str());
    bool ok = true;
    for (auto& pr : parts) ok = ok && fwrite(pr.first, 1, pr.second, f) == pr.second;
    ok = ok && fflush(f) == 0 && fsync(fileno(f)) == 0;
    fclose(f);
    REQ(ok, PTCG_EINVAL, "short write to %s", tmp.c_str());
    REQ(rename(tmp.c_str(), path) == 0, PTCG_EINVAL, "cannot rename %s -> %s", tmp.c_str(), path);
    return PTCG_OK;
}

// "PTCGSTA1" header of the reference's trainer state (bindings.cu:257-262),
// LP64: 8 + 3 x 8 bytes
struct StateHeader { char magic[8]; long global_step, epoch, n_params; };
// "PTCGADM1": the same fields plus the Adam step counter, then weights, m, v
struct AdamHeader { char magic[8]; long global_step, epoch, n_params, adam_step; };
static_assert(sizeof(StateHeader) == 32 && sizeof(AdamHeader) == 40, "LP64 header layout");

int ptcg_save_weights_file(PtcgModel* M, const char* path) {
    REQ(M && path, PTCG_EINVAL, "null argument");
    CK(cudaSetDevice(M->dev));
    CK(cudaDeviceSynchronize());
    std::vector<float> w;
    int e = arena_to_packed(M, M->params, w);
    if (e) return e;
    FILE* f = fopen(path, "wb");
    REQ(f, PTCG_EINVAL, "cannot open %s for writing", path);
    size_t nw = fwrite(w.data(), sizeof(float), w.size(), f);
    fclose(f);
    REQ(nw == w.size(), PTCG_EINVAL, "short write to %s", path);
    return PTCG_OK;
}

int ptcg_load_weights_file(PtcgModel* M, const char* path) {
    REQ(M && path, PTCG_EINVAL, "null argument");
    FILE* f = fopen(path, "rb");
    REQ(f, PTCG_EINVAL, "cannot open %s for reading", path);
    fseek(f, 0, SEEK_END);
    long bytes = ftell(f);
    fseek(f, 0, SEEK_SET);
    long n = packed_total(M);
    if (bytes != n * 4) {
        fclose(f);
        set_err("weight file size mismatch: expected %ld bytes, got %ld", n * 4, bytes);
        return PTCG_EINVAL;
    }
    std::vector<float> w(n);
    size_t nr = fread(w.data(), sizeof(float), n, f);
    fclose(f);
    REQ((long)nr == n, PTCG_EINVAL, "failed to read %s", path);
    return ptcg_load_weights(M, w.data(), n);
}

int ptcg_save_state(PtcgModel* M, const char* path, long global_step, long epoch, int format) {
    REQ(M && path, PTCG_EINVAL, "null argument");
    REQ(format == 0 || format == 1, PTCG_EINVAL, "format must be 0 (PTCGSTA1) or 1 (PTCGADM1)");
    CK(cudaSetDevice(M->dev));
    CK(cudaDeviceSynchronize());
    std::vector<float> w, m, v;
    int e = arena_to_packed(M, M->params, w);
    if (!e) e = arena_to_packed(M, M->am, m);
    if (e) return e;
    size_t nb = w.size() * sizeof(float);
    if (format == 0) {
        StateHeader h;
        memcpy(h.magic, "PTCGSTA1", 8);
        h.global_step = global_step; h.epoch = epoch; h.n_params = (long)w.size();
        return write_atomic(path, {{&h, sizeof h}, {w.data(), nb}, {m.data(), nb}});
    }
    e = arena_to_packed(M, M->av, v);
    if (e) return e;
    long long step = 0;
    CK(cudaMemcpy(&step, M->step_dev, sizeof step, cudaMemcpyDeviceToHost));
    AdamHeader h;
    memcpy(h.magic, "PTCGADM1", 8);
    h.global_step = global_step; h.epoch = epoch; h.n_params = (long)w.size();
    h.adam_step = (long)step;
    return write_atomic(path, {{&h, sizeof h}, {w.data(), nb}, {m.data(), nb}, {v.data(), nb}});
}

int ptcg_load_state(PtcgModel* M, const char* path, long* global_step, long* epoch) {
    REQ(M && path, PTCG_EINVAL, "null argument");
    FILE* f = fopen(path, "rb");
    REQ(f, PTCG_EINVAL, "cannot open %s for reading", path);
    char magic[8] = {0};
    size_t got = fread(magic, 1, 8, f);
    fseek(f, 0, SEEK_SET);
    bool sta = got == 8 && memcmp(magic, "PTCGSTA1", 8) == 0;
    bool adm = got == 8 && memcmp(magic, "PTCGADM1", 8) == 0;
    if (!sta && !adm) {
        fclose(f);
        set_err("%s is not a PTCGSTA1 / PTCGADM1 state file", path);
        return PTCG_EINVAL;
    }
    long n = packed_total(M);
    AdamHeader h{};
    size_t hb = sta ? sizeof(StateHeader) : sizeof(AdamHeader);
    bool ok = fread(&h, 1, hb, f) == hb;
    if (ok && h.n_params != n) {
        fclose(f);
        set_err("state param count mismatch: file %ld, model %ld", h.n_params, n);
        return PTCG_EINVAL;
    }
    std::vector<float> w(n), m(n), v;
    ok = ok && fread(w.data(), sizeof(float), n, f) == (size_t)n;
    ok = ok && fread(m.data(), sizeof(float), n, f) == (size_t)n;
    if (adm) {
        v.resize(n);
        ok = ok && fread(v.data(), sizeof(float), n, f) == (size_t)n;
    }
    fclose(f);
    REQ(ok, PTCG_EINVAL, "truncated state file %s", path);
    CK(cudaSetDevice(M->dev));
    int e = ptcg_load_weights(M, w.data(), n);
    if (!e) e = packed_to_arena(M, m.data(), M->am);
    if (!e && adm) e = packed_to_arena(M, v.data(), M->av);
    if (e) return e;
    if (adm) {
        long long step = h.adam_step;
        CK(cudaMemcpy(M->step_dev, &step, sizeof step, cudaMemcpyHostToDevice));
    }
    if (global_step) *global_step = h.global_step;
    if (epoch) *epoch = h.epoch;
    return PTCG_OK;
}

static int reserve_one(PtcgModel* M, Work& W, int rows, bool train) {
    if (rows <= 0) { free_work(W); return PTCG_OK; }
    if (W.base && W.R == rows) return PTCG_OK;
    free_work(W);
    Bump b{nullptr, 0, true};
    plan_work(W, b, rows, train, M->z, M->esz(), M->prec == PTCG_BF16);
    size_t bytes = (b.off + 255) & ~(size_t)255;
    void* base = nullptr;
    cudaError_t e = cudaMalloc(&base, bytes);
    if (e != cudaSuccess) {
        cudaGetLastError();
        set_err("reserve: cannot allocate %.2f GB for %d %s rows: %s", bytes / 1e9, rows,
                train ? "train" : "rollout", cudaGetErrorString(e));
        return PTCG_ECUDA;
    }
    CK(cudaMemset(base, 0, bytes));
    Bump b2{(char*)base, 0, false};
    plan_work(W, b2, rows, train, M->z, M->esz(), M->prec == PTCG_BF16);
    W.base = base; W.bytes = bytes;
    return PTCG_OK;
}

int ptcg_reserve(PtcgModel* M, int rollout_rows, int train_rows) {
    REQ(M && rollout_rows >= 0 && train_rows >= 0, PTCG_EINVAL, "bad arguments");
    CK(cudaSetDevice(M->dev));
    int e = reserve_one(M, M->roll, rollout_rows, false);
    if (e) return e;
    return reserve_one(M, M->trn, train_rows, true);
}

static int ready(PtcgModel* M) {
    REQ(M, PTCG_EINVAL, "null model");
    REQ(M->tables_ready, PTCG_ESTATE, "static tables not set (ptcg_set_tables)");
    REQ(M->weights_ready, PTCG_ESTATE, "weights not loaded (ptcg_load_weights)");
    return PTCG_OK;
}

int ptcg_forward(PtcgModel* M, const float* obs, int n, float* out, void* stream) {
    int e = ready(M);
    if (e) return e;
    REQ(obs && out && n >= 0, PTCG_EINVAL, "bad arguments");
    REQ(M->roll.base && n <= M->roll.R, PTCG_ERANGE, "rollout batch %d exceeds reserved %d", n,
        M->roll.R);
    if (n == 0) return PTCG_OK;
    CK(cudaSetDevice(M->dev));
    forward_impl(M, M->roll, M->tab, obs, n, out, false, !M->tab_fresh, (cudaStream_t)stream);
    M->tab_fresh = true;
    CKL();
    return PTCG_OK;
}

int ptcg_forward_sample(PtcgModel* M, const float* obs, int n, const float* mask,
                        long mask_stride, const float* uniforms, float* out, float* actions,
                        float* logprobs, float* values, void* stream) {
    int e = ready(M);
    if (e) return e;
    REQ(obs && out && uniforms && actions && logprobs && values && n >= 0, PTCG_EINVAL,
        "bad arguments");
    REQ(!mask || mask_stride >= M->z.NOPT, PTCG_EINVAL, "mask stride below the option count");
    REQ(M->roll.base && n <= M->roll.R, PTCG_ERANGE, "rollout batch %d exceeds reserved %d", n,
        M->roll.R);
    if (n == 0) return PTCG_OK;
    CK(cudaSetDevice(M->dev));
    SampleArgs sa{mask, mask_stride, uniforms, actions, logprobs, values};
    forward_impl(M, M->roll, M->tab, obs, n, out, false, !M->tab_fresh, (cudaStream_t)stream, &sa);
    M->tab_fresh = true;
    CKL();
    return PTCG_OK;
}

int ptcg_forward_train(PtcgModel* M, const float* obs, int n, float* out, void* stream) {
    int e = ready(M);
    if (e) return e;
    REQ(obs && out && n > 0, PTCG_EINVAL, "bad arguments");
    REQ(M->trn.base && n <= M->trn.R, PTCG_ERANGE, "train batch %d exceeds reserved %d", n, M->trn.R);
    CK(cudaSetDevice(M->dev));
    forward_impl(M, M->trn, M->tab, obs, n, out, true, !M->tab_fresh, (cudaStream_t)stream);
    M->tab_fresh = true;
    M->trn_last_obs = obs; M->trn_last_n = n;
    CKL();
    return PTCG_OK;
}

// Caller-owned rollout workspace: activations and static-table activations
// of their own, so rollout forwards on different streams (one per buffer)
// share nothing they write.
struct PtcgWorkspace {
    PtcgModel* M = nullptr;
    Work w;
    Tab tab;
    void* tab_base = nullptr;
};

int ptcg_workspace_create(PtcgModel* M, int rows, PtcgWorkspace** out) {
    REQ(M && out && rows > 0, PTCG_EINVAL, "bad arguments");
    *out = nullptr;
    CK(cudaSetDevice(M->dev));
    PtcgWorkspace* W = new PtcgWorkspace();
    W->M = M;
    int e = reserve_one(M, W->w, rows, false);
    if (e) { delete W; return e; }
    Bump b{nullptr, 0, true};
    plan_tab(W->tab, b, M->z);
    cudaError_t ce = cudaMalloc(&W->tab_base, b.off);
    if (ce != cudaSuccess) {
        cudaGetLastError();
        free_work(W->w);
        delete W;
        set_err("workspace: cannot allocate %.1f MB of table activations: %s", b.off / 1e6,
                cudaGetErrorString(ce));
        return PTCG_ECUDA;
    }
    CK(cudaMemset(W->tab_base, 0, b.off));
    Bump b2{(char*)W->tab_base, 0, false};
    plan_tab(W->tab, b2, M->z);
    *out = W;
    return PTCG_OK;
}

int ptcg_workspace_destroy(PtcgWorkspace* W) {
    if (!W) return PTCG_OK;
    CK(cudaSetDevice(W->M->dev));
    CK(cudaDeviceSynchronize());
    free_work(W->w);
    if (W->tab_base) cudaFree(W->tab_base);
    delete W;
    return PTCG_OK;
}

int ptcg_forward_ws(PtcgModel* M, PtcgWorkspace* W, const float* obs, int n, float* out,
                    void* stream) {
    int e = ready(M);
    if (e) return e;
    REQ(W && W->M == M, PTCG_EINVAL, "workspace belongs to another model");
    REQ(obs && out && n >= 0, PTCG_EINVAL, "bad arguments");
    REQ(n <= W->w.R, PTCG_ERANGE, "rollout batch %d exceeds the workspace's %d rows", n, W->w.R);
    if (n == 0) return PTCG_OK;
    CK(cudaSetDevice(M->dev));
    forward_impl(M, W->w, W->tab, obs, n, out, false, true, (cudaStream_t)stream);
    CKL();
    return PTCG_OK;
}

int ptcg_import_params(PtcgModel* M, const float* arena, long n_floats, void* stream) {
    REQ(M && arena, PTCG_EINVAL, "null argument");
    REQ(n_floats > 0 && n_floats <= M->n_arena, PTCG_EINVAL,
        "arena of %ld floats, the model's holds %ld", n_floats, M->n_arena);
    CK(cudaSetDevice(M->dev));
    cudaStream_t s = (cudaStream_t)stream;
    CK(cudaMemcpyAsync(M->params, arena, (size_t)n_floats * 4, cudaMemcpyDeviceToDevice, s));
    int e = refresh_copies(M, s);
    if (e) return e;
    M->weights_ready = true;
    return PTCG_OK;
}


int ptcg_backward(PtcgModel* M, const float* grad, const float* returns, int aux_norm_rows,
                  float prize_count, int accumulate, void* stream) {
    int e = ready(M);
    if (e) return e;
    REQ(grad && returns, PTCG_EINVAL, "null argument");
    REQ(M->trn_last_obs && M->trn_last_n > 0, PTCG_ESTATE,
        "ptcg_backward needs a preceding ptcg_forward_train");
    CK(cudaSetDevice(M->dev));
    cudaStream_t s = (cudaStream_t)stream;
    int R = M->trn_last_n;
    int norm = aux_norm_rows > 0 ? aux_norm_rows : R;
    float* cnt = M->d_misc + 2;
    float* aux = M->d_misc + 16;
    CK(cudaMemsetAsync(aux, 0, 3 * sizeof(float), s));
    if (prize_count <= 0.f) {
        CK(cudaMemsetAsync(cnt, 0, sizeof(float), s));
        ++g_ptcg_launches, k_count_unseen<<<64, 256, 0, s>>>(cnt, M->trn_last_obs, M->z.ol, R);
    }
    // bit 0: add into the arena; bit 1: more micro-batches follow, so the
    // grads are not final and the bucket hook must not fire yet
    const bool acc = (accumulate & PTCG_BWD_ACCUMULATE) != 0;
    const bool last = (accumulate & PTCG_BWD_PARTIAL) == 0;
    REQ((accumulate & ~(PTCG_BWD_ACCUMULATE | PTCG_BWD_PARTIAL)) == 0, PTCG_EINVAL,
        "ptcg_backward: unknown flag bits");
    if (!acc) CK(cudaMemsetAsync(M->grads, 0, (size_t)M->n_arena * 4, s));
    zero_table_grads(M, s);
    backward_impl(M, M->trn, M->trn_last_obs, grad, returns, R, norm,
                  prize_count > 0.f ? nullptr : cnt, prize_count, aux, last, s);
    tables_bwd(M, s);
    if (last) fire_hook(M, "card_id_emb", "zone_emb", s);
    if (M->dp_fail) { M->dp_fail = false; return PTCG_ENCCL; }
    CKL();
    return PTCG_OK;
}

int ptcg_ppo_loss(const float* dec_out, int nopt, const float* mask, const float* actions,
                  const float* old_logp, const float* advantages, const float* values,
                  const float* returns, const float* prio, int n_seg, int horizon,
                  float clip_coef, float vf_clip_coef, float vf_coef, float ent_coef,
                  float* grad_dec, float* new_logp, float* ratio, float* stats, float* scratch,
                  void* stream) {
    REQ(dec_out && mask && actions && old_logp && advantages && values && returns && prio &&
        grad_dec && new_logp && ratio && stats && scratch, PTCG_EINVAL, "null argument");
    REQ(n_seg > 0 && horizon > 0 && nopt > 0, PTCG_EINVAL, "bad sizes");
    cudaStream_t s = (cudaStream_t)stream;
    int nt = n_seg * horizon;
    float* adv_stats = scratch;
    float* partials = scratch + 16;
    ++g_ptcg_launches, k_adv_stats<<<1, 1024, 0, s>>>(adv_stats, advantages, nt);
    unsigned g = cdiv(nt, PPO_ROWS_PER_BLOCK);
    ++g_ptcg_launches, k_ppo_loss<<<g, PPO_ROWS_PER_BLOCK * 32, 0, s>>>(dec_out, nopt, mask, nopt, actions, old_logp,
        advantages, values, returns, prio, horizon, 0, nt, nt, adv_stats, clip_coef, vf_clip_coef,
        vf_coef, ent_coef, grad_dec, new_logp, ratio, partials);
    ++g_ptcg_launches, k_ppo_reduce<<<1, 32, 0, s>>>(stats, partials, (int)g, adv_stats, 0);
    CKL();
    return PTCG_OK;
}

// Library-owned PPO scratch for ptcg_ppo_loss_noalloc: one fixed array per
// device (the module's __device__ data), its address looked up once per
// device and cached.
static __device__ __align__(256) float g_ppo_noalloc_scratch[PTCG_PPO_SCRATCH_FLOATS(
    PTCG_PPO_NOALLOC_MAX_ROWS)];
static const int NOALLOC_MAX_DEVICES = 64;
static float* g_ppo_noalloc_ptr[NOALLOC_MAX_DEVICES];
static std::mutex g_ppo_noalloc_mu;

static int ppo_noalloc_scratch(float** out) {
    int dev = -1;
    CK(cudaGetDevice(&dev));
    REQ(dev >= 0 && dev < NOALLOC_MAX_DEVICES, PTCG_EINVAL,
        "device ordinal %d beyond the %d this entry point serves", dev, NOALLOC_MAX_DEVICES);
    std::lock_guard<std::mutex> lock(g_ppo_noalloc_mu);
    if (!g_ppo_noalloc_ptr[dev]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_ppo_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            cudaGetLastError();
            set_err("cudaGetSymbolAddress of the static PPO scratch failed on device %d: %s", dev,
                    cudaGetErrorString(e));
            return PTCG_ECUDA;
        }
        g_ppo_noalloc_ptr[dev] = (float*)p;
    }
    *out = g_ppo_noalloc_ptr[dev];
    return PTCG_OK;
}

int ptcg_ppo_loss_noalloc(const float* dec_out, int nopt, const float* mask, const float* actions,
                          const float* old_logp, const float* advantages, const float* values,
                          const float* returns, const float* prio, int n_seg, int horizon,
                          float clip_coef, float vf_clip_coef, float vf_coef, float ent_coef,
                          float* grad_dec, float* new_logp, float* ratio, float* stats,
                          void* stream) {
    REQ(n_seg > 0 && horizon > 0, PTCG_EINVAL, "bad sizes");
    REQ((long)n_seg * horizon <= PTCG_PPO_NOALLOC_MAX_ROWS, PTCG_ERANGE,
        "ptcg_ppo_loss_noalloc: n_seg * horizon = %ld rows exceeds its static scratch limit of "
        "%d rows; use ptcg_ppo_loss with caller scratch", (long)n_seg * horizon,
        PTCG_PPO_NOALLOC_MAX_ROWS);
    float* scratch = nullptr;
    int e = ppo_noalloc_scratch(&scratch);
    if (e) return e;
    return ptcg_ppo_loss(dec_out, nopt, mask, actions, old_logp, advantages, values, returns,
                         prio, n_seg, horizon, clip_coef, vf_clip_coef, vf_coef, ent_coef,
                         grad_dec, new_logp, ratio, stats, scratch, stream);
}

// After a vetoed step with a non-finite gradient norm (stats[0]), clear the
// train workspace on the device, so no Inf / NaN stays in rows that later
// forwards skip (k_zero_if_nonfinite).
static void clear_work_if_nonfinite(PtcgModel* M, const float* st, cudaStream_t s) {
    if (!M->trn.base) return;
    ++g_ptcg_launches, k_zero_if_nonfinite<<<M->adam_grid, 256, 0, s>>>(st, (uint4*)M->trn.base,
        (long)(M->trn.bytes / 16));
}

// Adam with the native data-parallel exchange: wait for the reduce-scatters
// of every span, clip with the global norm (this rank's shard sum of squares,
// all-reduced), update this rank's pieces, all-gather the updated weights and
// refresh the bf16 copies.  The same update as all-reduce + k_adam on every
// rank (native/src/muon.cu:209-214 then the optimizer).
static int dp_adam(PtcgModel* M, float lr, float b1, float b2, float eps, float max_norm,
                   const float* gate, float* st, cudaStream_t s) {
    int seen = 0;
    REQ(!dp_join(M->dp, s, &seen), PTCG_ENCCL, "data-parallel join: %s", dp_last_error());
    REQ(seen == dp_nbuckets(M->dp), PTCG_ESTATE,
        "data-parallel Adam: %d of %d gradient spans were reduce-scattered since the last step "
        "(run the final backward first)", seen, dp_nbuckets(M->dp));
    long used = 0;
    const long* seg = nullptr;
    int nseg = 0;
    double* ss = nullptr;
    float* shard = dp_shard(M->dp, &used, &seg, &nseg, &ss);
    ++g_ptcg_launches, k_sumsq<<<M->sumsq_grid, 256, 0, s>>>(M->d_partials, shard, used);
    ++g_ptcg_launches, k_sumsq_final<<<1, 256, 0, s>>>(ss, M->d_partials, M->sumsq_grid);
    REQ(!dp_allreduce_sum_f64(M->dp, ss, s), PTCG_ENCCL, "data-parallel norm: %s", dp_last_error());
    if (nseg > 0) {
        dim3 g((unsigned)std::max(1, M->adam_grid / nseg), (unsigned)nseg);
        ++g_ptcg_launches, k_adam_seg<<<g, 256, 0, s>>>(M->params, M->am, M->av, shard, seg, ss, lr,
            b1, b2, eps, max_norm, M->step_dev, gate, st);
    }
    ++g_ptcg_launches, k_step_inc<<<1, 1, 0, s>>>(M->step_dev, st);
    clear_work_if_nonfinite(M, st, s);
    REQ(!dp_gather_params(M->dp, M->params, s), PTCG_ENCCL, "data-parallel gather: %s",
        dp_last_error());
    CKL();
    return refresh_copies(M, s);
}

static int adam_impl(PtcgModel* M, float lr, float b1, float b2, float eps, float max_norm,
                     const float* gate, float* stats, cudaStream_t s) {
    float* st = stats ? stats : M->d_misc + 32;
    if (M->dp) return dp_adam(M, lr, b1, b2, eps, max_norm, gate, st, s);
    const bool timed = M->kt.mode == 4;
    if (timed) kt_mark(M, s);
    ++g_ptcg_launches, k_sumsq<<<M->sumsq_grid, 256, 0, s>>>(M->d_partials, M->grads, M->n_arena);
    ++g_ptcg_launches, k_adam<<<M->adam_grid, 256, 0, s>>>(M->params, M->am, M->av, M->grads, M->n_arena,
        M->d_partials, M->sumsq_grid, lr, b1, b2, eps, max_norm, M->step_dev, gate, st,
        M->d_copies, (int)M->copies.size(), M->d_chunk_copy, M->adam_chunk);
    ++g_ptcg_launches, k_step_inc<<<1, 1, 0, s>>>(M->step_dev, st);
    if (timed) { kt_mark(M, s); M->kt.launches++; }
    clear_work_if_nonfinite(M, st, s);
    refresh_tables(M, s);                   // k_adam refreshed the bf16 copies itself
    CKL();
    return PTCG_OK;
}

int ptcg_sumsq(PtcgModel* M, const float* x, long n, double* out, void* stream) {
    REQ(M && x && out && n >= 0, PTCG_EINVAL, "bad arguments");
    CK(cudaSetDevice(M->dev));
    cudaStream_t s = (cudaStream_t)stream;
    ++g_ptcg_launches, k_sumsq<<<M->sumsq_grid, 256, 0, s>>>(M->d_partials, x, n);
    ++g_ptcg_launches, k_sumsq_final<<<1, 256, 0, s>>>(out, M->d_partials, M->sumsq_grid);
    CKL();
    return PTCG_OK;
}

int ptcg_adam_segments(PtcgModel* M, const float* grad_src, const long* seg, int nseg,
                       const double* sumsq, float lr, float beta1, float beta2, float eps,
                       float max_norm, const float* gate, float* stats, void* stream) {
    int e = ready(M);
    if (e) return e;
    REQ(grad_src && seg && sumsq && nseg >= 0 && nseg <= 65535, PTCG_EINVAL, "bad arguments");
    CK(cudaSetDevice(M->dev));
    cudaStream_t s = (cudaStream_t)stream;
    float* st = stats ? stats : M->d_misc + 32;
    if (nseg > 0) {
        dim3 g((unsigned)std::max(1, M->adam_grid / std::max(1, nseg)), (unsigned)nseg);
        ++g_ptcg_launches, k_adam_seg<<<g, 256, 0, s>>>(M->params, M->am, M->av, grad_src, seg,
            sumsq, lr, beta1, beta2, eps, max_norm, M->step_dev, gate, st);
    }
    ++g_ptcg_launches, k_step_inc<<<1, 1, 0, s>>>(M->step_dev, st);
    clear_work_if_nonfinite(M, st, s);
    M->tab_fresh = false;                   // the caller gathers, then ptcg_refresh_copies
    CKL();
    return PTCG_OK;
}

int ptcg_refresh_copies(PtcgModel* M, void* stream) {
    REQ(M, PTCG_EINVAL, "null model");
    CK(cudaSetDevice(M->dev));
    return refresh_copies(M, (cudaStream_t)stream);
}

int ptcg_adam_step(PtcgModel* M, float lr, float beta1, float beta2, float eps, float max_norm,
                   const float* gate, float* stats, void* stream) {
    int e = ready(M);
    if (e) return e;
    CK(cudaSetDevice(M->dev));
    return adam_impl(M, lr, beta1, beta2, eps, max_norm, gate, stats, (cudaStream_t)stream);
}

// Newton-Schulz quintic coefficients (a, b, c) per iteration, muon.cu:116-122:
// X <- a X + (b G + c G^2) X (wide) / X (b G + c G^2) (tall), G = X X^T / X^T X
static const double kMuonNS[5][3] = {
    {4.0848, -6.8946, 2.9270}, {3.9505, -6.3029, 2.6377}, {3.7418, -5.5913, 2.3037},
    {2.8769, -3.1427, 1.2046}, {2.8366, -3.0525, 1.2012}};

// fp32-operand GEMM C[M x N] (ldc) = alpha * op + (accumulate ? C : 0) with
// A(m, k) at a (K-major: a[m * lda + k]; else a[k * lda + m]), B likewise
static void gemm_f(PtcgModel* M, int Mr, int N, int K, const float* a, long lda, int ak,
                   const float* b, long ldb, int bk, float* c, long ldc, float alpha, int acc,
                   cudaStream_t s) {
    GemmArgs g;
    g.M = Mr; g.N = N; g.K = K; g.dtype = DT_F32;
    g.A = a; g.lda = lda; g.a_kmajor = ak;
    g.B = b; g.ldb = ldb; g.b_kmajor = bk;
    g.out = c; g.ldo = ldc; g.out_dtype = DT_F32; g.alpha = alpha; g.accumulate = acc;
    gemm32(M, g, s);
}

static int muon_impl(PtcgModel* M, float lr, float mu, float wd, float wd_1d, float max_norm,
                     const float* gate, float* stats, cudaStream_t s) {
    float* st = stats ? stats : M->d_misc + 32;
    // global clip (always applied; the gate only vetoes state / weight writes)
    ++g_ptcg_launches, k_sumsq<<<M->sumsq_grid, 256, 0, s>>>(M->d_partials, M->grads, M->n_arena);
    ++g_ptcg_launches, k_muon_clip<<<M->sumsq_grid, 256, 0, s>>>(M->grads, M->n_arena, M->d_partials,
        M->sumsq_grid, max_norm, st);
    ++g_ptcg_launches, k_gate_stat<<<1, 1, 0, s>>>(st, gate);
    for (size_t i = 0; i < M->defs.size(); i++) {
        const ParamDef& d = M->defs[i];
        long n = numel(d);
        float* g = M->grads + M->off[i];
        float* w = M->params + M->off[i];
        float* mb = M->am + M->off[i];
        const float* upd = g;
        float scale = 1.f, wdi = wd;
        if (d.c > 0) {
            ++g_ptcg_launches, k_muon_nesterov<<<cdiv(n, TPB), TPB, 0, s>>>(mb, g, gate, mu, n);
            int np = (int)std::min<long>(M->sumsq_grid, cdiv(n, 256 * 4));
            if (np < 1) np = 1;
            ++g_ptcg_launches, k_sumsq<<<np, 256, 0, s>>>(M->mu_partials, g, n);
            ++g_ptcg_launches, k_muon_normalize<<<np, 256, 0, s>>>(g, n, M->mu_partials, np, 1e-7f);
            const long R = d.r, C = d.c, Mg = std::min(R, C);
            const bool tall = R > C;
            float* bufs[2] = {g, M->mu_x};
            for (int it = 0; it < 5; it++) {
                float* src = bufs[it & 1];
                float* dst = bufs[(it + 1) & 1];
                // G = X^T X (tall, C x C) or X X^T (wide, R x R)
                if (tall) gemm_f(M, (int)C, (int)C, (int)R, src, C, 0, src, C, 0, M->mu_gram, C, 1.f, 0, s);
                else gemm_f(M, (int)R, (int)R, (int)C, src, C, 1, src, C, 1, M->mu_gram, R, 1.f, 0, s);
                // B = b G + c G^2  (into mu_gram2)
                ++g_ptcg_launches, k_scale_to<<<cdiv(Mg * Mg, TPB), TPB, 0, s>>>(M->mu_gram2, M->mu_gram,
                    (float)kMuonNS[it][1], Mg * Mg);
                gemm_f(M, (int)Mg, (int)Mg, (int)Mg, M->mu_gram, Mg, 1, M->mu_gram, Mg, 0, M->mu_gram2,
                       Mg, (float)kMuonNS[it][2], 1, s);
                // X' = a X + X B (tall) / B X (wide)
                ++g_ptcg_launches, k_scale_to<<<cdiv(n, TPB), TPB, 0, s>>>(dst, src, (float)kMuonNS[it][0], n);
                if (tall) gemm_f(M, (int)R, (int)C, (int)C, src, C, 1, M->mu_gram2, C, 0, dst, C, 1.f, 1, s);
                else gemm_f(M, (int)R, (int)C, (int)R, M->mu_gram2, R, 1, src, C, 0, dst, C, 1.f, 1, s);
            }
            upd = M->mu_x;                                   // five iterations end in the scratch
            scale = sqrtf(fmaxf(1.f, (float)R / (float)C));
        } else {
            ++g_ptcg_launches, k_muon_nesterov_ema<<<cdiv(n, TPB), TPB, 0, s>>>(mb, g, gate, mu, n);
            wdi = wd_1d;
        }
        ++g_ptcg_launches, k_muon_update<<<cdiv(n, TPB), TPB, 0, s>>>(w, upd, lr, gate, wdi, scale, n);
    }
    return refresh_copies(M, s);
}

int ptcg_muon_step(PtcgModel* M, float lr, float momentum, float weight_decay, float wd_1d,
                   float max_norm, const float* gate, float* stats, void* stream) {
    int e = ready(M);
    if (e) return e;
    CK(cudaSetDevice(M->dev));
    e = muon_impl(M, lr, momentum, weight_decay, wd_1d, max_norm, gate, stats, (cudaStream_t)stream);
    if (e) return e;
    clear_work_if_nonfinite(M, stats ? stats : M->d_misc + 32, (cudaStream_t)stream);
    CKL();
    return PTCG_OK;
}

int ptcg_prio_replay(const float* advantages, int B, int T, float alpha, float beta,
                     int total_agents, int n_sel, const float* uniforms, int* idx,
                     float* mb_prio, float* probs, float* cdf, void* stream) {
    REQ(advantages && uniforms && idx && mb_prio && probs && cdf, PTCG_EINVAL, "null argument");
    REQ(B > 0 && T > 0 && n_sel >= 0, PTCG_EINVAL, "bad sizes");
    cudaStream_t s = (cudaStream_t)stream;
    ++g_ptcg_launches, k_prio_rowsum<<<B, 32, 0, s>>>(probs, advantages, T, alpha);
    ++g_ptcg_launches, k_prio_normalize<<<1, 256, 0, s>>>(probs, B);
    ++g_ptcg_launches, k_prio_cdf<<<1, 1, 0, s>>>(cdf, probs, B);
    if (n_sel > 0)
        ++g_ptcg_launches, k_prio_sample<<<cdiv(n_sel, 256), 256, 0, s>>>(idx, mb_prio, cdf, probs, uniforms, B,
            n_sel, total_agents, beta);
    CKL();
    return PTCG_OK;
}

static void gather_rows(float* dst, const float* src, const int* idx, int n, long row_floats,
                        cudaStream_t s) {
    if (n <= 0 || row_floats <= 0) return;
    long per = (row_floats & 3) == 0 ? row_floats / 4 : row_floats;
    unsigned gx = (unsigned)std::min<long>(cdiv(per, 256), 64);
    ++g_ptcg_launches, k_gather_rows<<<dim3(gx, n), 256, 0, s>>>(dst, src, idx, row_floats);
}

int ptcg_select_copy(const int* idx, int n_sel, int T, long obs_size, int nopt,
                     const float* obs, const float* actions, const float* logprobs,
                     const float* values, const float* advantages, const float* mask,
                     float* mb_obs, float* mb_actions, float* mb_logprobs, float* mb_values,
                     float* mb_advantages, float* mb_returns, float* mb_mask, void* stream) {
    REQ(idx && obs && actions && logprobs && values && advantages && mb_obs && mb_actions &&
        mb_logprobs && mb_values && mb_advantages && mb_returns, PTCG_EINVAL, "null argument");
    REQ(n_sel >= 0 && T > 0 && obs_size > 0, PTCG_EINVAL, "bad sizes");
    REQ((mask == nullptr) == (mb_mask == nullptr) && (mask == nullptr || nopt > 0), PTCG_EINVAL,
        "mask and mb_mask must both be given (with nopt > 0) or both be NULL");
    cudaStream_t s = (cudaStream_t)stream;
    gather_rows(mb_obs, obs, idx, n_sel, (long)T * obs_size, s);
    gather_rows(mb_actions, actions, idx, n_sel, T, s);
    gather_rows(mb_logprobs, logprobs, idx, n_sel, T, s);
    gather_rows(mb_values, values, idx, n_sel, T, s);
    gather_rows(mb_advantages, advantages, idx, n_sel, T, s);
    if (mask) gather_rows(mb_mask, mask, idx, n_sel, (long)T * nopt, s);
    long n = (long)n_sel * T;
    if (n > 0)
        ++g_ptcg_launches, k_add_rows_flat<<<cdiv(n, TPB), TPB, 0, s>>>(mb_returns, mb_values, mb_advantages, n);
    CKL();
    return PTCG_OK;
}

int ptcg_index_copy(float* dst, const int* idx, const float* src, int n, long row_floats,
                    void* stream) {
    REQ(dst && idx && src && n >= 0 && row_floats > 0, PTCG_EINVAL, "bad arguments");
    if (n == 0) return PTCG_OK;
    unsigned gx = (unsigned)std::min<long>(cdiv(row_floats, 256), 64);
    ++g_ptcg_launches, k_scatter_rows<<<dim3(gx, n), 256, 0, (cudaStream_t)stream>>>(dst, src, idx, row_floats);
    CKL();
    return PTCG_OK;
}

int ptcg_sample_logits(const float* dec_out, int n, int nopt, const float* mask, long mask_stride,
                       const float* uniforms, float* actions, float* logprobs, float* values,
                       void* stream) {
    REQ(dec_out && mask && uniforms && actions && logprobs && values, PTCG_EINVAL, "null argument");
    REQ(n >= 0 && nopt > 0 && mask_stride >= nopt, PTCG_EINVAL, "bad sizes");
    if (n == 0) return PTCG_OK;
    ++g_ptcg_launches, k_sample<<<cdiv(n, 8), 256, 0, (cudaStream_t)stream>>>(dec_out, n, nopt, mask, mask_stride,
        uniforms, actions, logprobs, values);
    CKL();
    return PTCG_OK;
}

int ptcg_negamax_advantage(const float* values, const float* rewards, const float* dones,
                        const float* importance, const float* obs, long obs_size, int seat_col,
                        int B, int T, float gamma, float lambda, float rho_clip, float c_clip,
                        float* advantages, void* stream) {
    REQ(values && rewards && dones && importance && obs && advantages, PTCG_EINVAL, "null argument");
    REQ(B > 0 && T > 0 && seat_col >= 0 && seat_col < obs_size, PTCG_EINVAL, "bad sizes");
    ++g_ptcg_launches, k_negamax_adv<<<cdiv(B, 128), 128, 0, (cudaStream_t)stream>>>(values, rewards, dones,
        importance, obs, obs_size, seat_col, advantages, gamma, lambda, rho_clip, c_clip, B, T);
    CKL();
    return PTCG_OK;
}

int ptcg_set_grad_hook(PtcgModel* M, ptcg_grad_hook fn, void* user) {
    REQ(M, PTCG_EINVAL, "null model");
    M->hook = fn; M->hook_user = user;
    return PTCG_OK;
}

int ptcg_train_step(PtcgModel* M, const float* obs, const float* actions, const float* old_logp,
                    const float* advantages, const float* values, const float* returns,
                    const float* prio, int n_seg, int horizon, float clip_coef,
                    float vf_clip_coef, float vf_coef, float ent_coef, float lr, float beta1,
                    float beta2, float eps, float max_norm, int skip_adam, float* stats,
                    void* stream) {
    int e = ready(M);
    if (e) return e;
    REQ(obs && actions && old_logp && advantages && values && returns && prio && stats,
        PTCG_EINVAL, "null argument");
    REQ(n_seg > 0 && horizon > 0, PTCG_EINVAL, "bad sizes");
    REQ(M->trn.base, PTCG_ESTATE, "no train workspace (ptcg_reserve)");
    CK(cudaSetDevice(M->dev));
    cudaStream_t s = (cudaStream_t)stream;
    const Dims& z = M->z;
    Work& Wk = M->trn;
    const int nt = n_seg * horizon, R = Wk.R;
    float* adv_stats = M->d_misc;
    float* cnt = M->d_misc + 2;
    CK(cudaMemsetAsync(stats, 0, 16 * sizeof(float), s));
    CK(cudaMemsetAsync(cnt, 0, sizeof(float), s));
    ++g_ptcg_launches, k_adv_stats<<<1, 1024, 0, s>>>(adv_stats, advantages, nt);
    ++g_ptcg_launches, k_count_unseen<<<128, 256, 0, s>>>(cnt, obs, z.ol, nt);
    CK(cudaMemsetAsync(M->grads, 0, (size_t)M->n_arena * 4, s));
    zero_table_grads(M, s);
    if (!M->tab_fresh) refresh_tables(M, s);
    int nmb = (nt + R - 1) / R;
    for (int mb = 0; mb < nmb; mb++) {
        int r0 = mb * R, rows = nt - r0 < R ? nt - r0 : R;
        const float* ob = obs + (long)r0 * z.ol.obs;
        forward_impl(M, Wk, M->tab, ob, rows, Wk.fused, true, false, s);
        unsigned g = cdiv(rows, PPO_ROWS_PER_BLOCK);
        ++g_ptcg_launches, k_ppo_loss<<<g, PPO_ROWS_PER_BLOCK * 32, 0, s>>>(Wk.fused, z.NOPT, ob + z.ol.mask, z.ol.obs,
            actions + r0, old_logp + r0, advantages + r0, values + r0, returns + r0, prio, horizon,
            r0, rows, nt, adv_stats, clip_coef, vf_clip_coef, vf_coef, ent_coef, Wk.dgrad, Wk.nlp,
            Wk.ratio, Wk.ppo_scratch);
        ++g_ptcg_launches, k_ppo_reduce<<<1, 32, 0, s>>>(stats, Wk.ppo_scratch, (int)g, adv_stats, 1);
        backward_impl(M, Wk, ob, Wk.dgrad, returns + r0, rows, nt, cnt, 0.f, stats + 10,
                      mb == nmb - 1, s);
    }
    tables_bwd(M, s);
    fire_hook(M, "card_id_emb", "zone_emb", s);
    if (M->dp_fail) { M->dp_fail = false; return PTCG_ENCCL; }
    if (!skip_adam) {
        e = adam_impl(M, lr, beta1, beta2, eps, max_norm, nullptr, stats + 8, s);
        if (e) return e;
    }
    CKL();
    return PTCG_OK;
}

int ptcg_arena(PtcgModel* M, int which, float** ptr, long* n_floats) {
    REQ(M && ptr && n_floats, PTCG_EINVAL, "null argument");
    float* p[] = {M->params, M->grads, M->am, M->av};
    REQ(which >= 0 && which < 4, PTCG_EINVAL, "bad arena %d", which);
    if (which == 0) M->tab_fresh = false;   // the caller may write the weights
    *ptr = p[which];
    *n_floats = M->n_arena;
    return PTCG_OK;
}

long ptcg_param_offset(PtcgModel* M, int i) {
    if (!M || i < 0 || i >= (int)M->defs.size()) return -1;
    return M->off[i];
}

int ptcg_get_step(PtcgModel* M, long* step) {
    REQ(M && step, PTCG_EINVAL, "null argument");
    CK(cudaSetDevice(M->dev));
    long long v = 0;
    CK(cudaMemcpy(&v, M->step_dev, sizeof v, cudaMemcpyDeviceToHost));
    *step = (long)v;
    return PTCG_OK;
}

int ptcg_set_step(PtcgModel* M, long step) {
    REQ(M && step >= 0, PTCG_EINVAL, "bad arguments");
    CK(cudaSetDevice(M->dev));
    long long v = step;
    CK(cudaMemcpy(M->step_dev, &v, sizeof v, cudaMemcpyHostToDevice));
    return PTCG_OK;
}

long long ptcg_launch_count(void) { return g_ptcg_launches; }

int ptcg_gemm_ex(int M, int N, int K, const void* A, long lda, int a_kmajor, const void* B,
                 long ldb, int b_kmajor, int operand_dtype, void* C, long ldc, int out_dtype,
                 const float* bias, int act, const void* aux, long ld_aux, void* out2, long ldo2,
                 float* colsum, int accumulate, int engine, void* stream) {
    REQ(A && B && C && M >= 0 && N >= 0 && K >= 0, PTCG_EINVAL, "bad arguments");
    REQ(act >= 0 && act <= 2 && engine >= 0 && engine <= 3, PTCG_EINVAL, "bad act / engine");
    GemmArgs a;
    a.M = M; a.N = N; a.K = K; a.dtype = operand_dtype == PTCG_BF16 ? DT_BF16 : DT_F32;
    a.A = A; a.lda = lda; a.a_kmajor = a_kmajor;
    a.B = B; a.ldb = ldb; a.b_kmajor = b_kmajor;
    a.out = C; a.ldo = ldc; a.out_dtype = out_dtype == PTCG_BF16 ? DT_BF16 : DT_F32;
    a.accumulate = accumulate; a.bias = bias; a.act = act;
    a.aux = aux; a.ld_aux = ld_aux; a.aux_dtype = a.out_dtype;
    a.out2 = out2; a.ldo2 = ldo2; a.out2_dtype = a.out_dtype; a.colsum = colsum;
    if (engine == 3) { a.allow_tf32 = 1; engine = 1; }
    cudaStream_t s = (cudaStream_t)stream;
    if (engine == 2) { gemm_simt(a, s); CKL(); return PTCG_OK; }
    bool done = gemm_tc_available() && gemm_tc(a, s);
    if (!done) {
        REQ(engine == 0, PTCG_EINVAL, "tcgen05 GEMM does not support this problem");
        gemm_simt(a, s);
    }
    CKL();
    return PTCG_OK;
}

int ptcg_attention_fwd(int operand_dtype, const void* qkv, long ldqkv, const unsigned char* keep,
                       void* out, long ldo, float* lse, int nseq, int L, int H, void* stream) {
    REQ(qkv && keep && out && lse && nseq >= 0 && L > 0 && L <= 320 && H > 0, PTCG_EINVAL,
        "bad arguments");
    attn_fwd(operand_dtype == PTCG_BF16 ? DT_BF16 : DT_F32, qkv, ldqkv, keep, out, ldo, lse, nseq,
             L, H, (cudaStream_t)stream);
    CKL();
    return PTCG_OK;
}

int ptcg_attention_bwd(int operand_dtype, const void* qkv, long ldqkv, const unsigned char* keep,
                       const void* out, long ldo, const void* dout, long lddo, const float* lse,
                       void* dqkv, long lddqkv, float* dbias, int nseq, int L, int H,
                       void* stream) {
    REQ(qkv && keep && out && dout && lse && dqkv && nseq >= 0 && L > 0 && L <= 320 && H > 0,
        PTCG_EINVAL, "bad arguments");
    attn_bwd(operand_dtype == PTCG_BF16 ? DT_BF16 : DT_F32, qkv, ldqkv, keep, out, ldo, dout, lddo,
             lse, dqkv, lddqkv, dbias, nseq, L, H, (cudaStream_t)stream);
    CKL();
    return PTCG_OK;
}

static __global__ void k_eval_gelu(const float* x, float* g, float* dg, int n) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    // the tensor-core epilogue's GELU pair (values 2i, 2i+1)
    if (2 * i + 1 < n) gelu2(x[2 * i], x[2 * i + 1], g[2 * i], g[2 * i + 1], dg[2 * i], dg[2 * i + 1]);
    else if (2 * i < n) { float t0, t1; gelu2(x[2 * i], 0.f, g[2 * i], t0, dg[2 * i], t1); }
}

int ptcg_eval_gelu(const float* x, float* gelu, float* gelu_grad, int n, void* stream) {
    REQ(x && gelu && gelu_grad && n >= 0, PTCG_EINVAL, "bad arguments");
    if (n == 0) return PTCG_OK;
    ++g_ptcg_launches, k_eval_gelu<<<cdiv(n, 256), 256, 0, (cudaStream_t)stream>>>(x, gelu, gelu_grad, n);
    CKL();
    return PTCG_OK;
}

int ptcg_tc_profile(int enable, unsigned long long* counters) {
    CK(cudaDeviceSynchronize());
    ptcg_tc_profile_ctl(enable, counters);
    CKL();
    return PTCG_OK;
}

int ptcg_tensor_cores(void) { return gemm_tc_available() ? 1 : 0; }

int ptcg_set_attention_impl(int impl) {
    REQ(impl >= 0 && impl <= 2, PTCG_EINVAL, "attention implementation must be 0, 1 or 2");
    attn_set_impl(impl);
    return PTCG_OK;
}

int ptcg_get_attention_impl(void) { return attn_get_impl(); }

int ptcg_set_fused_mlp(int on) {
    g_fused_mlp.store(on ? 1 : 0);
    return PTCG_OK;
}

int ptcg_device_error(void) {
    const int g = ptcg_tc_error_read_reset(), a = attn_tc_error_read_reset(),
              m = mlp_tc_error_read_reset();
    return g ? g : (a ? 100 + a : (m ? 200 + m : 0));
}

int ptcg_gemm(int M, int N, int K, const void* A, long lda, int a_kmajor, const void* B, long ldb,
              int b_kmajor, int operand_dtype, float* C, long ldc, int accumulate, int engine,
              void* stream) {
    REQ(A && B && C && M >= 0 && N >= 0 && K >= 0, PTCG_EINVAL, "bad arguments");
    REQ(operand_dtype == PTCG_FP32 || operand_dtype == PTCG_BF16, PTCG_EINVAL, "bad dtype");
    REQ(engine >= 0 && engine <= 3, PTCG_EINVAL, "bad engine");
    GemmArgs a;
    a.M = M; a.N = N; a.K = K; a.dtype = operand_dtype == PTCG_BF16 ? DT_BF16 : DT_F32;
    a.A = A; a.lda = lda; a.a_kmajor = a_kmajor;
    a.B = B; a.ldb = ldb; a.b_kmajor = b_kmajor;
    a.out = C; a.ldo = ldc; a.out_dtype = DT_F32; a.accumulate = accumulate;
    if (engine == 3) { a.allow_tf32 = 1; engine = 1; }
    cudaStream_t s = (cudaStream_t)stream;
    if (engine == 2) { gemm_simt(a, s); CKL(); return PTCG_OK; }
    bool done = gemm_tc_available() && gemm_tc(a, s);
    if (!done) {
        REQ(engine == 0, PTCG_EINVAL, "tcgen05 GEMM does not support this problem");
        gemm_simt(a, s);
    }
    CKL();
    return PTCG_OK;
}

int ptcg_kernel_timer(PtcgModel* M, int mode) {
    REQ(M && mode >= 0 && mode <= 4, PTCG_EINVAL, "bad arguments");
    M->kt.mode = mode; M->kt.used = 0; M->kt.flops = 0; M->kt.bytes = 0; M->kt.launches = 0;
    M->kt.meta.clear();
    return PTCG_OK;
}

int ptcg_kernel_timer_entries(PtcgModel* M, int max, float* ms, int* meta) {
    REQ(M && ms && meta && max >= 0, PTCG_EINVAL, "null argument");
    CK(cudaSetDevice(M->dev));
    int n = (int)(M->kt.meta.size() / 8);
    if (n > max) n = max;
    for (int i = 0; i < n; i++) {
        CK(cudaEventSynchronize(M->kt.ev[2 * i + 1]));
        CK(cudaEventElapsedTime(&ms[i], M->kt.ev[2 * i], M->kt.ev[2 * i + 1]));
        for (int k = 0; k < 8; k++) meta[8 * i + k] = M->kt.meta[8 * i + k];
    }
    return n;
}

int ptcg_kernel_timer_read(PtcgModel* M, double* ms, long* launches, double* flops) {
    REQ(M && ms && launches && flops, PTCG_EINVAL, "null argument");
    CK(cudaSetDevice(M->dev));
    double t = 0.0;
    for (int i = 0; i + 1 < M->kt.used; i += 2) {
        float e = 0.f;
        CK(cudaEventSynchronize(M->kt.ev[i + 1]));
        CK(cudaEventElapsedTime(&e, M->kt.ev[i], M->kt.ev[i + 1]));
        t += e;
    }
    *ms = t; *launches = M->kt.launches; *flops = M->kt.flops;
    return PTCG_OK;
}

int ptcg_kernel_timer_bytes(PtcgModel* M, double* bytes) {
    REQ(M && bytes, PTCG_EINVAL, "null argument");
    *bytes = M->kt.bytes;
    return PTCG_OK;
}

int ptcg_dp_unique_id(void* out) {
    REQ(out, PTCG_EINVAL, "null argument");
    REQ(!dp_unique_id(out), PTCG_ENCCL, "ptcg_dp_unique_id: %s", dp_last_error());
    return PTCG_OK;
}

int ptcg_dp_init(PtcgModel* M, const void* uid, int rank, int world) {
    REQ(M && uid, PTCG_EINVAL, "null argument");
    REQ(world >= 1 && rank >= 0 && rank < world, PTCG_EINVAL, "bad rank %d / world %d", rank, world);
    REQ(!M->dp, PTCG_ESTATE, "ptcg_dp_init: the data-parallel exchange is already on");
    CK(cudaSetDevice(M->dev));
    CK(cudaDeviceSynchronize());
    std::vector<long> sp = hook_spans(M);
    DpState* d = nullptr;
    REQ(!dp_create(&d, uid, rank, world, M->dev, sp.data(), (int)(sp.size() / 2), M->n_arena),
        PTCG_ENCCL, "ptcg_dp_init: %s", dp_last_error());
    M->dp = d;
    return PTCG_OK;
}

int ptcg_dp_weights_agree(PtcgModel* M, long long* minmax_dev, void* stream) {
    REQ(M && minmax_dev, PTCG_EINVAL, "null argument");
    REQ(M->dp, PTCG_ESTATE, "ptcg_dp_weights_agree: no data-parallel exchange (ptcg_dp_init)");
    CK(cudaSetDevice(M->dev));
    cudaStream_t s = (cudaStream_t)stream;
    CK(cudaMemsetAsync(M->d_ck, 0, 8, s));
    ++g_ptcg_launches, k_checksum<<<256, 256, 0, s>>>(M->d_ck, M->params, M->n_arena);
    CKL();
    REQ(!dp_weights_agree(M->dp, M->d_ck, minmax_dev, s), PTCG_ENCCL,
        "ptcg_dp_weights_agree: %s", dp_last_error());
    return PTCG_OK;
}

int ptcg_dp_finalize(PtcgModel* M, int abort) {
    REQ(M, PTCG_EINVAL, "null model");
    if (!M->dp) return PTCG_OK;
    CK(cudaSetDevice(M->dev));
    dp_destroy(M->dp, abort != 0);
    M->dp = nullptr;
    return PTCG_OK;
}

int ptcg_weights_checksum(PtcgModel* M, unsigned int* out_dev, void* stream) {
    REQ(M && out_dev, PTCG_EINVAL, "null argument");
    cudaStream_t s = (cudaStream_t)stream;
    CK(cudaMemsetAsync(out_dev, 0, 8, s));
    ++g_ptcg_launches, k_checksum<<<256, 256, 0, s>>>(out_dev, M->params, M->n_arena);
    CKL();
    return PTCG_OK;
}

}  // extern "C"
