// PufferLib plug-in face of the library (include/ptcg_puffer.h): the
// Encoder / Decoder / Network vtable slots that the reference's patched
// native trainer calls (native/src/models.cu:16-76, filled for "ptcg" by
// native/src/ocean.cu:5-46; the reference's implementations are
// native/model/ptcg_model4.cu:236-354), on top of the ptcg_* C-ABI.
//
// Ownership.  The trainer owns three Allocator arenas (params, grads,
// activations) and creates them after every reg_* call
// (native/src/pufferlib.cu:2609-2673).  Its optimizer (muon_step) updates
// its params arena in place and all-reduces its grads arena, so those two
// arenas hold the truth:
//  - reg_params / reg_train register the PT_PARAMS tensors into them, in the
//    reference's order and alignment;
//  - init_weights loads $PTCG_INIT_WEIGHTS into the trainer's params arena
//    (as the reference does) and copies it into the model's own master
//    weights (ptcg_import_params, which also refreshes the bf16 copies);
//  - every train forward imports the params arena again (the optimizer may
//    have stepped since), and the first rollout forward after a backward
//    does, once for all rollout buffers;
//  - backward writes the model's grads and copies them into the trainer's
//    grads arena.
// The two arenas share one layout (checked at init_weights), so each
// exchange is one device-to-device copy of the arena (c0: 28 MB, a few us).
//
// Rollout buffers get one workspace each (ptcg_workspace_create), so their
// forwards on per-buffer streams (pufferlib.cu:503-509) share nothing they
// write.  As in the reference, the trainer keeps rollout and train phases
// apart: a train step (forward, backward, optimizer) is not in flight while
// a rollout forward runs.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "ptcg_b200.h"
#include "ptcg_puffer.h"

// The env library (native/ptcg/tables.c) exports these in the reference's
// trainer process; weak, so this library also loads where they are absent.
extern "C" {
__attribute__((weak)) const float* pt_tab_card_static(void);
__attribute__((weak)) const int* pt_tab_card_attacks(void);
__attribute__((weak)) const int* pt_tab_card_skills(void);
__attribute__((weak)) const float* pt_tab_att_static(void);
__attribute__((weak)) const float* pt_tab_card_text(void);
__attribute__((weak)) const float* pt_tab_att_text(void);
__attribute__((weak)) const float* pt_tab_skill_text(void);
}

namespace {

struct Config {
    // the reference's default shape (native/model/ptcg_model.cu:14-82)
    PtcgShape shape{256, 8, 512, 4, 160, 64, 56, 1284, 1573, 448};
    int precision = PTCG_FP32;
    int device = -1;
};
Config g_cfg;
std::mutex g_cfg_mu;

struct HostTables {
    const float *card_static = nullptr, *att_static = nullptr, *card_text = nullptr,
                *att_text = nullptr, *skill_text = nullptr;
    const int *card_attacks = nullptr, *card_skills = nullptr;
};
HostTables g_tabs;
bool g_tabs_set = false;

bool g_abort = true;
thread_local char g_perr[1024];

// mb_returns of the bound TrainGraph (ptcg_bind_train_graph)
const float* g_mb_returns = nullptr;
long g_mb_returns_n = 0;

void fail(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_perr, sizeof(g_perr), fmt, ap);
    va_end(ap);
    if (g_abort) {
        fprintf(stderr, "ptcg_b200 plug-in: %s\n", g_perr);
        abort();
    }
}

long numel(const int64_t* shape) {
    long n = 1;
    bool any = false;
    for (int i = 0; i < PTCG_PUF_MAX_DIMS && shape[i] != 0; i++) {
        n *= shape[i];
        any = true;
    }
    return any ? n : 0;
}

// alloc_register_impl of native/src/kernels.cu:433-440, on the trainer's struct
void reg(PtcgPufAllocator* a, PtcgPufTensor* t) {
    a->regs = (PtcgPufAllocEntry*)realloc(a->regs, (a->num_regs + 1) * sizeof(PtcgPufAllocEntry));
    a->regs[a->num_regs++] = {(void**)&t->data, t->shape, (int)sizeof(float)};
    long n = numel(t->shape);
    a->total_elems += n;
    a->total_bytes = (a->total_bytes + 15) & ~15L;
    a->total_bytes += n * (long)sizeof(float);
}

void set_shape(PtcgPufTensor* t, long r, long c) {
    memset(t, 0, sizeof(*t));
    t->shape[0] = r;
    if (c > 0) t->shape[1] = c;
}

struct ActsImpl;

struct Weights {
    PtcgShape shape;
    int precision = PTCG_FP32, device = -1;
    int nparam = 0;
    std::vector<PtcgPufTensor> p;       // registered in the trainer's params arena
    std::vector<long> rows, cols;
    long arena_floats = 0;              // end of the last tensor, in floats
    PtcgModel* m = nullptr;
    std::vector<ActsImpl*> acts;        // every registered activation set
    std::mutex mu;
    bool stale = true;                  // trainer params may differ from the model's copy
    cudaEvent_t imported = nullptr;     // last rollout-side import
    bool imported_rec = false;
};

// Encoder activations: the trainer callocs activation_size bytes; the tensor
// registered in its activation arena must live there (the Allocator keeps
// the address of its data field), the rest is on the heap.
struct EncSlot {
    PtcgPufTensor out;                  // [rows, nopt + 1] fused [scores | value]
    ActsImpl* impl;
};

struct ActsImpl {
    Weights* w = nullptr;
    int train = 0, rows = 0;
    std::vector<PtcgPufTensor> grads;   // train: registered in the trainer's grads arena
    PtcgWorkspace* ws = nullptr;        // rollout
};

struct DecSlot {
    PtcgPufTensor grad_out;             // [B_TT, nopt + 1]
    int B_TT, nopt;
};

bool ok(int rc, const char* what) {
    if (rc == PTCG_OK) return true;
    fail("%s failed (%d): %s", what, rc, ptcg_last_error());
    return false;
}

bool cuda_ok(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return true;
    fail("%s: %s", what, cudaGetErrorString(e));
    return false;
}

// the trainer arena `t` (first tensor at t[0].data) must have the model's
// offsets for every tensor
bool same_layout(const Weights* W, const PtcgPufTensor* t, const char* which) {
    const char* base = (const char*)t[0].data;
    if (!base) {
        fail("%s arena not created (alloc_create) before init_weights", which);
        return false;
    }
    for (int i = 0; i < W->nparam; i++) {
        long want = ptcg_param_offset(W->m, i) * (long)sizeof(float);
        if ((const char*)t[i].data - base != want) {
            fail("%s arena: tensor %d at byte %ld, the model expects %ld", which, i,
                 (long)((const char*)t[i].data - base), want);
            return false;
        }
    }
    return true;
}

// ---------------------------------------------------------------- encoder
void* enc_create_weights(void* self) {
    (void)self;
    Weights* W = new Weights();
    std::lock_guard<std::mutex> lock(g_cfg_mu);
    W->shape = g_cfg.shape;
    W->precision = g_cfg.precision;
    W->device = g_cfg.device;
    W->nparam = ptcg_num_params(&W->shape);
    if (W->nparam <= 0) {
        fail("bad model shape: %s", ptcg_last_error());
        return W;
    }
    W->p.resize(W->nparam);
    W->rows.resize(W->nparam);
    W->cols.resize(W->nparam);
    for (int i = 0; i < W->nparam; i++) {
        const char* name = nullptr;
        ptcg_param_info(&W->shape, i, &name, &W->rows[i], &W->cols[i]);
    }
    return W;
}

void enc_reg_params(void* wv, PtcgPufAllocator* alloc) {
    Weights* W = (Weights*)wv;
    for (int i = 0; i < W->nparam; i++) {
        set_shape(&W->p[i], W->rows[i], W->cols[i]);
        reg(alloc, &W->p[i]);
    }
}

ActsImpl* new_acts(Weights* W, void* actv, int train, int rows) {
    EncSlot* slot = (EncSlot*)actv;
    ActsImpl* a = new ActsImpl();
    a->w = W;
    a->train = train;
    a->rows = rows;
    slot->impl = a;
    set_shape(&slot->out, rows, W->shape.nopt + 1);
    W->acts.push_back(a);
    return a;
}

void enc_reg_train(void* wv, void* actv, PtcgPufAllocator* acts, PtcgPufAllocator* grads,
                   int B_TT) {
    Weights* W = (Weights*)wv;
    ActsImpl* a = new_acts(W, actv, 1, B_TT);
    a->grads.resize(W->nparam);
    for (int i = 0; i < W->nparam; i++) {
        set_shape(&a->grads[i], W->rows[i], W->cols[i]);
        reg(grads, &a->grads[i]);
    }
    reg(acts, &((EncSlot*)actv)->out);
}

void enc_reg_rollout(void* wv, void* actv, PtcgPufAllocator* alloc, int B) {
    Weights* W = (Weights*)wv;
    new_acts(W, actv, 0, B);
    reg(alloc, &((EncSlot*)actv)->out);
}

bool set_tables(PtcgModel* m) {
    HostTables t = g_tabs;
    if (!g_tabs_set) {
        if (!pt_tab_card_static || !pt_tab_card_attacks || !pt_tab_card_skills ||
            !pt_tab_att_static || !pt_tab_card_text || !pt_tab_att_text || !pt_tab_skill_text) {
            fail("no static tables: call ptcg_puf_set_tables or link the env's pt_tab_* getters");
            return false;
        }
        t.card_static = pt_tab_card_static();
        t.card_attacks = pt_tab_card_attacks();
        t.card_skills = pt_tab_card_skills();
        t.att_static = pt_tab_att_static();
        t.card_text = pt_tab_card_text();
        t.att_text = pt_tab_att_text();
        t.skill_text = pt_tab_skill_text();
    }
    return ok(ptcg_set_tables(m, t.card_static, t.card_attacks, t.card_skills, t.att_static,
                              t.card_text, t.att_text, t.skill_text),
              "ptcg_set_tables");
}

void enc_init_weights(void* wv, unsigned long* seed, void* stream) {
    (void)seed;                          // weights come from $PTCG_INIT_WEIGHTS, as in the reference
    Weights* W = (Weights*)wv;
    int dev = W->device;
    if (dev < 0 && !cuda_ok(cudaGetDevice(&dev), "cudaGetDevice")) return;
    if (!cuda_ok(cudaSetDevice(dev), "cudaSetDevice")) return;
    if (!W->m) {
        if (!ok(ptcg_create(&W->shape, W->precision, dev, &W->m), "ptcg_create")) return;
        if (!set_tables(W->m)) return;
    }
    const int last = W->nparam - 1;
    W->arena_floats = ptcg_param_offset(W->m, last) +
                      W->rows[last] * (W->cols[last] > 0 ? W->cols[last] : 1);
    if (!same_layout(W, W->p.data(), "params")) return;
    int train_rows = 0;
    for (ActsImpl* a : W->acts) {
        if (a->train) {
            if (!same_layout(W, a->grads.data(), "grads")) return;
            train_rows = a->rows > train_rows ? a->rows : train_rows;
        } else if (!a->ws) {
            if (!ok(ptcg_workspace_create(W->m, a->rows, &a->ws), "ptcg_workspace_create")) return;
        }
    }
    if (!ok(ptcg_reserve(W->m, 0, train_rows), "ptcg_reserve")) return;
    long total = 0;
    for (int i = 0; i < W->nparam; i++) total += numel(W->p[i].shape);
    ptcg_load_init_weights_regs(W->p.data(), W->nparam, total, stream);
    if (!ok(ptcg_import_params(W->m, W->p[0].data, W->arena_floats, stream), "ptcg_import_params"))
        return;
    if (!W->imported &&
        !cuda_ok(cudaEventCreateWithFlags(&W->imported, cudaEventDisableTiming), "cudaEventCreate"))
        return;
    cuda_ok(cudaStreamSynchronize((cudaStream_t)stream), "init_weights");
    W->stale = false;
}

PtcgPufTensor enc_forward(void* wv, void* actv, PtcgPufTensor input, void* stream) {
    Weights* W = (Weights*)wv;
    EncSlot* slot = (EncSlot*)actv;
    ActsImpl* a = slot->impl;
    PtcgPufTensor out = slot->out;
    const int n = (int)input.shape[0];
    out.shape[0] = n;
    if (!W->m) {
        fail("forward before init_weights");
        return out;
    }
    if (a->train) {
        // the trainer's optimizer may have stepped its params since the last call
        if (!ok(ptcg_import_params(W->m, W->p[0].data, W->arena_floats, stream),
                "ptcg_import_params"))
            return out;
        ok(ptcg_forward_train(W->m, input.data, n, slot->out.data, stream), "ptcg_forward_train");
        return out;
    }
    {
        std::lock_guard<std::mutex> lock(W->mu);
        if (W->stale) {
            if (!ok(ptcg_import_params(W->m, W->p[0].data, W->arena_floats, stream),
                    "ptcg_import_params") ||
                !cuda_ok(cudaEventRecord(W->imported, (cudaStream_t)stream), "cudaEventRecord"))
                return out;
            W->imported_rec = true;
            W->stale = false;
        } else if (W->imported_rec &&
                   !cuda_ok(cudaStreamWaitEvent((cudaStream_t)stream, W->imported, 0),
                            "cudaStreamWaitEvent")) {
            return out;
        }
    }
    ok(ptcg_forward_ws(W->m, a->ws, input.data, n, slot->out.data, stream), "ptcg_forward_ws");
    return out;
}

void enc_backward(void* wv, void* actv, PtcgPufTensor grad, void* stream) {
    Weights* W = (Weights*)wv;
    ActsImpl* a = ((EncSlot*)actv)->impl;
    if (!a->train) {
        fail("backward on rollout activations");
        return;
    }
    if (!g_mb_returns) {
        fail("backward needs mb_returns: call ptcg_bind_train_graph after alloc_create");
        return;
    }
    // zeroes the grad arena first, like ptcg_backward_core (ptcg_model4.cu:15-21)
    if (!ok(ptcg_backward(W->m, grad.data, g_mb_returns, 0, 0.f, 0, stream), "ptcg_backward"))
        return;
    float* g = nullptr;
    long ng = 0;
    if (!ok(ptcg_arena(W->m, 1, &g, &ng), "ptcg_arena")) return;
    if (!cuda_ok(cudaMemcpyAsync(a->grads[0].data, g, (size_t)W->arena_floats * sizeof(float),
                                 cudaMemcpyDeviceToDevice, (cudaStream_t)stream),
                 "grad export"))
        return;
    std::lock_guard<std::mutex> lock(W->mu);
    W->stale = true;                     // an optimizer step on the trainer's params follows
}

void enc_free_weights(void* wv) {
    Weights* W = (Weights*)wv;
    if (!W) return;
    if (W->imported) cudaEventDestroy(W->imported);
    if (W->m) ptcg_destroy(W->m);
    delete W;
}

void enc_free_activations(void* actv) {
    EncSlot* slot = (EncSlot*)actv;
    if (!slot) return;
    ActsImpl* a = slot->impl;
    if (a) {
        Weights* W = a->w;
        if (a->ws) ptcg_workspace_destroy(a->ws);
        if (W) {
            for (size_t i = 0; i < W->acts.size(); i++)
                if (W->acts[i] == a) { W->acts.erase(W->acts.begin() + i); break; }
        }
        delete a;
    }
    free(actv);
}

// ---------------------------------------------------------------- decoder
// passthrough forward; backward assembles [grad_logits | grad_value]
// (ptcg_model4.cu:286-306)
__global__ void k_assemble_dec_grad(float* dst, const float* gl, const float* gv, int rows,
                                    int nopt) {
    const int od = nopt + 1;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < (long)rows * od;
         i += (long)gridDim.x * blockDim.x) {
        long r = i / od;
        int c = (int)(i - r * od);
        dst[i] = c < nopt ? gl[r * nopt + c] : gv[r];
    }
}

PtcgPufTensor dec_forward(void* w, void* actv, PtcgPufTensor input, void* stream) {
    (void)w; (void)actv; (void)stream;
    return input;
}

PtcgPufTensor dec_backward(void* w, void* actv, PtcgPufTensor grad_logits,
                           PtcgPufTensor grad_logstd, PtcgPufTensor grad_value, void* stream) {
    (void)w; (void)grad_logstd;
    DecSlot* a = (DecSlot*)actv;
    int rows = a->B_TT;
    if (grad_logits.shape[0] > 0 && grad_logits.shape[0] < rows) rows = (int)grad_logits.shape[0];
    if (grad_logits.shape[1] != 0 && grad_logits.shape[1] != a->nopt) {
        fail("decoder backward: grad_logits has %ld columns, the model scores %d options",
             (long)grad_logits.shape[1], a->nopt);
        return a->grad_out;
    }
    long n = (long)rows * (a->nopt + 1);
    int blocks = (int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
    if (blocks > 0)
        k_assemble_dec_grad<<<blocks, 256, 0, (cudaStream_t)stream>>>(
            a->grad_out.data, grad_logits.data, grad_value.data, rows, a->nopt);
    cuda_ok(cudaGetLastError(), "decoder backward launch");
    return a->grad_out;
}

void dec_reg_train(void* w, void* actv, PtcgPufAllocator* acts, PtcgPufAllocator* grads,
                   int B_TT) {
    (void)w; (void)grads;
    DecSlot* a = (DecSlot*)actv;
    {
        std::lock_guard<std::mutex> lock(g_cfg_mu);
        a->nopt = g_cfg.shape.nopt;
    }
    a->B_TT = B_TT;
    set_shape(&a->grad_out, B_TT, a->nopt + 1);
    reg(acts, &a->grad_out);
}

void noop_init(void* w, unsigned long* seed, void* s) { (void)w; (void)seed; (void)s; }
void noop_reg_params(void* w, PtcgPufAllocator* a) { (void)w; (void)a; }
void noop_reg_train(void* w, void* actv, PtcgPufAllocator* acts, PtcgPufAllocator* grads,
                    int B_TT) {
    (void)w; (void)actv; (void)acts; (void)grads; (void)B_TT;
}
void noop_reg_rollout(void* w, void* actv, PtcgPufAllocator* a, int B) {
    (void)w; (void)actv; (void)a; (void)B;
}
void* small_create(void* self) { (void)self; return calloc(1, 8); }
void plain_free(void* p) { free(p); }

// ---------------------------------------------------------------- network
// identity: the policy is stateless (MinGRU bypassed, native/PATCHES.md:19-26)
PtcgPufTensor net_forward(void* w, PtcgPufTensor x, PtcgPufTensor state, void* actv, void* s) {
    (void)w; (void)state; (void)actv; (void)s;
    return x;
}
PtcgPufTensor net_backward(void* w, PtcgPufTensor grad, void* actv, void* s) {
    (void)w; (void)actv; (void)s;
    return grad;
}

}  // namespace

extern "C" {

int ptcg_puf_configure(const PtcgShape* shape, int precision, int device) {
    if (shape && ptcg_obs_size(shape) < 0) return PTCG_EINVAL;
    if (precision != PTCG_FP32 && precision != PTCG_BF16) return PTCG_EINVAL;
    std::lock_guard<std::mutex> lock(g_cfg_mu);
    if (shape) g_cfg.shape = *shape;
    g_cfg.precision = precision;
    g_cfg.device = device;
    return PTCG_OK;
}

int ptcg_puf_set_tables(const float* card_static, const int* card_attacks,
                        const int* card_skills, const float* att_static,
                        const float* card_text, const float* att_text,
                        const float* skill_text) {
    if (!card_static || !card_attacks || !card_skills || !att_static || !card_text ||
        !att_text || !skill_text)
        return PTCG_EINVAL;
    g_tabs = HostTables{card_static, att_static, card_text, att_text, skill_text, card_attacks,
                        card_skills};
    g_tabs_set = true;
    return PTCG_OK;
}

void ptcg_puf_fill_encoder(PtcgPufEncoder* enc) {
    enc->forward = enc_forward;
    enc->backward = enc_backward;
    enc->init_weights = enc_init_weights;
    enc->reg_params = enc_reg_params;
    enc->reg_train = enc_reg_train;
    enc->reg_rollout = enc_reg_rollout;
    enc->create_weights = enc_create_weights;
    enc->free_weights = enc_free_weights;
    enc->free_activations = enc_free_activations;
    enc->activation_size = sizeof(EncSlot);
}

void ptcg_puf_fill_decoder(PtcgPufDecoder* dec) {
    dec->forward = dec_forward;
    dec->backward = dec_backward;
    dec->init_weights = noop_init;
    dec->reg_params = noop_reg_params;
    dec->reg_train = dec_reg_train;
    dec->reg_rollout = noop_reg_rollout;
    dec->create_weights = small_create;
    dec->free_weights = plain_free;
    dec->free_activations = plain_free;
    dec->activation_size = (int)sizeof(DecSlot);
}

void ptcg_puf_fill_network(PtcgPufNetwork* net) {
    net->forward = net_forward;
    net->forward_train = net_forward;
    net->backward = net_backward;
    net->init_weights = noop_init;
    net->reg_params = noop_reg_params;
    net->reg_train = noop_reg_train;
    net->reg_rollout = noop_reg_rollout;
    net->create_weights = small_create;
    net->free_weights = plain_free;
    net->free_activations = plain_free;
}

PtcgModel* ptcg_puf_model(void* weights) {
    return weights ? ((Weights*)weights)->m : nullptr;
}

void ptcg_puf_set_abort(int abort_on_error) { g_abort = abort_on_error != 0; }

const char* ptcg_puf_last_error(void) { return g_perr; }

void ptcg_puff_advantage(PtcgPufTensor* values, PtcgPufTensor* rewards, PtcgPufTensor* dones,
                         PtcgPufTensor* importance, PtcgPufTensor* obs,
                         PtcgPufTensor* advantages, float gamma, float lambda, float rho_clip,
                         float c_clip, void* stream) {
    PtcgShape shape;
    {
        std::lock_guard<std::mutex> lock(g_cfg_mu);
        shape = g_cfg.shape;
    }
    const int B = (int)values->shape[0], T = (int)values->shape[1];
    long obs_size = ptcg_obs_size(&shape);
    // (B, T, obs) or (B * T, obs): the row width is the last dimension
    long last = 0;
    for (int i = 0; i < PTCG_PUF_MAX_DIMS && obs->shape[i] != 0; i++) last = obs->shape[i];
    if (last != obs_size) {
        fail("ptcg_puff_advantage: observation rows of %ld floats, the configured shape has %ld",
             last, obs_size);
        return;
    }
    ok(ptcg_negamax_advantage(values->data, rewards->data, dones->data, importance->data,
                              obs->data, obs_size, (int)ptcg_seat_column(&shape), B, T, gamma,
                              lambda, rho_clip, c_clip, advantages->data, stream),
       "ptcg_negamax_advantage");
}

void ptcg_bind_train_graph(void* train_buf_ptr) {
    // TrainGraph is a struct of PrecisionTensors; member 6 is mb_returns
    // (native/src/pufferlib.cu:116-129)
    const PtcgPufTensor* t = (const PtcgPufTensor*)train_buf_ptr;
    g_mb_returns = t[6].data;
    g_mb_returns_n = numel(t[6].shape);
}

void ptcg_load_init_weights_regs(PtcgPufTensor* p, int n_params, long n_total, void* stream) {
    const char* path = getenv("PTCG_INIT_WEIGHTS");
    if (!path) {
        fail("PTCG_INIT_WEIGHTS not set: refusing random init (the torch-matching init is required)");
        return;
    }
    FILE* f = fopen(path, "rb");
    if (!f) {
        fail("cannot open %s", path);
        return;
    }
    fseek(f, 0, SEEK_END);
    long bytes = ftell(f);
    fseek(f, 0, SEEK_SET);
    if (bytes != n_total * (long)sizeof(float)) {
        fclose(f);
        fail("%s has %ld bytes, expected %ld", path, bytes, n_total * (long)sizeof(float));
        return;
    }
    std::vector<float> host((size_t)n_total);
    size_t got = fread(host.data(), 1, (size_t)bytes, f);
    fclose(f);
    if (got != (size_t)bytes) {
        fail("short read of %s", path);
        return;
    }
    long off = 0;
    for (int i = 0; i < n_params; i++) {
        long ne = numel(p[i].shape);
        if (off + ne > n_total) {
            fail("registered tensors hold more than the blob's %ld floats", n_total);
            return;
        }
        if (!cuda_ok(cudaMemcpyAsync(p[i].data, host.data() + off, ne * sizeof(float),
                                     cudaMemcpyHostToDevice, (cudaStream_t)stream),
                     "weight upload"))
            return;
        off += ne;
    }
    if (!cuda_ok(cudaStreamSynchronize((cudaStream_t)stream), "weight upload")) return;
    if (off != n_total) fail("consumed %ld of %ld blob floats", off, n_total);
}

}  // extern "C"
