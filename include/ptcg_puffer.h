/*
 * ptcg_puffer.h -- the PufferLib plug-in face of libptcg_b200.so.
 *
 * The reference's patched PufferLib native trainer calls its policy through
 * three structs of C function pointers, Encoder / Decoder / Network
 * (native/src/models.cu:16-76), which native/src/ocean.cu:5-46 fills for the
 * "ptcg" env, plus three extern "C" functions of native/model
 * (ptcg_model2.cu:313-330, ptcg_model4.cu:196-233).  This header restates
 * those types with the same memory layout (the reference's fp32 build,
 * -DPRECISION_FLOAT, native/build_native.sh:88), and declares:
 *
 *  - ptcg_puf_fill_encoder / _decoder / _network: fill the trainer's structs
 *    with this library's implementations (the body of the replacement
 *    create_custom_encoder / _decoder / _network);
 *  - ptcg_puff_advantage, ptcg_bind_train_graph and
 *    ptcg_load_init_weights_regs with the reference's exact names and
 *    signatures.
 *
 * Layout notes (why these types match the trainer's):
 *  - PtcgPufTensor = PrecisionTensor / FloatTensor of native/src/tensor.h:7-45
 *    (data pointer + int64 shape[8]; precision_t = float in the fp32 build);
 *  - PtcgPufAllocator / PtcgPufAllocEntry = Allocator / AllocEntry of
 *    native/src/kernels.cu:412-424.  Registration follows alloc_register_impl
 *    (:433-440): entries appended with realloc, total_bytes advanced to the
 *    next 16-byte boundary before each tensor;
 *  - the vtable structs list the same members in the same order as
 *    Encoder / Decoder / Network; cudaStream_t is passed as void*.
 *
 * Errors: the vtable slots return void like the reference's, so a failure
 * prints a message to stderr and aborts, as the reference does
 * (ptcg_model4.cu:199-230).  ptcg_puf_set_abort(0) makes failures return
 * instead (leaving outputs unwritten) with the message in
 * ptcg_puf_last_error(), for embedding in a process that must not abort.
 */
#ifndef PTCG_PUFFER_H
#define PTCG_PUFFER_H

#include <stdint.h>

#include "ptcg_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

#define PTCG_PUF_MAX_DIMS 8

#ifdef __cplusplus
#define PTCG_PUF_BOOL bool
#else
#define PTCG_PUF_BOOL _Bool
#endif

/* A translation unit that already has the trainer's own types (the
 * replacement ocean.cu, compiled inside pufferlib.cu) defines
 * PTCG_PUF_TENSOR to PrecisionTensor and PTCG_PUF_ALLOCATOR to Allocator
 * before including this header, so that the trainer's calls to
 * ptcg_puff_advantage / ptcg_bind_train_graph type-check unchanged. */
#ifdef PTCG_PUF_TENSOR
typedef PTCG_PUF_TENSOR PtcgPufTensor;
#else
typedef struct PtcgPufTensor {
    float* data;
    int64_t shape[PTCG_PUF_MAX_DIMS];
} PtcgPufTensor;
#endif

#ifdef PTCG_PUF_ALLOCATOR
typedef PTCG_PUF_ALLOCATOR PtcgPufAllocator;
#else
typedef struct PtcgPufAllocEntry {
    void** data_ptr;
    int64_t* shape;
    int elem_size;
} PtcgPufAllocEntry;

typedef struct PtcgPufAllocator {
    PtcgPufAllocEntry* regs;
    int num_regs;
    void* mem;
    long total_elems;
    long total_bytes;
} PtcgPufAllocator;
#endif

typedef void (*ptcg_puf_init_weights_fn)(void* weights, unsigned long* seed, void* stream);
typedef void (*ptcg_puf_reg_params_fn)(void* weights, PtcgPufAllocator* alloc);
typedef void (*ptcg_puf_reg_train_fn)(void* weights, void* acts, PtcgPufAllocator* act_alloc,
                                      PtcgPufAllocator* grad_alloc, int B_TT);
typedef void (*ptcg_puf_reg_rollout_fn)(void* weights, void* acts, PtcgPufAllocator* alloc,
                                        int B);
typedef void* (*ptcg_puf_create_weights_fn)(void* self);
typedef void (*ptcg_puf_free_fn)(void* p);
typedef PtcgPufTensor (*ptcg_puf_forward_fn)(void* weights, void* acts, PtcgPufTensor input,
                                             void* stream);
typedef void (*ptcg_puf_enc_backward_fn)(void* weights, void* acts, PtcgPufTensor grad,
                                         void* stream);
typedef PtcgPufTensor (*ptcg_puf_dec_backward_fn)(void* weights, void* acts,
                                                  PtcgPufTensor grad_logits,
                                                  PtcgPufTensor grad_logstd,
                                                  PtcgPufTensor grad_value, void* stream);
typedef PtcgPufTensor (*ptcg_puf_net_forward_fn)(void* weights, PtcgPufTensor x,
                                                 PtcgPufTensor state, void* acts, void* stream);
typedef PtcgPufTensor (*ptcg_puf_net_backward_fn)(void* weights, PtcgPufTensor grad,
                                                  void* acts, void* stream);

/* struct Encoder, native/src/models.cu:35-47 */
typedef struct PtcgPufEncoder {
    ptcg_puf_forward_fn forward;
    ptcg_puf_enc_backward_fn backward;
    ptcg_puf_init_weights_fn init_weights;
    ptcg_puf_reg_params_fn reg_params;
    ptcg_puf_reg_train_fn reg_train;
    ptcg_puf_reg_rollout_fn reg_rollout;
    ptcg_puf_create_weights_fn create_weights;
    ptcg_puf_free_fn free_weights;
    ptcg_puf_free_fn free_activations;
    int in_dim, out_dim;
    size_t activation_size;
} PtcgPufEncoder;

/* struct Decoder, native/src/models.cu:49-62 */
typedef struct PtcgPufDecoder {
    ptcg_puf_forward_fn forward;
    ptcg_puf_dec_backward_fn backward;
    ptcg_puf_init_weights_fn init_weights;
    ptcg_puf_reg_params_fn reg_params;
    ptcg_puf_reg_train_fn reg_train;
    ptcg_puf_reg_rollout_fn reg_rollout;
    ptcg_puf_create_weights_fn create_weights;
    ptcg_puf_free_fn free_weights;
    ptcg_puf_free_fn free_activations;
    int hidden_dim, output_dim;
    PTCG_PUF_BOOL continuous;
    int activation_size;
} PtcgPufDecoder;

/* struct Network, native/src/models.cu:64-76 */
typedef struct PtcgPufNetwork {
    ptcg_puf_net_forward_fn forward;
    ptcg_puf_net_forward_fn forward_train;
    ptcg_puf_net_backward_fn backward;
    ptcg_puf_init_weights_fn init_weights;
    ptcg_puf_reg_params_fn reg_params;
    ptcg_puf_reg_train_fn reg_train;
    ptcg_puf_reg_rollout_fn reg_rollout;
    ptcg_puf_create_weights_fn create_weights;
    ptcg_puf_free_fn free_weights;
    ptcg_puf_free_fn free_activations;
    int hidden, num_layers, horizon;
} PtcgPufNetwork;

/* Model configuration for the weights created after this call (the
 * reference fixes these at compile time, native/model/ptcg_model.cu:14-82).
 * shape NULL keeps the current one.  Default: the reference's default shape
 * (d256, 4 layers, 8 heads, FFN 512, 160 tokens, 64 options), PTCG_FP32
 * (the reference's own precision), device = the current device when the
 * weights are created.  Returns a PTCG_E* code. */
int ptcg_puf_configure(const PtcgShape* shape, int precision, int device);

/* Host copies of the static tables (layouts as ptcg_set_tables).  Without
 * this call, init_weights takes them from the env's pt_tab_* getters
 * (native/ptcg/tables.c, imported as in native/model/ptcg_model2.cu:390-398)
 * when the process provides them.  The pointers must stay valid until the
 * next init_weights. */
int ptcg_puf_set_tables(const float* card_static, const int* card_attacks,
                        const int* card_skills, const float* att_static,
                        const float* card_text, const float* att_text,
                        const float* skill_text);

/* Fill the trainer's vtable structs (pointers to the structs of
 * native/src/models.cu).  Only the function pointers and
 * activation_size are written; the dims stay as build_policy set them
 * (native/src/pufferlib.cu:2192-2242). */
void ptcg_puf_fill_encoder(PtcgPufEncoder* enc);
void ptcg_puf_fill_decoder(PtcgPufDecoder* dec);
void ptcg_puf_fill_network(PtcgPufNetwork* net);

/* The PtcgModel behind a weights pointer from create_weights (NULL before
 * init_weights), for callers that mix the vtable path with ptcg_* calls. */
PtcgModel* ptcg_puf_model(void* weights);

/* Failure handling of the vtable slots: abort (1, the default, as the
 * reference) or record and return (0). */
void ptcg_puf_set_abort(int abort_on_error);
const char* ptcg_puf_last_error(void);

/* ---- the reference's extern "C" exports, same names and signatures ------ */

/* Seat-flipping GAE / V-trace over (B, T) = values->shape rollouts, seats
 * from the observation rows (obs->shape = (B, T, obs_size)), written to
 * advantages.  native/model/ptcg_model2.cu:313-321, called from
 * native/src/pufferlib.cu:1969-1973 under PTCG_NATIVE. */
void ptcg_puff_advantage(PtcgPufTensor* values, PtcgPufTensor* rewards, PtcgPufTensor* dones,
                         PtcgPufTensor* importance, PtcgPufTensor* obs,
                         PtcgPufTensor* advantages, float gamma, float lambda, float rho_clip,
                         float c_clip, void* stream);

/* Binds the trainer's TrainGraph (native/src/pufferlib.cu:116-129): member 6,
 * mb_returns, feeds the blind-V aux loss of the next backward calls.
 * native/model/ptcg_model2.cu:323-330, called at pufferlib.cu:2676-2678. */
void ptcg_bind_train_graph(void* train_buf_ptr);

/* Loads the packed fp32 blob named by $PTCG_INIT_WEIGHTS into the n_params
 * registered tensors p[] (n_total floats in all), on `stream`; aborts when
 * the variable is unset, the file is missing or its size differs, as
 * native/model/ptcg_model4.cu:196-233 does. */
void ptcg_load_init_weights_regs(PtcgPufTensor* p, int n_params, long n_total, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PTCG_PUFFER_H */
