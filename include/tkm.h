/*
 * tkm.h -- public C API of the Tokamak engine, as implemented by tokamak_b200's
 * host runtime (libtkm.so) on B200 (sm_100a).
 *
 * Binary compatible with the reference's include/tkm.h (BSODsystem32/Tokamak
 * v4.1.0): identical capacities, enum values, struct layouts and function
 * signatures, so callers built against the reference link against libtkm.so
 * unchanged.  Additions at the end (tkm_*_ex, tkm_runtime_step_i32 ...) are
 * new entry points; no existing signature changed.
 */
#ifndef TKM_H
#define TKM_H

#include <stddef.h>
#include <stdint.h>
#include <stdio.h>

#if defined(_WIN32) && defined(TKM_BUILD_DLL)
#define TKM_API __declspec(dllexport)
#elif defined(_WIN32) && defined(TKM_USE_DLL)
#define TKM_API __declspec(dllimport)
#else
#define TKM_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* capacities (part of the ABI: they size the structs below) */
#define TKM_MAX_NODES   1024
#define TKM_MAX_GROUPS  256
#define TKM_MAX_BUFFERS 512
#define TKM_MAX_CHAIN   8
#define TKM_MAX_KARGS   28
#define TKM_MAX_TENSORS 512

/* pseudo-random generators available to stochastic operators */
typedef enum { RNG_DEFAULT = 0, RNG_XORSHIFT32, RNG_WANG_XORSHIFT32, RNG_PCG32, RNG_PHILOX } TkmRngType;

/* per-operator resources the runtime allocates and binds to generated kernels */
typedef enum {
    RES_NONE = 0,
    RES_PARAM_BIAS = 1 << 0,   /* learnable per-channel bias            */
    RES_PARAM_WEIGHT = 1 << 1, /* learnable per-channel gain            */
    RES_PARAM_BETA = 1 << 2,   /* learnable per-channel shift           */
    RES_SAVE_ISTD = 1 << 3,    /* per-row inverse std saved for backward */
    RES_SAVE_XHAT = 1 << 4,    /* normalized activations saved          */
    RES_SAVE_MASK = 1 << 5,    /* dropout / pooling mask saved          */
    RES_RNG_SEED = 1 << 6,     /* reads the per-step seed               */
    RES_BRANCH_IN = 1 << 7,    /* second input (residual branch)        */
    RES_AUG_PIXEL = 1 << 8,
    RES_AUG_COLOR = 1 << 9
} TkmResourceFlags;

typedef enum { CAT_META = 0, CAT_ANCHOR, CAT_SPATIAL, CAT_COORD, CAT_NORM, CAT_FLUID } TkmOpCat;

typedef enum {
    OP_NONE = 0,
    OP_INPUT,
    OP_CONV, OP_FC, OP_FC_TWIN_FUSED, OP_FC_QKV_FUSED, OP_GQA_ATTN,
    OP_MIXPOOL, OP_AVGPOOL, OP_FLATTEN,
    OP_BORDER_REFLECT,
    OP_RAND_SHIFT, OP_RAND_ROTATE, OP_RAND_SCALE, OP_RAND_FLIPX, OP_RAND_FLIPY,
    OP_RAND_ELASTIC, OP_RAND_NOISE, OP_RAND_CUTOUT, OP_RAND_BRIGHTNESS, OP_RAND_CONTRAST,
    OP_RAND_SATURATION, OP_RAND_HUE, OP_RAND_GRAYSCALE, OP_RAND_CHANNEL_SCALE,
    OP_RAND_SOLARIZE, OP_RAND_ERASING,
    OP_BN, OP_LN, OP_RMSNORM, OP_L2NORM, OP_QKNORM,
    OP_BIAS, OP_SILU, OP_RELU, OP_RELU2, OP_LEAKY_RELU, OP_ELU,
    OP_GELU, OP_MISH, OP_HARDSWISH, OP_HARDSIGMOID, OP_TANH, OP_SIGMOID,
    OP_SWISH_BETA, OP_SIN, OP_COSGATE, OP_SOFTCAP, OP_CLAMP,
    OP_SCALE, OP_LAYERSCALE, OP_DYT, OP_PRELU, OP_XATLU,
    OP_ROPE, OP_DROP, OP_ADD, OP_MUL,
    OP_SOFTMAX, OP_SOFTMAX_CE, OP_SOFTMAX_FOCAL, OP_SOFTMAX_MSE,
    OP_USER_FLUID,
    OP_COUNT
} TkmOpType;

/* One registry entry: DSL name, category, resources, default scalar, and the
 * per-channel-pair forward/backward bodies as CUDA snippets or as scalar
 * formulas in x and fval (one of the two per direction). */
typedef struct {
    TkmOpType op;
    const char *dsl_name;
    TkmOpCat cat;
    uint32_t res_flags;
    float default_fval;
    const char *fwd_cuda;
    const char *bwd_cuda;
    const char *fwd_expr;
    const char *bwd_expr;
} TkmOpSpec;

typedef enum {
    KARG_IN_MAIN = 0, KARG_OUT_MAIN, KARG_DOUT_MAIN, KARG_DIN_MAIN,
    KARG_BRANCH_IN, KARG_DBRANCH_OUT,
    KARG_BIAS, KARG_DBIAS, KARG_WEIGHT_VEC, KARG_DWEIGHT_VEC, KARG_BETA, KARG_DBETA,
    KARG_SAVE_ISTD, KARG_SAVE_XHAT, KARG_SAVE_MASK, KARG_STEP_SEED
} TkmArgKind;

typedef struct {
    TkmArgKind kind;
    int node_id;
    char c_type[32];
    char c_name[32];
} TkmKernelArg;

/* ABI of one generated kernel: name, ordered arguments, launch shape */
typedef struct {
    char func_name[64];
    TkmKernelArg args[TKM_MAX_KARGS];
    int num_args;
    int grid_x, block_x;
} TkmKernelSig;

typedef struct {
    int id;
    int spec_id;
    char tag[32];
    TkmOpType op;
    TkmOpCat cat;
    int dead;

    int in0, in1, in2;
    int users;
    int plasma_grp;

    int c_out, k, s, p;
    int q_c, k_c, v_c;
    int q_heads, kv_heads, head_dim;
    int has_qknorm, has_rope, causal;
    int qkv_prep_nid;
    float fval;
    float fval2;
    float rope_theta, rope_scale, rope_low_freq_factor, rope_high_freq_factor;
    float rope_original_context_length;
    TkmRngType rng_type;

    int left_nodes[TKM_MAX_CHAIN];
    int left_len;
    int right_nodes[TKM_MAX_CHAIN];
    int right_len;

    int H, W, C;
    int out_buf_id;
    size_t out_offset, out_bytes;
} TkmNode;

/* a fused chain of row-wise operators executed by one generated kernel pair */
typedef struct {
    int id;
    int anchor_id;
    int node_ids[16];
    int count;
    int has_norm;
    int is_twin_epilogue;
    int is_coord_group;
    int is_qkv_prep;
    int use_reflect_border;
    int out_node_id;
    int H, W, C;
    TkmKernelSig fwd_sig;
    TkmKernelSig bwd_sig;
} PlasmaGroup;

typedef struct TkmGraph {
    TkmNode nodes[TKM_MAX_NODES];
    int num_nodes;
    PlasmaGroup groups[TKM_MAX_GROUPS];
    int num_groups;
    int batch_size;
    TkmRngType default_rng;
    size_t total_arena_bytes;
    size_t naive_arena_bytes;
} TkmGraph;

typedef struct {
    const char *name;
    int (*match)(const TkmGraph *g, int node_id);
    void (*apply)(TkmGraph *g, int node_id);
} TkmFusionRule;

/* registry */
const TkmOpSpec *tkm_find_spec_by_op(TkmOpType op);
const TkmOpSpec *tkm_find_spec_by_name(const char *dsl_name);
const TkmOpSpec *tkm_find_spec_by_index(int index);
const TkmOpSpec *tkm_find_spec_by_node(const TkmNode *node);
int tkm_get_spec_index(const TkmOpSpec *spec);
int tkm_get_spec_count(void);
int tkm_eval_math_expr(const char *expr, float x, float fval, float *out_value);
const TkmFusionRule *tkm_get_fusion_rules(int *out_count);
const char *tkm_rng_name(TkmRngType r);
const char *tkm_rng_struct_name(TkmRngType r);
TkmRngType tkm_parse_rng_name(const char *s);

/* compiler */
TKM_API int tkm_verify_registry(void);
TKM_API void tkm_parse_dsl(TkmGraph *g, const char *dsl_text, int batch_size);
TKM_API void tkm_infer_shapes(TkmGraph *g);
TKM_API void tkm_optimize_and_bind(TkmGraph *g);
TKM_API void tkm_plan_memory(TkmGraph *g);
TKM_API void tkm_dump_summary(const TkmGraph *g, FILE *out);
TKM_API char *tkm_codegen_cuda_string(const TkmGraph *g);

/* runtime */
typedef struct TkmRuntime TkmRuntime;
typedef struct TkmDataset TkmDataset;

/* Fills up to `capacity` samples; returns > 0 for a batch, 0 at the end, < 0
 * on error.  Training loaders return exactly the batch size. */
typedef int (*TkmDatasetNext)(void *user, float *h_input, uint8_t *h_labels, size_t capacity,
                              size_t *out_count);

TKM_API TkmRuntime *tkm_runtime_ignite(const TkmGraph *g, const char *cuda_src);
TKM_API TkmRuntime *tkm_runtime_ignite_inference(const TkmGraph *g, const char *cuda_src);
TKM_API TkmRuntime *tkm_load_file(const char *tkm_path, int batch_size);
TKM_API TkmRuntime *tkm_load_string(const char *dsl_text, int batch_size);
TKM_API TkmRuntime *tkm_load_buffer(const char *dsl_data, size_t dsl_size, int batch_size);
TKM_API float tkm_runtime_step(TkmRuntime *rt, const float *h_input, const uint8_t *h_labels, float lr);
TKM_API int tkm_runtime_eval(TkmRuntime *rt, const float *h_input, const uint8_t *h_labels, int count);
TKM_API size_t tkm_runtime_forward(TkmRuntime *rt, const float *h_input, float *h_output, size_t output_capacity);
TKM_API size_t tkm_runtime_input_elements(const TkmRuntime *rt);
TKM_API size_t tkm_runtime_output_elements(const TkmRuntime *rt);
TKM_API size_t tkm_runtime_weight_bytes(const TkmRuntime *rt);
TKM_API int tkm_runtime_train_dataset(TkmRuntime *rt, TkmDatasetNext next_batch, void *user,
                                      size_t max_batches, float lr, float *out_average_loss);
TKM_API TkmDataset *tkm_dataset_create(TkmRuntime *rt, const float *h_images, const uint8_t *h_labels,
                                       size_t num_samples);
TKM_API void tkm_dataset_free(TkmDataset *ds);
TKM_API int tkm_dataset_is_resident(const TkmDataset *ds);
TKM_API int tkm_runtime_train_epoch(TkmRuntime *rt, TkmDataset *ds, const uint32_t *h_order, float peak_lr,
                                    float min_lr_ratio, size_t global_step_start, size_t total_steps,
                                    size_t warmup_steps, float *out_average_loss);
TKM_API int tkm_runtime_eval_dataset(TkmRuntime *rt, TkmDatasetNext next_batch, void *user, size_t max_batches,
                                     int *out_correct, size_t *out_samples);
TKM_API int tkm_save_weights(TkmRuntime *rt, const char *bin_path);
TKM_API int tkm_load_weights(TkmRuntime *rt, const char *bin_path);
TKM_API int tkm_save_weights_buffer(TkmRuntime *rt, void *buffer, size_t capacity, size_t *out_size);
TKM_API int tkm_load_weights_buffer(TkmRuntime *rt, const void *buffer, size_t size);
TKM_API void tkm_runtime_free(TkmRuntime *rt);

/* finite-difference gradient probes */
TKM_API float tkm_get_grad_sample(TkmRuntime *rt, int node_id, int elem_idx);
TKM_API void tkm_perturb_tensor(TkmRuntime *rt, int node_id, int elem_idx, float delta);
TKM_API float tkm_eval_current_loss(TkmRuntime *rt);

/* ---------------------------------------------------------------- additions
 * Not in the reference API (no counterpart there). */

/* Storage type of activations: TKM_DTYPE_BF16 (default) or TKM_DTYPE_F32
 * (the fp32 mode).  Parameters are fp32 masters in both. */
#define TKM_DTYPE_F32 0
#define TKM_DTYPE_BF16 1
TKM_API TkmRuntime *tkm_runtime_ignite_ex(const TkmGraph *g, const char *cuda_src, int training, int dtype);
TKM_API TkmRuntime *tkm_load_string_ex(const char *dsl_text, int batch_size, int dtype);
/* One training step with one int32 label per output row (B*H*W of the loss
 * node's input), for sequence models and vocabularies above 256. */
TKM_API float tkm_runtime_step_i32(TkmRuntime *rt, const float *h_input, const int32_t *h_labels, float lr);
/* Copies d(loss)/d(input) of the last step (fp32, tkm_runtime_input_elements
 * values) to the host; returns the element count or 0. */
TKM_API size_t tkm_runtime_input_grad(TkmRuntime *rt, float *h_grad, size_t capacity);
/* Output rows of the node feeding the loss (logits), fp32, from the last step. */
TKM_API size_t tkm_runtime_logits(TkmRuntime *rt, float *h_out, size_t capacity);
/* Gradient of one learnable tensor (registration order) from the last step. */
TKM_API size_t tkm_runtime_param_grad(TkmRuntime *rt, int tensor_index, float *h_out, size_t capacity);
TKM_API int tkm_runtime_param_count(const TkmRuntime *rt);
/* Last error message of the runtime (empty when none). */
TKM_API const char *tkm_last_error(void);

/* SGD momentum state, beside the TKM1 weight checkpoint: magic "TKMV", tensor
 * count, then per tensor (TKM1 order) its value count and fp32 velocities; a
 * tensor the step does not update (dead node) has 0 values.  Saving both and
 * loading both resumes training exactly where it stopped. */
TKM_API size_t tkm_runtime_optimizer_bytes(const TkmRuntime *rt);
TKM_API int tkm_save_optimizer_buffer(TkmRuntime *rt, void *buffer, size_t capacity, size_t *out_size);
TKM_API int tkm_load_optimizer_buffer(TkmRuntime *rt, const void *buffer, size_t size);

/* Data-parallel training over NCCL: rank 0 creates a 128-byte NCCL unique id,
 * the caller sends it to every rank (any transport), then each rank calls
 * tkm_runtime_init_dp before its first step.  Every step then averages the
 * gradients of all ranks with one all-reduce inside the captured step graph
 * before the SGD update (a world of one rank runs the same exchange, an
 * identity).  Returns 1 on success. */
TKM_API int tkm_nccl_unique_id(void *out128);
TKM_API int tkm_runtime_init_dp(TkmRuntime *rt, const void *unique_id128, int rank, int world_size);

/* The same with the dtype the gradients cross NVLink in: 0 fp32 (what
 * tkm_runtime_init_dp uses), 1 bf16 (each bucket is rounded to bf16 on the
 * communication stream, averaged by NCCL in bf16 and widened back to fp32
 * before the SGD update: half the bytes on the links). */
TKM_API int tkm_runtime_init_dp_ex(TkmRuntime *rt, const void *unique_id128, int rank, int world_size,
                                   int grad_dtype);

/* Times the data-parallel gradient exchange alone: `iters` rounds of every
 * bucket's all-reduce (with the bf16 conversions when selected) on the
 * runtime's communication stream, outside the step.  The gradients are
 * averaged in place (call it between steps, not inside one).  Writes the
 * average milliseconds of one round to *ms_out and returns the bytes one rank
 * sends into the all-reduce per round (0 on failure or without data
 * parallelism). */
TKM_API size_t tkm_runtime_dp_allreduce_time(TkmRuntime *rt, int iters, float *ms_out);

/* The gradient buckets of the data-parallel step (host logic, no device
 * state).  Inputs, per learnable tensor in registration (checkpoint) order:
 * its value count n[t], its node id node[t] and has_grad[t] (non-zero when
 * the step updates it; those tensors own consecutive gradient slots, each
 * rounded up to 64 values).  Buckets are cut at node boundaries walking from
 * the last tensor, which the backward finishes first, to the first; a bucket
 * closes once it holds at least target_elems values.  Writes up to `cap`
 * buckets (start node, first slot value, value count) in the order they are
 * exchanged and returns their number; together they cover every slot once. */
TKM_API int tkm_dp_plan_buckets(int ntens, const size_t *n, const int *node, const int *has_grad,
                                size_t target_elems, int cap, int *bucket_node, size_t *bucket_off,
                                size_t *bucket_len);

/* Per-launch device timing of the training step: runs `iters` eager steps
 * (weights are updated with the current learning rate), timing every launch
 * of the step with CUDA events, and fills up to `capacity` entries in step
 * order with average milliseconds and the launch's algorithmic work.
 * kind: 0 plasma group, 1 GEMM, 2 attention, 3 softmax / loss, 4 SGD,
 * 5 collective.  Returns the number of entries. */
typedef struct {
    char name[64];
    int node, kind, backward;
    double bytes, flops;
    float ms;
} TkmProfileEntry;
TKM_API int tkm_runtime_profile(TkmRuntime *rt, int iters, TkmProfileEntry *out, int capacity);

/* Re-draws every learnable tensor on the device: GEMM weights N(0, std)
 * (std <= 0 keeps the He scale sqrt(2 / fan_in) the engine starts with),
 * gains 1, biases and shifts 0; velocities are cleared. */
TKM_API int tkm_runtime_init_weights(TkmRuntime *rt, unsigned long long seed, float std);

/* The runtime's CUDA stream (a cudaStream_t), for callers that time or order
 * their own work against it. */
TKM_API void *tkm_runtime_stream(const TkmRuntime *rt);

/* Datasets beyond the reference's uint8 per-sample labels, for
 * tkm_runtime_train_epoch.  Like tkm_dataset_create they live on the device
 * when they fit in half the free device memory (tkm_dataset_is_resident);
 * an epoch then gathers every batch on the device inside one captured graph
 * per step and reads the loss back once.
 *   _i32:    h_inputs as tkm_dataset_create, and one int32 label per loss
 *            row: [num_samples][loss rows per sample] (sequence models,
 *            vocabularies above 256).
 *   _tokens: token sequences h_tokens [num_seqs][S + 1] (S = the input's
 *            rows per sample) over an embedding table h_embed [vocab][C]
 *            (C = the input's channels): input row p of a sequence is
 *            h_embed[token p], its label is token p + 1.  Needs one loss row
 *            per input row.
 * Labels and tokens are checked against the loss width and the table. */
TKM_API TkmDataset *tkm_dataset_create_i32(TkmRuntime *rt, const float *h_inputs, const int32_t *h_labels,
                                           size_t num_samples);
TKM_API TkmDataset *tkm_dataset_create_tokens(TkmRuntime *rt, const float *h_embed, int vocab,
                                              const int32_t *h_tokens, size_t num_seqs);

#ifdef __cplusplus
}
#endif

#endif /* TKM_H */
