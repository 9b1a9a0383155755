/*
 * tkm_internal.h -- private declarations shared by the host runtime sources
 * (registry, DSL front end, code generator, runtime).
 */
#ifndef TKM_INTERNAL_H
#define TKM_INTERNAL_H

#include <stdarg.h>
#include <stddef.h>

#include "tkm.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Diagnostics.  The reference prints and calls exit(1) on every malformed
 * graph (src/tkm_core.c:147-150, 289-293 ...); this build records the message
 * (tkm_last_error), prints it to stderr, and leaves the graph empty
 * (num_nodes = 0) so later stages return NULL / 0 instead of exiting. */
void tkm_set_error(const char *fmt, ...);
void tkm_clear_error(void);
void tkm_graph_error(TkmGraph *g, const char *fmt, ...);
/* Informational lines (fusion hits, ignite summary) go to stdout only when the
 * environment variable TKM_VERBOSE is set to a non-zero value. */
void tkm_log(const char *fmt, ...);
int tkm_verbose(void);

/* First line of every tkm_codegen_cuda_string() result.  tkm_runtime_ignite()
 * accepts only sources that carry it: the generated kernels and the runtime
 * share one private launch contract (argument lists, storage type, gradient
 * store modes) that a foreign source would not follow. */
#define TKM_CODEGEN_MARKER "// tokamak-b200 plasma codegen v1"

/* ------------------------------------------------ backward write planning
 * Backward schedule: nodes in reverse order; a plasma group runs at its output
 * node.  Each write into an activation-gradient slot either overwrites (the
 * slot's first writer) or accumulates.  Values: 0 overwrite, 1 accumulate,
 * -1 no such write. */
typedef struct {
    signed char group_din_acc[TKM_MAX_GROUPS];
    signed char node_din_acc[TKM_MAX_NODES];   /* runtime operators writing d(in0) */
    signed char add_branch_acc[TKM_MAX_NODES]; /* Add node id -> its d(in1) write */
    unsigned char zero_first[TKM_MAX_NODES];   /* slots cleared before the backward */
} TkmGradPlan;

void tkm_plan_grads(const TkmGraph *g, TkmGradPlan *plan);
/* storage owner of a node's output (Flatten shares its input's storage) */
int tkm_slot_of(const TkmGraph *g, int node);

/* ------------------------------------------------- plasma kernel geometry
 * Fixed by the channel count and the storage type (act_bytes 2 = bf16,
 * 4 = fp32); computed identically by the code generator and the runtime. */
typedef struct {
    int C, C2;   /* channels, channel pairs */
    int vp;      /* pairs per 16-byte chunk */
    int nch;     /* chunks per row */
    int tpr;     /* threads per row */
    int kch;     /* chunks per thread */
    int rpb;     /* rows per block */
    int threads; /* block size */
    int ncb;     /* column blocks: > 1 splits a row over blockIdx.y (no row statistics) */
    int rows;    /* batch_size * H * W */
    int fwd_grid;
    int persist; /* forward kernel loops over row blocks with the next one prefetched
                  * (groups without a normalisation); else one row block per block */
} TkmRowGeom;

void tkm_row_geom(const TkmGraph *g, const PlasmaGroup *pg, int act_bytes, TkmRowGeom *geom);
/* backward kernel geometry: the forward's (two chunks per thread for
 * normalisation rows, column blocks of up to 1024 threads for a twin
 * epilogue and of up to 256 for other elementwise groups) */
void tkm_row_geom_bwd(const TkmGraph *g, const PlasmaGroup *pg, int act_bytes, TkmRowGeom *geom);
int tkm_sm_count_hint(void);
/* dynamic shared memory of a plasma backward kernel: its two stages of row
 * inputs (0: the kernel loads rows directly) */
int tkm_group_bwd_stage_bytes(const TkmGraph *g, const PlasmaGroup *pg, int act_bytes);
/* row-sized inputs a plasma backward kernel reads (dout, the group input and
 * replayed Add branches when its backward needs them; a twin input counts 2) */
int tkm_group_bwd_row_inputs(const TkmGraph *g, const PlasmaGroup *pg);
/* dynamic shared memory of a plasma forward kernel (normalisation groups run
 * persistent with staged rows when it is > 0) */
int tkm_group_fwd_stage_bytes(const TkmGraph *g, const PlasmaGroup *pg, int act_bytes);

/* ------------------------------------------------ plasma kernel arguments
 * Argument list of a generated kernel (forward or backward).  The code
 * generator names argument i "a<i>"; the runtime passes the pointer that the
 * entry resolves to.  Structurally equal groups therefore produce the same
 * text and share one compiled kernel. */
enum {
    KA_IN = 0,   /* activations of the group input (anchor) */
    KA_OUT,      /* activations of the group output */
    KA_DOUT,     /* gradient of the group output */
    KA_DIN,      /* gradient of the group input */
    KA_PARAM,    /* per-channel parameter: node, which (0 weight, 1 beta, 2 bias) */
    KA_MASK,     /* dropout mask of node */
    KA_SEED,     /* step seed */
    KA_BRANCH,   /* activations of Add node's second input */
    KA_DBRANCH,  /* gradient of Add node's second input */
    KA_PART,     /* partial rows of parameter gradients */
    KA_ROPE      /* cos/sin table of a QKV prep group */
};

typedef struct {
    int kind;
    int node;  /* global node id (KA_PARAM, KA_MASK, KA_SEED, KA_BRANCH, KA_DBRANCH) */
    int which; /* KA_PARAM: 0 weight, 1 beta, 2 bias */
} TkmKArg;

#define TKM_MAX_GROUP_ARGS 96
int tkm_group_kargs(const TkmGraph *g, const PlasmaGroup *pg, int bwd, TkmKArg *out);
/* parameters whose gradients a group reduces, in partial-row order */
int tkm_group_params(const TkmGraph *g, const PlasmaGroup *pg, int *node, int *which);
/* class id of every group (groups with identical generated code share one) */
int tkm_codegen_classes(const TkmGraph *g, int *class_of);
/* NULL if every group can be generated, else the reason of the first that cannot */
const char *tkm_codegen_unsupported(const TkmGraph *g, int *group);

/* device prelude compiled in front of the generated source (tkm_prelude.cuh) */
extern const char tkm_prelude_src[];

#ifdef __cplusplus
}
#endif

#endif
