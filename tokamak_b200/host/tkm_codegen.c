/*
 * tkm_codegen.c -- NVRTC code generator for sm_100a plasma groups.
 *
 * Replaces the reference's table-driven emitter (src/tkm_codegen.c:297-634).
 * Kept from the reference: the fused semantics of a plasma group (a chain of
 * fluid operators around at most one normalisation, the twin-branch
 * `[gate|up]` epilogue, the QKV prep with QKNorm and RoPE), and the registry's
 * per-pair CUDA bodies and scalar formulas, which run unchanged in the same
 * snippet environment (v / dy / pre as float2, fval, tid, row, idx2, active,
 * w_vec / b_vec / beta_vec, acc_dw / acc_db / acc_dbeta, save_mask, rng).
 *
 * This build's own design:
 *   - activations are bf16 (fp32 in the fp32 mode; macro TKM_ACT_BYTES at
 *     compile time) and rows move in 16-byte chunks: each thread owns whole
 *     chunks, interleaved across the threads of a row, so warp accesses are
 *     coalesced (tkm_row_geom);
 *   - row statistics are warp-shuffle reductions plus one shared-memory step
 *     when a row spans several warps (the reference reduces within one warp,
 *     which is wrong for rows wider than 64 channels);
 *   - the backward replays the chain from the group input in registers instead
 *     of reading saved x-hat / istd tensors (never allocated);
 *   - each gradient slot is overwritten by its first backward writer and
 *     accumulated by later ones (tkm_plan_grads), so the gradient arena is not
 *     cleared every step;
 *   - per-channel parameter gradients are reduced deterministically: each
 *     backward block writes one partial row, a finalize kernel sums the rows
 *     in block order (no atomics);
 *   - kernels take canonical argument names (tkm_group_kargs), so groups with
 *     identical structure share one compiled kernel ("class").
 */
#include <ctype.h>
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "tkm_internal.h"

/* ----------------------------------------------------------- string build */

typedef struct {
    char *s;
    size_t n, cap;
    int oom;
} Buf;

static void bprintf(Buf *b, const char *fmt, ...) {
    if (b->oom) return;
    va_list ap;
    va_start(ap, fmt);
    const int need = vsnprintf(NULL, 0, fmt, ap);
    va_end(ap);
    if (need < 0) return;
    if (b->n + (size_t)need + 1 > b->cap) {
        size_t cap = b->cap ? b->cap : 65536;
        while (b->n + (size_t)need + 1 > cap) cap *= 2;
        char *s = (char *)realloc(b->s, cap);
        if (!s) {
            b->oom = 1;
            return;
        }
        b->s = s;
        b->cap = cap;
    }
    va_start(ap, fmt);
    vsnprintf(b->s + b->n, (size_t)need + 1, fmt, ap);
    va_end(ap);
    b->n += (size_t)need;
}

/* ---------------------------------------------------------------- geometry */

int tkm_sm_count_hint(void) { return 148; }

static int pow2_at_least(int v) {
    int p = 1;
    while (p < v) p *= 2;
    return p;
}

static int round_up(int v, int m) { return (v + m - 1) / m * m; }

static int group_has_norm(const TkmGraph *g, const PlasmaGroup *pg);

/* Rows move in 16-byte chunks of `vp` channel pairs.  A group with a
 * normalisation needs whole rows in one block (row statistics): up to 1024
 * threads per row, each owning kch chunks.  Any other group is elementwise
 * along the row: a row is split over `ncb` column blocks (blockIdx.y) of at
 * most 256 threads with one chunk per thread, which keeps registers low and
 * occupancy high.  Small rows pack rpb rows into a 256-thread block. */
void tkm_row_geom(const TkmGraph *g, const PlasmaGroup *pg, int act_bytes, TkmRowGeom *o) {
    memset(o, 0, sizeof(*o));
    o->C = pg->C;
    o->C2 = pg->C / 2;
    o->rows = g->batch_size * pg->H * pg->W;
    int vp = act_bytes == 2 ? 4 : 2; /* channel pairs in 16 bytes */
    while (vp > 1 && o->C2 % vp) vp /= 2;
    o->vp = vp;
    o->nch = o->C2 / vp;
    const int nch = o->nch > 0 ? o->nch : 1;
    o->kch = 1;
    o->ncb = 1;
    if (nch <= 32) {
        o->tpr = pow2_at_least(nch);
    } else if (group_has_norm(g, pg)) {
        /* two or more chunks per thread keep 32+ bytes per operand in flight */
        o->kch = nch >= 64 ? 2 : 1;
        if ((nch + o->kch - 1) / o->kch > 1024) o->kch = (nch + 1023) / 1024;
        o->tpr = round_up((nch + o->kch - 1) / o->kch, 32);
    } else {
        /* column blocks of at most 256 threads; a twin epilogue's of up to
         * 1024 (configuration 3, same box, alternated twice: twin forward
         * 184-186 -> 166 us, backward 360-370 -> 335-337 us with 1024;
         * the one-input Bias on 32000-wide rows is best at 256: 176 us
         * there, 204 us at 1024) */
        const int cap = pg->is_twin_epilogue ? 1024 : 256;
        o->ncb = (nch + cap - 1) / cap;
        o->tpr = round_up((nch + o->ncb - 1) / o->ncb, 32);
    }
    o->rpb = o->tpr >= 256 ? 1 : 256 / o->tpr;
    o->threads = o->tpr * o->rpb;
    o->fwd_grid = (o->rows + o->rpb - 1) / o->rpb;
    /* measured: prefetching the next row pays for elementwise groups (twin
     * 0.69 -> 0.76, bias 0.82 -> 0.91 of HBM) but costs a normalisation the
     * resident blocks that its row reduction needs (0.65 -> 0.60) */
    /* the QKV prep's normalisation is per 64-wide head, within a warp: it
     * needs no block-wide reduction and its forward is persistent too */
    o->persist = !group_has_norm(g, pg) || pg->is_qkv_prep;
}

/* The backward uses the forward's geometry.  It used to give a normalisation
 * group one chunk per thread (twice the threads): at configuration 3 the
 * Bias+Add+RMSNorm backward took 148.7-149.7 us that way against 125.4-125.6
 * us with the forward's two chunks per thread (0.70 -> 0.84 of HBM, same
 * box, alternated three times). */
void tkm_row_geom_bwd(const TkmGraph *g, const PlasmaGroup *pg, int act_bytes, TkmRowGeom *o) {
    tkm_row_geom(g, pg, act_bytes, o);
}

/* ---------------------------------------------------------- node lists */

/* nodes a group's kernels touch: twin left chain, twin right chain, then
 * the group chain (without the twin Mul, which is the product itself) */
typedef struct {
    int ids[3 * TKM_MAX_CHAIN + 16];
    int nl, nr, nc, n;
} Lists;

static void group_lists(const TkmGraph *g, const PlasmaGroup *pg, Lists *L) {
    memset(L, 0, sizeof(*L));
    int start = 0;
    if (pg->is_twin_epilogue) {
        const TkmNode *m = &g->nodes[pg->node_ids[0]];
        for (int i = 0; i < m->left_len; i++) L->ids[L->n++] = m->left_nodes[i];
        for (int i = 0; i < m->right_len; i++) L->ids[L->n++] = m->right_nodes[i];
        L->nl = m->left_len;
        L->nr = m->right_len;
        start = 1;
    }
    for (int i = start; i < pg->count; i++) L->ids[L->n++] = pg->node_ids[i];
    L->nc = L->n - L->nl - L->nr;
}

/* Rows a backward kernel stages (tkm_group_bwd_stage_bytes): the group input
 * (both halves for a twin epilogue), dout, and the second input of every Add
 * but a trailing one (whose forward the backward does not replay). */
static int bwd_needs_input(const TkmGraph *g, const PlasmaGroup *pg);

static int bwd_staged_rows(const TkmGraph *g, const PlasmaGroup *pg) {
    Lists L;
    group_lists(g, pg, &L);
    if (!pg->is_twin_epilogue && !bwd_needs_input(g, pg)) return 1; /* dout only */
    int n = (pg->is_twin_epilogue ? 2 : 1) + 1;
    const int last = L.n - 1;
    const int skip = (L.nc > 0 && g->nodes[L.ids[last]].cat != CAT_NORM) ? last : -1;
    for (int i = 0; i < L.n; i++)
        if (g->nodes[L.ids[i]].op == OP_ADD && i != skip) n++;
    return n;
}

/* A chain of Bias and Add operators only (outside a twin epilogue) has a
 * backward that needs dout alone: its input is neither loaded nor replayed. */
static int bwd_needs_input(const TkmGraph *g, const PlasmaGroup *pg) {
    if (pg->is_twin_epilogue) return 1;
    Lists L;
    group_lists(g, pg, &L);
    for (int i = L.nl + L.nr; i < L.n; i++) {
        const int op = g->nodes[L.ids[i]].op;
        if (op != OP_BIAS && op != OP_ADD) return 1;
    }
    return 0;
}

int tkm_group_bwd_row_inputs(const TkmGraph *g, const PlasmaGroup *pg) { return bwd_staged_rows(g, pg); }

/* Row blocks in flight in a staged kernel's cp.async ring (its slots):
 * TKM_FWD_SLOTS / TKM_BWD_SLOTS (2-4) override the default of 2.  Measured
 * at configuration 3 (same box, alternated twice): 3 or 4 backward slots
 * left the norm backward at 145-150 us (2: 145 us) and slowed the twin
 * backward (338 -> 350-369 us); 3 forward slots slowed the norm forward
 * (66 -> 68-69 us).  The rows are not latency-bound at two slots. */
static int stage_slots(int bwd) {
    const char *e = getenv(bwd ? "TKM_BWD_SLOTS" : "TKM_FWD_SLOTS");
    const int v = e ? atoi(e) : 2;
    return v < 2 ? 2 : (v > 4 ? 4 : v);
}

/* Forward row staging: the row inputs (the group input, both halves for a
 * twin, and every Add branch) of the next two row blocks are brought by
 * cp.async into dynamic shared memory while the current one computes.
 * Measured: a normalisation group 0.66 -> 0.92 of HBM, the twin epilogue
 * 0.76 -> 0.90; a one-input elementwise group runs faster with its next row
 * prefetched into registers (0.91 vs 0.87), so it is not staged. */
static int fwd_stage_bytes_raw(const TkmGraph *g, const PlasmaGroup *pg, int act_bytes) {
    if (pg->is_qkv_prep) return 0;
    TkmRowGeom gm;
    tkm_row_geom(g, pg, act_bytes, &gm);
    Lists L;
    group_lists(g, pg, &L);
    int n = pg->is_twin_epilogue ? 2 : 1;
    for (int i = 0; i < L.n; i++)
        if (g->nodes[L.ids[i]].op == OP_ADD) n++;
    if (gm.persist && n < 2) return 0;
    const long bytes = (long)stage_slots(0) * n * gm.kch * gm.threads * 16;
    return bytes <= 128 * 1024 ? (int)bytes : 0;
}

/* Elementwise groups (persistent in every form) are staged only when both
 * storage types stage, so that the kernel always loops over row blocks;
 * a normalisation group without staging runs one row block per block. */
int tkm_group_fwd_stage_bytes(const TkmGraph *g, const PlasmaGroup *pg, int act_bytes) {
    TkmRowGeom gm;
    tkm_row_geom(g, pg, act_bytes, &gm);
    if (gm.persist && (!fwd_stage_bytes_raw(g, pg, 2) || !fwd_stage_bytes_raw(g, pg, 4))) return 0;
    return fwd_stage_bytes_raw(g, pg, act_bytes);
}

/* measured: staging pays for backward kernels that read several rows per row
 * (twin 0.78 -> 0.82 of HBM, norm 166 -> 163 us); one that streams dout alone
 * runs faster on plain loads (182 vs 210 us) */
int tkm_group_bwd_stage_bytes(const TkmGraph *g, const PlasmaGroup *pg, int act_bytes) {
    if (pg->is_qkv_prep) return 0;
    const int nrows = bwd_staged_rows(g, pg);
    if (nrows < 2) return 0;
    TkmRowGeom gm;
    tkm_row_geom_bwd(g, pg, act_bytes, &gm);
    const long bytes = (long)stage_slots(1) * nrows * gm.kch * gm.threads * 16;
    return bytes <= 128 * 1024 ? (int)bytes : 0;
}

static uint32_t node_flags(const TkmGraph *g, int id) {
    const TkmOpSpec *sp = tkm_find_spec_by_node(&g->nodes[id]);
    return sp ? sp->res_flags : 0;
}

static int group_has_norm(const TkmGraph *g, const PlasmaGroup *pg) {
    if (pg->is_qkv_prep) return 0;
    Lists L;
    group_lists(g, pg, &L);
    for (int i = 0; i < L.n; i++)
        if (g->nodes[L.ids[i]].cat == CAT_NORM) return 1;
    return 0;
}

int tkm_group_params(const TkmGraph *g, const PlasmaGroup *pg, int *node, int *which) {
    int cnt = 0;
    if (pg->is_qkv_prep) {
        const TkmNode *n = &g->nodes[pg->node_ids[0]];
        if (n->has_qknorm) node[cnt] = n->id, which[cnt++] = 0;
        node[cnt] = n->id, which[cnt++] = 2;
        return cnt;
    }
    Lists L;
    group_lists(g, pg, &L);
    for (int i = 0; i < L.n; i++) {
        const uint32_t f = node_flags(g, L.ids[i]);
        if (f & RES_PARAM_WEIGHT) node[cnt] = L.ids[i], which[cnt++] = 0;
        if (f & RES_PARAM_BETA) node[cnt] = L.ids[i], which[cnt++] = 1;
        if (f & RES_PARAM_BIAS) node[cnt] = L.ids[i], which[cnt++] = 2;
    }
    return cnt;
}

static int push_arg(TkmKArg *out, int n, int kind, int node, int which) {
    if (n < TKM_MAX_GROUP_ARGS) out[n] = (TkmKArg){kind, node, which};
    return n + 1;
}

int tkm_group_kargs(const TkmGraph *g, const PlasmaGroup *pg, int bwd, TkmKArg *out) {
    int n = 0;
    if (!bwd) {
        n = push_arg(out, n, KA_IN, -1, 0);
        n = push_arg(out, n, KA_OUT, -1, 0);
    } else {
        n = push_arg(out, n, KA_DOUT, -1, 0);
        n = push_arg(out, n, KA_IN, -1, 0);
        n = push_arg(out, n, KA_DIN, -1, 0);
        n = push_arg(out, n, KA_PART, -1, 0);
    }
    if (pg->is_qkv_prep) {
        const TkmNode *p = &g->nodes[pg->node_ids[0]];
        n = push_arg(out, n, KA_PARAM, p->id, 2);
        if (p->has_qknorm) n = push_arg(out, n, KA_PARAM, p->id, 0);
        if (p->has_rope) n = push_arg(out, n, KA_ROPE, -1, 0);
        return n;
    }
    Lists L;
    group_lists(g, pg, &L);
    for (int i = 0; i < L.n; i++) {
        const int id = L.ids[i];
        const uint32_t f = node_flags(g, id);
        if (f & RES_PARAM_WEIGHT) n = push_arg(out, n, KA_PARAM, id, 0);
        if (f & RES_PARAM_BETA) n = push_arg(out, n, KA_PARAM, id, 1);
        if (f & RES_PARAM_BIAS) n = push_arg(out, n, KA_PARAM, id, 2);
        if (f & RES_SAVE_MASK) n = push_arg(out, n, KA_MASK, id, 0);
        if ((f & RES_RNG_SEED) && !bwd) n = push_arg(out, n, KA_SEED, id, 0);
        if (g->nodes[id].op == OP_ADD) {
            n = push_arg(out, n, KA_BRANCH, id, 0);
            if (bwd) n = push_arg(out, n, KA_DBRANCH, id, 0);
        }
    }
    return n;
}

/* --------------------------------------------------------- write planning */

int tkm_slot_of(const TkmGraph *g, int node) {
    while (node > 0 && !g->nodes[node].dead && g->nodes[node].op == OP_FLATTEN) node = g->nodes[node].in0;
    return node;
}

void tkm_plan_grads(const TkmGraph *g, TkmGradPlan *plan) {
    memset(plan, 0, sizeof(*plan));
    memset(plan->group_din_acc, -1, sizeof(plan->group_din_acc));
    memset(plan->node_din_acc, -1, sizeof(plan->node_din_acc));
    memset(plan->add_branch_acc, -1, sizeof(plan->add_branch_acc));
    unsigned char written[TKM_MAX_NODES];
    memset(written, 0, sizeof(written));
    for (int i = g->num_nodes - 1; i >= 1; i--) {
        const TkmNode *n = &g->nodes[i];
        if (n->dead) continue;
        if (n->plasma_grp >= 0) {
            const PlasmaGroup *pg = &g->groups[n->plasma_grp];
            if (pg->out_node_id != i || pg->is_coord_group) continue;
            /* the backward visits the chain from its last operator */
            for (int j = pg->count - 1; j >= 0; j--) {
                const TkmNode *cn = &g->nodes[pg->node_ids[j]];
                if (cn->op != OP_ADD) continue;
                const int s = tkm_slot_of(g, cn->in1);
                plan->add_branch_acc[cn->id] = written[s];
                written[s] = 1;
            }
            const int s = tkm_slot_of(g, pg->anchor_id);
            plan->group_din_acc[pg->id] = written[s];
            written[s] = 1;
            continue;
        }
        switch (n->op) {
            case OP_FC:
            case OP_FC_TWIN_FUSED:
            case OP_FC_QKV_FUSED:
            case OP_GQA_ATTN:
            case OP_SOFTMAX:
            case OP_SOFTMAX_CE:
            case OP_SOFTMAX_FOCAL:
            case OP_SOFTMAX_MSE: {
                const int s = tkm_slot_of(g, n->in0);
                plan->node_din_acc[i] = written[s];
                written[s] = 1;
                break;
            }
            default:
                break;
        }
    }
    /* the standalone softmax backward only accumulates: clear its slot first */
    for (int i = 1; i < g->num_nodes; i++) {
        const TkmNode *n = &g->nodes[i];
        if (!n->dead && n->plasma_grp < 0 && n->op == OP_SOFTMAX && plan->node_din_acc[i] == 0)
            plan->zero_first[tkm_slot_of(g, n->in0)] = 1;
    }
}

/* ------------------------------------------------------------ validation */

static int native_op(const TkmNode *n) {
    return n->cat == CAT_NORM || n->op == OP_ADD || n->op == OP_MUL || n->op == OP_QKNORM || n->op == OP_ROPE ||
           n->op == OP_BIAS;
}

static const char *group_unsupported(const TkmGraph *g, const PlasmaGroup *pg) {
    if (pg->is_coord_group) return "image augmentation (coordinate) groups are not supported by this build";
    if (pg->C <= 0 || pg->C % 2) return "plasma groups need a positive, even channel count";
    TkmRowGeom g2, g4;
    tkm_row_geom(g, pg, 2, &g2);
    tkm_row_geom(g, pg, 4, &g4);
    if (g2.kch > 16 || g4.kch > 16) return "rows wider than 65536 channels are not supported in plasma groups";
    if (pg->is_qkv_prep) {
        const TkmNode *n = &g->nodes[pg->node_ids[0]];
        const int hd2 = n->head_dim / 2;
        if (n->head_dim <= 0 || hd2 % 4 || n->q_c % n->head_dim || n->k_c % n->head_dim)
            return "QKV prep needs a head dimension that is a multiple of 8 and whole heads";
        if (n->has_qknorm && n->head_dim != 64) return "QKNorm supports 64-dimensional heads only";
        if (n->has_qknorm && ((g2.tpr % (hd2 / g2.vp)) || (g4.tpr % (hd2 / g4.vp))))
            return "QKV prep row layout does not keep heads within one warp";
        return NULL;
    }
    Lists L;
    group_lists(g, pg, &L);
    for (int i = 0; i < pg->count; i++) {
        const TkmNode *n = &g->nodes[pg->node_ids[i]];
        if (n->op == OP_MUL && !(i == 0 && pg->is_twin_epilogue))
            return "Mul merges need FC-rooted branches that fuse into a twin GEMM";
    }
    for (int i = 0; i < L.n; i++) {
        const TkmNode *n = &g->nodes[L.ids[i]];
        if (n->op == OP_QKNORM || n->op == OP_ROPE)
            return "QKNorm and RoPE are supported only on the Q/K branches feeding a GQA node";
        const TkmOpSpec *sp = tkm_find_spec_by_node(n);
        if (!sp) return "node without a registry entry";
        if (native_op(n)) continue;
        if (!(sp->fwd_cuda || sp->fwd_expr) || !(sp->bwd_cuda || sp->bwd_expr))
            return "fluid operator without forward and backward definitions";
        if ((sp->fwd_cuda && strstr(sp->fwd_cuda, "row_reduce_sum")) ||
            (sp->bwd_cuda && strstr(sp->bwd_cuda, "row_reduce_sum")))
            return "fluid operators that call row_reduce_sum are not supported (use a normalisation operator)";
        if ((sp->res_flags & RES_SAVE_MASK) && n->op != OP_DROP) return "only Drop may use a saved mask";
        if ((sp->res_flags & RES_RNG_SEED) && n->op != OP_DROP) return "only Drop may draw random numbers";
    }
    return NULL;
}

const char *tkm_codegen_unsupported(const TkmGraph *g, int *group) {
    for (int i = 0; i < g->num_groups; i++) {
        const char *why = group_unsupported(g, &g->groups[i]);
        if (why) {
            if (group) *group = i;
            return why;
        }
    }
    return NULL;
}

/* --------------------------------------------------------------- emitter */

typedef struct {
    const TkmGraph *g;
    const PlasmaGroup *pg;
    const TkmGradPlan *plan;
    Buf *b;
    Lists L;
    TkmKArg args[TKM_MAX_GROUP_ARGS];
    int nargs;
    char name_buf[8][16];
    int name_next;
    int acc_smem;   /* parameter-gradient accumulators in shared memory (TKM_ACC) */
    int param_regs; /* per-channel parameters preloaded into registers (tp*_j) */
    char pexpr_buf[4][64];
    int pexpr_next;
} Em;

static int local_of(const Em *e, int node) {
    for (int i = 0; i < e->L.n; i++)
        if (e->L.ids[i] == node) return i;
    return -1;
}

static const char *A(Em *e, int kind, int node, int which);

/* a per-channel parameter (which: 0 weight, 1 beta, 2 bias) of node n at the
 * pair `tid` inside a pairs loop: the preloaded register or a read-only load */
static const char *pexpr(Em *e, const TkmNode *n, int which) {
    static const char *pfx[3] = {"tpw", "tpt", "tpc"};
    char *out = e->pexpr_buf[e->pexpr_next++ & 3];
    if (e->param_regs)
        snprintf(out, 64, "%s_%d[k][q]", pfx[which], local_of(e, n->id));
    else
        snprintf(out, 64, "__ldg(&%s[tid])", A(e, KA_PARAM, n->id, which));
    return out;
}

/* canonical name "a<i>" of an argument of the kernel being emitted */
static const char *A(Em *e, int kind, int node, int which) {
    for (int i = 0; i < e->nargs; i++) {
        const TkmKArg *a = &e->args[i];
        if (a->kind == kind && a->node == node && a->which == which) {
            char *s = e->name_buf[e->name_next++ & 7];
            snprintf(s, 16, "a%d", i);
            return s;
        }
    }
    return "MISSING_ARGUMENT";
}

static void emit_float(Buf *b, double v) {
    if (isinf(v)) bprintf(b, v > 0 ? "__int_as_float(0x7f800000)" : "__int_as_float(0xff800000)");
    else if (isnan(v)) bprintf(b, "__int_as_float(0x7fc00000)");
    else bprintf(b, "%.9ef", v);
}

/* scalar formula -> CUDA expression, x replaced by `var` */
static void emit_formula(Buf *b, const char *expr, const char *var) {
    static const char *map[][2] = {{"exp", "expf"}, {"log", "logf"}, {"ln", "logf"}, {"sqrt", "sqrtf"},
                                   {"sin", "sinf"}, {"cos", "cosf"}, {"tanh", "tanhf"}, {"abs", "fabsf"},
                                   {"max", "fmaxf"}, {"min", "fminf"}, {"pow", "powf"}};
    bprintf(b, "(");
    for (const char *p = expr; *p;) {
        if (isalpha((unsigned char)*p) || *p == '_') {
            char name[32];
            size_t n = 0;
            while (isalnum((unsigned char)*p) || *p == '_') {
                if (n + 1 < sizeof(name)) name[n++] = *p;
                p++;
            }
            name[n] = 0;
            const char *out = name;
            if (!strcmp(name, "x")) out = var;
            else if (!strcmp(name, "pi")) out = "3.14159265358979323846f";
            else
                for (size_t k = 0; k < sizeof(map) / sizeof(map[0]); k++)
                    if (!strcmp(name, map[k][0])) out = map[k][1];
            bprintf(b, "%s", out);
        } else if (isdigit((unsigned char)*p) || (*p == '.' && isdigit((unsigned char)p[1]))) {
            /* numbers become float literals so that 1/2 divides in floating point */
            char *end;
            const double v = strtod(p, &end);
            emit_float(b, v);
            p = end;
        } else {
            bprintf(b, "%c", *p++);
        }
    }
    bprintf(b, ")");
}

/* loops over the channel pairs this thread owns in its row */
static void pairs_begin(Buf *b) {
    bprintf(b,
            "    _Pragma(\"unroll\") for (int k = 0; k < TKG_KCH; ++k) {\n"
            "      const int tkm_ch = tkm_lr + k * TKG_TPR;\n"
            "      if (tkm_row_ok && tkm_ch < TKG_NCH) {\n"
            "        _Pragma(\"unroll\") for (int q = 0; q < TKG_VP; ++q) {\n"
            "          const int tid = tkm_ch * TKG_VP + q; (void)tid;\n"
            "          const long long idx2 = (long long)row * TKG_C2 + tid; (void)idx2;\n"
            "          const int active = 1; (void)active;\n");
}

static void pairs_end(Buf *b) { bprintf(b, "        }\n      }\n    }\n"); }

static void chunks_begin(Buf *b) {
    bprintf(b,
            "    _Pragma(\"unroll\") for (int k = 0; k < TKG_KCH; ++k) {\n"
            "      const int tkm_ch = tkm_lr + k * TKG_TPR;\n"
            "      if (tkm_row_ok && tkm_ch < TKG_NCH) {\n");
}

static void chunks_end(Buf *b) { bprintf(b, "      }\n    }\n"); }

static void decl_array(Buf *b, const char *name) { bprintf(b, "  float2 %s[TKG_KCH][TKG_VP];\n", name); }

static void zero_array(Buf *b, const char *name) {
    bprintf(b, "  _Pragma(\"unroll\") for (int k = 0; k < TKG_KCH; ++k) tkm_zero<TKG_VP>(%s[k]);\n", name);
}

static void copy_array(Buf *b, const char *dst, const char *src) {
    bprintf(b, "  _Pragma(\"unroll\") for (int k = 0; k < TKG_KCH; ++k) _Pragma(\"unroll\") for (int q = 0; q < TKG_VP; ++q) %s[k][q] = %s[k][q];\n",
            dst, src);
}

/* loads `arr` (declared by the caller) from row `rowv` when `okv` holds */
static void load_into(Buf *b, const char *arr, const char *src, const char *row_pairs, const char *col0,
                      const char *rowv, const char *okv) {
    bprintf(b,
            "  _Pragma(\"unroll\") for (int k = 0; k < TKG_KCH; ++k) {\n"
            "    const int tkm_ch = tkm_lr + k * TKG_TPR;\n"
            "    if (%s && tkm_ch < TKG_NCH) tkm_ld<TKG_VP>(%s, (long long)%s * %s + %s + tkm_ch * TKG_VP, %s[k]);\n"
            "    else tkm_zero<TKG_VP>(%s[k]);\n  }\n",
            okv, src, rowv, row_pairs, col0, arr, arr);
}

static void load_array(Buf *b, const char *arr, const char *src, const char *row_pairs, const char *col0) {
    decl_array(b, arr);
    load_into(b, arr, src, row_pairs, col0, "row", "tkm_row_ok");
}

static void store_array(Buf *b, const char *dst, const char *row_pairs, const char *col0, const char *arr, int acc) {
    chunks_begin(b);
    bprintf(b, "        %s<TKG_VP>(%s, (long long)row * %s + %s + tkm_ch * TKG_VP, %s[k]);\n",
            acc ? "tkm_st_add" : "tkm_st", dst, row_pairs, col0, arr);
    chunks_end(b);
}

/* does the backward of node n read the node's input value? */
static int needs_pre(const TkmNode *n) {
    if (n->cat == CAT_NORM) return 1;
    if (native_op(n) || n->op == OP_DROP) return 0;
    const TkmOpSpec *sp = tkm_find_spec_by_node(n);
    if (!sp) return 0;
    if (sp->bwd_expr) return 1;
    return sp->bwd_cuda && strstr(sp->bwd_cuda, "pre") != NULL;
}

static const char *which_name(int which) { return which == 0 ? "w" : (which == 1 ? "beta" : "b"); }

/* snippet environment of node n (local index j) */
static void snippet_env(Em *e, const TkmNode *n, int bwd) {
    Buf *b = e->b;
    const uint32_t f = node_flags(e->g, n->id);
    bprintf(b, "    const float fval = ");
    emit_float(b, n->fval);
    bprintf(b, "; (void)fval;\n    const float fval2 = ");
    emit_float(b, n->fval2);
    bprintf(b, "; (void)fval2;\n");
    if (f & RES_PARAM_BIAS) bprintf(b, "    const float2* __restrict__ b_vec = %s; (void)b_vec;\n", A(e, KA_PARAM, n->id, 2));
    if (f & RES_PARAM_WEIGHT) bprintf(b, "    const float2* __restrict__ w_vec = %s; (void)w_vec;\n", A(e, KA_PARAM, n->id, 0));
    if (f & RES_PARAM_BETA)
        bprintf(b, "    const float2* __restrict__ beta_vec = %s; (void)beta_vec;\n", A(e, KA_PARAM, n->id, 1));
    if (f & RES_SAVE_MASK) bprintf(b, "    %suint16_t* __restrict__ save_mask = %s;\n", bwd ? "const " : "", A(e, KA_MASK, n->id, 0));
    if ((f & RES_RNG_SEED) && !bwd)
        bprintf(b, "    const uint32_t tkm_seed = (*%s) ^ %uu;\n", A(e, KA_SEED, n->id, 0), (unsigned)(n->id * 19937 + 1));
}

/* forward of operator n on register array `arr` (statistics kept in st_*_j) */
static void emit_op_fwd(Em *e, const TkmNode *n, const char *arr, int replay) {
    Buf *b = e->b;
    const int j = local_of(e, n->id);
    const TkmOpSpec *sp = tkm_find_spec_by_node(n);
    const uint32_t f = sp->res_flags;
    bprintf(b, "  { /* %s */\n", sp->dsl_name);
    if (n->cat == CAT_NORM) {
        const int centered = n->op == OP_LN || n->op == OP_BN;
        bprintf(b, "    const float eps = ");
        emit_float(b, n->fval);
        bprintf(b, ";\n    float s = 0.f;\n");
        if (centered) {
            pairs_begin(b);
            bprintf(b, "          s += %s[k][q].x + %s[k][q].y;\n", arr, arr);
            pairs_end(b);
            bprintf(b, "    st_mean_%d = tkm_row_sum<TKG_TPR, TKG_RPB>(s, tkm_red) * TKG_INV_C;\n    s = 0.f;\n", j);
            pairs_begin(b);
            bprintf(b, "          const float d0 = %s[k][q].x - st_mean_%d, d1 = %s[k][q].y - st_mean_%d;\n"
                       "          s += d0 * d0 + d1 * d1;\n",
                    arr, j, arr, j);
            pairs_end(b);
        } else {
            pairs_begin(b);
            bprintf(b, "          s += %s[k][q].x * %s[k][q].x + %s[k][q].y * %s[k][q].y;\n", arr, arr, arr, arr);
            pairs_end(b);
        }
        bprintf(b, "    st_istd_%d = rsqrtf(tkm_row_sum<TKG_TPR, TKG_RPB>(s, tkm_red) * TKG_INV_C + eps);\n", j);
        pairs_begin(b);
        bprintf(b, "          float2 xh = make_float2((%s[k][q].x - st_mean_%d) * st_istd_%d, (%s[k][q].y - st_mean_%d) * st_istd_%d);\n",
                arr, j, j, arr, j, j);
        if (f & RES_PARAM_WEIGHT)
            bprintf(b, "          const float2 gm = %s; xh.x *= gm.x; xh.y *= gm.y;\n", pexpr(e, n, 0));
        if (f & RES_PARAM_BETA)
            bprintf(b, "          const float2 bt = %s; xh.x += bt.x; xh.y += bt.y;\n", pexpr(e, n, 1));
        bprintf(b, "          %s[k][q] = xh;\n", arr);
        pairs_end(b);
    } else if (n->op == OP_ADD) {
        /* the branch row was loaded with the row's other inputs (tbr_j) */
        bprintf(b, "    _Pragma(\"unroll\") for (int k = 0; k < TKG_KCH; ++k) _Pragma(\"unroll\") for (int q = 0; q < TKG_VP; ++q) {\n"
                   "      %s[k][q].x += tbr_%d[k][q].x; %s[k][q].y += tbr_%d[k][q].y;\n    }\n",
                arr, j, arr, j);
    } else if (n->op == OP_BIAS) {
        pairs_begin(b);
        bprintf(b, "          const float2 bb = %s; %s[k][q].x += bb.x; %s[k][q].y += bb.y;\n", pexpr(e, n, 2), arr, arr);
        pairs_end(b);
    } else if (n->op == OP_DROP && replay) {
        /* the replay applies the mask the forward saved */
        bprintf(b, "    const float keep = 1.0f - ");
        emit_float(b, n->fval);
        bprintf(b, ";\n");
        pairs_begin(b);
        bprintf(b, "          const uint16_t mk = %s[idx2];\n"
                   "          %s[k][q] = make_float2((mk & 0xFFu) ? %s[k][q].x / keep : 0.0f, (mk >> 8) ? %s[k][q].y / keep : 0.0f);\n",
                A(e, KA_MASK, n->id, 0), arr, arr, arr);
        pairs_end(b);
    } else {
        snippet_env(e, n, 0);
        pairs_begin(b);
        bprintf(b, "          float2 v = %s[k][q];\n", arr);
        if (f & RES_RNG_SEED)
            bprintf(b, "          %s rng; rng_init(&rng, tkm_seed, (uint32_t)idx2);\n", tkm_rng_struct_name(n->rng_type));
        if (sp->fwd_expr) {
            bprintf(b, "          v.x = ");
            emit_formula(b, sp->fwd_expr, "v.x");
            bprintf(b, ";\n          v.y = ");
            emit_formula(b, sp->fwd_expr, "v.y");
            bprintf(b, ";\n");
        } else {
            bprintf(b, "          {\n%s\n          }\n", sp->fwd_cuda);
        }
        bprintf(b, "          %s[k][q] = v;\n", arr);
        pairs_end(b);
    }
    bprintf(b, "  }\n");
}

/* Does Add node n's branch gradient land in the same slot as the group's own
 * input gradient (a residual whose skip is the group input)?  Both writes then
 * target one buffer: the kernel sums them in registers and stores once,
 * instead of two stores through pointers the compiler may reorder. */
static int add_aliases_din(const Em *e, const TkmNode *n) {
    return n->op == OP_ADD && !e->pg->is_twin_epilogue &&
           tkm_slot_of(e->g, n->in1) == tkm_slot_of(e->g, e->pg->anchor_id);
}

/* the first planned write among the aliased Add branches (the backward
 * plans a group's Adds from its last operator), or -1 */
static int first_aliased_add(const Em *e) {
    for (int j = e->pg->count - 1; j >= 0; j--) {
        const TkmNode *n = &e->g->nodes[e->pg->node_ids[j]];
        if (add_aliases_din(e, n)) return n->id;
    }
    return -1;
}

/* backward of operator n: `dy` array updated in place, `pre` = its input */
static void emit_op_bwd(Em *e, const TkmNode *n, const char *dy) {
    Buf *b = e->b;
    const int j = local_of(e, n->id);
    const TkmOpSpec *sp = tkm_find_spec_by_node(n);
    const uint32_t f = sp->res_flags;
    bprintf(b, "  { /* backward %s */\n", sp->dsl_name);
    if (n->cat == CAT_NORM) {
        const int centered = n->op == OP_LN || n->op == OP_BN;
        char gm[48];
        if (f & RES_PARAM_WEIGHT) snprintf(gm, sizeof(gm), "%s", pexpr(e, n, 0));
        else snprintf(gm, sizeof(gm), "make_float2(1.f, 1.f)");
        bprintf(b, "    float2 m = make_float2(0.f, 0.f);\n");
        pairs_begin(b);
        bprintf(b, "          const float2 xh = make_float2((tpre_%d[k][q].x - st_mean_%d) * st_istd_%d, (tpre_%d[k][q].y - st_mean_%d) * st_istd_%d);\n"
                   "          const float2 gy = %s[k][q], gm = %s;\n"
                   "          const float2 dxh = make_float2(gy.x * gm.x, gy.y * gm.y);\n",
                j, j, j, j, j, j, dy, gm);
        if (f & RES_PARAM_WEIGHT) bprintf(b, "          TKM_ACC(tacc_w_%d).x += gy.x * xh.x; TKM_ACC(tacc_w_%d).y += gy.y * xh.y;\n", j, j);
        if (f & RES_PARAM_BETA) bprintf(b, "          TKM_ACC(tacc_beta_%d).x += gy.x; TKM_ACC(tacc_beta_%d).y += gy.y;\n", j, j);
        if (centered) bprintf(b, "          m.x += dxh.x + dxh.y;\n");
        bprintf(b, "          m.y += dxh.x * xh.x + dxh.y * xh.y;\n");
        pairs_end(b);
        bprintf(b, "    m = tkm_row_sum2<TKG_TPR, TKG_RPB>(m, tkm_red2);\n"
                   "    const float m1 = %s, m2 = m.y * TKG_INV_C;\n",
                centered ? "m.x * TKG_INV_C" : "0.f");
        pairs_begin(b);
        bprintf(b, "          const float2 xh = make_float2((tpre_%d[k][q].x - st_mean_%d) * st_istd_%d, (tpre_%d[k][q].y - st_mean_%d) * st_istd_%d);\n"
                   "          const float2 gy = %s[k][q], gm = %s;\n"
                   "          %s[k][q] = make_float2(st_istd_%d * (gy.x * gm.x - m1 - xh.x * m2), st_istd_%d * (gy.y * gm.y - m1 - xh.y * m2));\n",
                j, j, j, j, j, j, dy, gm, dy, j, j);
        pairs_end(b);
    } else if (n->op == OP_ADD) {
        /* the branch receives the incoming gradient; the main path keeps it */
        if (add_aliases_din(e, n))
            bprintf(b, "    _Pragma(\"unroll\") for (int k = 0; k < TKG_KCH; ++k) _Pragma(\"unroll\") for (int q = 0; q < TKG_VP; ++q) {\n"
                       "      tdbr[k][q].x += %s[k][q].x; tdbr[k][q].y += %s[k][q].y;\n    }\n",
                    dy, dy);
        else
            store_array(b, A(e, KA_DBRANCH, n->id, 0), "TKG_C2", "0", dy, e->plan->add_branch_acc[n->id] > 0);
    } else if (n->op == OP_BIAS) {
        pairs_begin(b);
        bprintf(b, "          TKM_ACC(tacc_b_%d).x += %s[k][q].x; TKM_ACC(tacc_b_%d).y += %s[k][q].y;\n", j, dy, j, dy);
        pairs_end(b);
    } else {
        snippet_env(e, n, 1);
        pairs_begin(b);
        bprintf(b, "          float2 dy = %s[k][q];\n", dy);
        if (needs_pre(n)) bprintf(b, "          const float2 pre = tpre_%d[k][q];\n", j);
        else bprintf(b, "          const float2 pre = make_float2(0.f, 0.f); (void)pre;\n");
        if (f & RES_PARAM_WEIGHT) bprintf(b, "          float2 acc_dw = TKM_ACC(tacc_w_%d);\n", j);
        if (f & RES_PARAM_BETA) bprintf(b, "          float2 acc_dbeta = TKM_ACC(tacc_beta_%d);\n", j);
        if (f & RES_PARAM_BIAS) bprintf(b, "          float2 acc_db = TKM_ACC(tacc_b_%d);\n", j);
        if (sp->bwd_expr) {
            bprintf(b, "          dy.x *= ");
            emit_formula(b, sp->bwd_expr, "pre.x");
            bprintf(b, ";\n          dy.y *= ");
            emit_formula(b, sp->bwd_expr, "pre.y");
            bprintf(b, ";\n");
        } else {
            bprintf(b, "          {\n%s\n          }\n", sp->bwd_cuda);
        }
        if (f & RES_PARAM_WEIGHT) bprintf(b, "          TKM_ACC(tacc_w_%d) = acc_dw;\n", j);
        if (f & RES_PARAM_BETA) bprintf(b, "          TKM_ACC(tacc_beta_%d) = acc_dbeta;\n", j);
        if (f & RES_PARAM_BIAS) bprintf(b, "          TKM_ACC(tacc_b_%d) = acc_db;\n", j);
        bprintf(b, "          %s[k][q] = dy;\n", dy);
        pairs_end(b);
    }
    bprintf(b, "  }\n");
}

static void emit_params(Em *e) {
    Buf *b = e->b;
    for (int i = 0; i < e->nargs; i++) {
        const char *t = "void*";
        switch (e->args[i].kind) {
            case KA_IN:
            case KA_DOUT:
            case KA_BRANCH: t = "const tkm_act_t* __restrict__"; break;
            case KA_OUT:
            case KA_DIN:
            case KA_DBRANCH: t = "tkm_act_t* __restrict__"; break;
            case KA_PARAM: t = "const float2* __restrict__"; break;
            case KA_MASK: t = "uint16_t* __restrict__"; break;
            case KA_SEED: t = "const uint32_t* __restrict__"; break;
            case KA_PART: t = "float2* __restrict__"; break;
            case KA_ROPE: t = "const float2* __restrict__"; break;
        }
        bprintf(b, "%s    %s a%d", i ? ",\n" : "", t, i);
    }
    bprintf(b, ")");
}

static void set_args(Em *e, int bwd) { e->nargs = tkm_group_kargs(e->g, e->pg, bwd, e->args); }

static void emit_geom_macros(Em *e, int bwd) {
    Buf *b = e->b;
    TkmRowGeom g2, g4;
    if (bwd) {
        tkm_row_geom_bwd(e->g, e->pg, 2, &g2);
        tkm_row_geom_bwd(e->g, e->pg, 4, &g4);
    } else {
        tkm_row_geom(e->g, e->pg, 2, &g2);
        tkm_row_geom(e->g, e->pg, 4, &g4);
    }
    const TkmRowGeom *gs[2] = {&g2, &g4};
    for (int i = 0; i < 2; i++) {
        const TkmRowGeom *gm = gs[i];
        bprintf(b, i == 0 ? "#if TKM_ACT_BYTES == 2\n" : "#else\n");
        bprintf(b, "#define TKG_VP %d\n#define TKG_NCH %d\n#define TKG_TPR %d\n#define TKG_KCH %d\n#define TKG_RPB %d\n"
                   "#define TKG_THREADS %d\n#define TKG_CB %d\n#define TKG_STAGE_BYTES %d\n",
                gm->vp, gm->nch, gm->tpr, gm->kch, gm->rpb, gm->threads, gm->ncb,
                bwd ? tkm_group_bwd_stage_bytes(e->g, e->pg, i == 0 ? 2 : 4)
                    : tkm_group_fwd_stage_bytes(e->g, e->pg, i == 0 ? 2 : 4));
    }
    bprintf(b, "#endif\n#define TKG_NSLOT %d\n#define TKG_C2 %d\n#define TKG_ROWS %d\n#define TKG_INV_C ",
            stage_slots(bwd), g2.C2, g2.rows);
    emit_float(b, 1.0 / (double)g2.C);
    bprintf(b, "\n#define TKG_NRB ((TKG_ROWS + TKG_RPB - 1) / TKG_RPB)\n");
}

static void undef_geom(Buf *b) {
    bprintf(b, "#undef TKG_VP\n#undef TKG_NCH\n#undef TKG_TPR\n#undef TKG_KCH\n#undef TKG_RPB\n#undef TKG_THREADS\n#undef TKG_CB\n"
               "#undef TKG_STAGE_BYTES\n#undef TKG_NSLOT\n"
               "#undef TKG_C2\n#undef TKG_ROWS\n#undef TKG_INV_C\n#undef TKG_NRB\n");
}

static int range_has_norm(const Em *e, int lo, int hi) {
    for (int i = lo; i < hi; i++)
        if (e->g->nodes[e->L.ids[i]].cat == CAT_NORM) return 1;
    return 0;
}

static void declare_stats(Em *e) {
    for (int i = 0; i < e->L.n; i++)
        if (e->g->nodes[e->L.ids[i]].cat == CAT_NORM)
            bprintf(e->b, "  float st_istd_%d = 0.f, st_mean_%d = 0.f; (void)st_mean_%d;\n", i, i, i);
}

static void kernel_head(Em *e, const char *name, int row_from_block) {
    Buf *b = e->b;
    bprintf(b, "extern \"C\" __global__ void __launch_bounds__(TKG_THREADS) TKM_KNAME(%s)(\n", name);
    emit_params(e);
    bprintf(b, " {\n  const int tkm_ll = threadIdx.x %% TKG_TPR; (void)tkm_ll;\n"
               "  const int tkm_lr = tkm_ll + blockIdx.y * TKG_TPR;\n");
    if (row_from_block)
        bprintf(b, "  const int row = blockIdx.x * TKG_RPB + threadIdx.x / TKG_TPR;\n"
                   "  const bool tkm_row_ok = row < TKG_ROWS;\n");
}

/* per-channel parameters of natively emitted operators, loaded once per
 * thread (its chunks are the same for every row it handles) */
static void emit_param_preload(Em *e) {
    for (int i = 0; i < e->L.n; i++) {
        const TkmNode *n = &e->g->nodes[e->L.ids[i]];
        const uint32_t f = node_flags(e->g, n->id);
        const int norm = n->cat == CAT_NORM, bias = n->op == OP_BIAS;
        if (!norm && !bias) continue;
        const struct { uint32_t flag; int which; const char *pfx; } want[3] = {
            {RES_PARAM_WEIGHT, 0, "tpw"}, {RES_PARAM_BETA, 1, "tpt"}, {RES_PARAM_BIAS, 2, "tpc"}};
        for (int w = 0; w < 3; w++) {
            if (!(f & want[w].flag)) continue;
            if (bias && want[w].which != 2) continue;
            if (norm && want[w].which == 2) continue;
            bprintf(e->b,
                    "  float2 %s_%d[TKG_KCH][TKG_VP];\n"
                    "  _Pragma(\"unroll\") for (int k = 0; k < TKG_KCH; ++k) {\n"
                    "    const int tkm_ch = tkm_lr + k * TKG_TPR;\n"
                    "    _Pragma(\"unroll\") for (int q = 0; q < TKG_VP; ++q)\n"
                    "      %s_%d[k][q] = tkm_ch < TKG_NCH ? __ldg(&%s[tkm_ch * TKG_VP + q]) : make_float2(0.f, 0.f);\n"
                    "  }\n",
                    want[w].pfx, i, want[w].pfx, i, A(e, KA_PARAM, n->id, want[w].which));
        }
    }
}

/* the row's Add branch inputs, loaded together with its other inputs; `skip`
 * names a local whose operator is not applied (the backward's last one) */
static void emit_branch_loads(Em *e, int skip) {
    for (int i = 0; i < e->L.n; i++) {
        const TkmNode *n = &e->g->nodes[e->L.ids[i]];
        if (n->op != OP_ADD || i == skip) continue;
        char name[16];
        snprintf(name, sizeof(name), "tbr_%d", i);
        load_array(e->b, name, A(e, KA_BRANCH, n->id, 0), "TKG_C2", "0");
    }
}

/* inputs of one forward row: (array, source, row stride in pairs, column offset) */
typedef struct {
    char arr[16];
    const char *src;
    const char *stride;
    const char *col0;
} FwdInput;

static int fwd_inputs(Em *e, FwdInput *in) {
    int n = 0;
    const char *a = A(e, KA_IN, -1, 0);
    if (e->pg->is_twin_epilogue) {
        in[n++] = (FwdInput){"txl", a, "(2 * TKG_C2)", "0"};
        in[n++] = (FwdInput){"txr", a, "(2 * TKG_C2)", "TKG_C2"};
    } else {
        in[n++] = (FwdInput){"tx", a, "TKG_C2", "0"};
    }
    for (int i = 0; i < e->L.n && n < 16; i++) {
        const TkmNode *nd = &e->g->nodes[e->L.ids[i]];
        if (nd->op != OP_ADD) continue;
        FwdInput f = {"", A(e, KA_BRANCH, nd->id, 0), "TKG_C2", "0"};
        snprintf(f.arr, sizeof(f.arr), "tbr_%d", i);
        in[n++] = f;
    }
    return n;
}

/* The forward is persistent: each block walks row blocks tkm_rb, blockIdx.x +
 * k gridDim.x, with the next row block's inputs requested before the current
 * one is computed, and loads its per-channel parameters once. */
static void emit_plasma_fwd_rowblock(Em *e);

static void emit_plasma_fwd(Em *e) {
    TkmRowGeom gm;
    tkm_row_geom(e->g, e->pg, 2, &gm);
    if (!gm.persist || tkm_group_fwd_stage_bytes(e->g, e->pg, 2) > 0) {
        emit_plasma_fwd_rowblock(e);
        return;
    }
    Buf *b = e->b;
    const Lists *L = &e->L;
    set_args(e, 0);
    e->acc_smem = 0;
    e->param_regs = 1;
    kernel_head(e, "fwd", 0);
    if (range_has_norm(e, 0, L->n)) bprintf(b, "  __shared__ float tkm_red[TKM_RED_SLOTS(TKG_TPR, TKG_RPB)];\n");
    emit_param_preload(e);
    FwdInput in[16];
    const int nin = fwd_inputs(e, in);
    char nx[24];
    bprintf(b, "  int tkm_rb = blockIdx.x;\n"
               "  {\n    const int rown = tkm_rb * TKG_RPB + threadIdx.x / TKG_TPR;\n"
               "    const bool okn = tkm_rb < TKG_NRB && rown < TKG_ROWS;\n");
    for (int i = 0; i < nin; i++) {
        snprintf(nx, sizeof(nx), "%s_nx", in[i].arr);
        bprintf(b, "  float2 %s[TKG_KCH][TKG_VP];\n", nx);
        load_into(b, nx, in[i].src, in[i].stride, in[i].col0, "rown", "okn");
    }
    bprintf(b, "  for (; tkm_rb < TKG_NRB; tkm_rb += gridDim.x) {\n"
               "  const int row = tkm_rb * TKG_RPB + threadIdx.x / TKG_TPR;\n"
               "  const bool tkm_row_ok = row < TKG_ROWS;\n");
    for (int i = 0; i < nin; i++) {
        snprintf(nx, sizeof(nx), "%s_nx", in[i].arr);
        decl_array(b, in[i].arr);
        copy_array(b, in[i].arr, nx);
    }
    bprintf(b, "  {\n    const int rbn = tkm_rb + gridDim.x;\n"
               "    const int rown = rbn * TKG_RPB + threadIdx.x / TKG_TPR;\n"
               "    const bool okn = rbn < TKG_NRB && rown < TKG_ROWS;\n");
    for (int i = 0; i < nin; i++) {
        snprintf(nx, sizeof(nx), "%s_nx", in[i].arr);
        load_into(b, nx, in[i].src, in[i].stride, in[i].col0, "rown", "okn");
    }
    bprintf(b, "  }\n");
    declare_stats(e);
    if (e->pg->is_twin_epilogue) {
        for (int i = 0; i < L->nl; i++) emit_op_fwd(e, &e->g->nodes[L->ids[i]], "txl", 0);
        for (int i = L->nl; i < L->nl + L->nr; i++) emit_op_fwd(e, &e->g->nodes[L->ids[i]], "txr", 0);
        decl_array(b, "tx");
        bprintf(b, "  _Pragma(\"unroll\") for (int k = 0; k < TKG_KCH; ++k) _Pragma(\"unroll\") for (int q = 0; q < TKG_VP; ++q)\n"
                   "    tx[k][q] = make_float2(txl[k][q].x * txr[k][q].x, txl[k][q].y * txr[k][q].y);\n");
    }
    for (int i = L->nl + L->nr; i < L->n; i++) emit_op_fwd(e, &e->g->nodes[L->ids[i]], "tx", 0);
    store_array(b, A(e, KA_OUT, -1, 0), "TKG_C2", "0", "tx", 0);
    bprintf(b, "  }\n  }\n}\n\n");
}

static void emit_stage_issue(Em *e, const FwdInput *rin, int nin, const char *slot_fmt, int slot_val);

/* the forward chain of one row from its loaded inputs, and the store */
static void emit_fwd_body(Em *e) {
    Buf *b = e->b;
    const Lists *L = &e->L;
    if (e->pg->is_twin_epilogue) {
        for (int i = 0; i < L->nl; i++) emit_op_fwd(e, &e->g->nodes[L->ids[i]], "txl", 0);
        for (int i = L->nl; i < L->nl + L->nr; i++) emit_op_fwd(e, &e->g->nodes[L->ids[i]], "txr", 0);
        decl_array(b, "tx");
        bprintf(b, "  _Pragma(\"unroll\") for (int k = 0; k < TKG_KCH; ++k) _Pragma(\"unroll\") for (int q = 0; q < TKG_VP; ++q)\n"
                   "    tx[k][q] = make_float2(txl[k][q].x * txr[k][q].x, txl[k][q].y * txr[k][q].y);\n");
    }
    for (int i = L->nl + L->nr; i < L->n; i++) emit_op_fwd(e, &e->g->nodes[L->ids[i]], "tx", 0);
    store_array(b, A(e, KA_OUT, -1, 0), "TKG_C2", "0", "tx", 0);
}

/* Staged forward (tkm_group_fwd_stage_bytes).  TKG_STAGE_BYTES > 0:
 * persistent, the row inputs of the next TKG_NSLOT row blocks staged by cp.async in
 * dynamic shared memory; else (a normalisation group whose stages would not
 * fit) one row block per block. */
static void emit_plasma_fwd_rowblock(Em *e) {
    Buf *b = e->b;
    const Lists *L = &e->L;
    set_args(e, 0);
    e->acc_smem = 0;
    e->param_regs = 1;
    kernel_head(e, "fwd", 0);
    if (range_has_norm(e, 0, L->n)) bprintf(b, "  __shared__ float tkm_red[TKM_RED_SLOTS(TKG_TPR, TKG_RPB)];\n");
    emit_param_preload(e);
    FwdInput in[16];
    const int nin = fwd_inputs(e, in);
    bprintf(b, "#if TKG_STAGE_BYTES > 0\n"
               "  extern __shared__ uint4 tkm_dyn[];\n"
               "#define TKM_STG(s, a, k) tkm_dyn[(((s) * %d + (a)) * TKG_KCH + (k)) * TKG_THREADS + threadIdx.x]\n",
            nin);
    for (int ahead = 0; ahead < stage_slots(0); ahead++) {
        bprintf(b, "  {\n    const int rbn = blockIdx.x + %d * gridDim.x;\n", ahead);
        emit_stage_issue(e, in, nin, "%d", ahead);
        bprintf(b, "  }\n  tkm_cp_commit();\n");
    }
    bprintf(b, "  int tkm_it = 0;\n"
               "  for (int tkm_rb = blockIdx.x; tkm_rb < TKG_NRB; tkm_rb += gridDim.x, ++tkm_it) {\n"
               "  const int row = tkm_rb * TKG_RPB + threadIdx.x / TKG_TPR;\n"
               "  const bool tkm_row_ok = row < TKG_ROWS;\n"
               "  const int tkm_sl = tkm_it %% TKG_NSLOT;\n  tkm_cp_wait<TKG_NSLOT - 1>();\n");
    declare_stats(e);
    for (int i = 0; i < nin; i++) {
        decl_array(b, in[i].arr);
        bprintf(b, "  _Pragma(\"unroll\") for (int k = 0; k < TKG_KCH; ++k) tkm_lds<TKG_VP>(&TKM_STG(tkm_sl, %d, k), %s[k]);\n",
                i, in[i].arr);
    }
    bprintf(b, "  {\n    const int rbn = tkm_rb + TKG_NSLOT * gridDim.x;\n");
    emit_stage_issue(e, in, nin, "tkm_sl", -1);
    bprintf(b, "  }\n  tkm_cp_commit();\n");
    emit_fwd_body(e);
    bprintf(b, "  }\n  tkm_cp_wait<0>();\n#undef TKM_STG\n#else\n  {\n"
               "  const int row = blockIdx.x * TKG_RPB + threadIdx.x / TKG_TPR;\n"
               "  const bool tkm_row_ok = row < TKG_ROWS;\n");
    declare_stats(e);
    for (int i = 0; i < nin; i++) load_array(b, in[i].arr, in[i].src, in[i].stride, in[i].col0);
    emit_fwd_body(e);
    bprintf(b, "  }\n#endif\n}\n\n");
}

/* replays locals [lo, hi) on `arr`, keeping each operator's input in pre_<j>
 * when its backward reads it; with skip_last the last operator is not applied
 * (its output is the group output, which the backward never needs) unless it
 * is a normalisation, whose statistics the backward uses */
static void emit_replay(Em *e, int lo, int hi, const char *arr, int skip_last) {
    for (int i = lo; i < hi; i++) {
        const TkmNode *n = &e->g->nodes[e->L.ids[i]];
        if (needs_pre(n)) {
            char name[16];
            snprintf(name, sizeof(name), "tpre_%d", i);
            decl_array(e->b, name);
            copy_array(e->b, name, arr);
        }
        if (i == hi - 1 && skip_last && n->cat != CAT_NORM) continue;
        emit_op_fwd(e, n, arr, 1);
    }
}

static void emit_bwd_range(Em *e, int lo, int hi, const char *dy) {
    for (int i = hi - 1; i >= lo; i--) emit_op_bwd(e, &e->g->nodes[e->L.ids[i]], dy);
}

/* Parameter-gradient accumulators, one per channel pair a thread owns.  In
 * shared memory (slot (k * VP + q) * THREADS + thread: private to the thread,
 * conflict-free) they cost no registers, which lets more rows of a wide
 * normalisation be in flight per SM; very wide rows keep them in registers. */
static void declare_accs(Em *e) {
    for (int i = 0; i < e->L.n; i++) {
        const uint32_t f = node_flags(e->g, e->L.ids[i]);
        const uint32_t flags[3] = {RES_PARAM_WEIGHT, RES_PARAM_BETA, RES_PARAM_BIAS};
        for (int w = 0; w < 3; w++)
            if (f & flags[w]) {
                char name[24];
                snprintf(name, sizeof(name), "tacc_%s_%d", which_name(w), i);
                if (e->acc_smem) {
                    bprintf(e->b, "  __shared__ float2 %s[TKG_KCH * TKG_VP * TKG_THREADS];\n"
                                  "  _Pragma(\"unroll\") for (int k = 0; k < TKG_KCH; ++k) _Pragma(\"unroll\") for (int q = 0; q < TKG_VP; ++q)\n"
                                  "    TKM_ACC(%s) = make_float2(0.f, 0.f);\n",
                            name, name);
                } else {
                    decl_array(e->b, name);
                    zero_array(e->b, name);
                }
            }
    }
}

/* shared-memory bytes of the accumulators of the group's backward kernel
 * (the larger of the two storage types' geometries) */
static long acc_smem_bytes(Em *e) {
    int nodes[64], which[64];
    const int np = tkm_group_params(e->g, e->pg, nodes, which);
    long worst = 0;
    for (int ab = 2; ab <= 4; ab += 2) {
        TkmRowGeom gm;
        tkm_row_geom_bwd(e->g, e->pg, ab, &gm);
        const long bytes = (long)np * gm.kch * gm.vp * gm.threads * 8;
        if (bytes > worst) worst = bytes;
    }
    return worst;
}

/* one partial row of every reduced parameter gradient per block */
static void emit_partials(Em *e, int qkv) {
    int nodes[64], which[64];
    const int np = tkm_group_params(e->g, e->pg, nodes, which);
    if (!np) return;
    Buf *b = e->b;
    if (!e->acc_smem)
        bprintf(b, "  __shared__ float2 tkm_pbuf[TKG_RPB > 1 ? TKG_THREADS * TKG_KCH * TKG_VP : 1];\n");
    else
        bprintf(b, "  if (TKG_RPB > 1) __syncthreads();\n");
    for (int p = 0; p < np; p++) {
        char acc[24];
        snprintf(acc, sizeof(acc), "tacc_%s_%d", which_name(which[p]), qkv ? 0 : local_of(e, nodes[p]));
        if (e->acc_smem)
            bprintf(b, "  tkm_block_partial_s<TKG_VP, TKG_KCH, TKG_TPR, TKG_RPB, TKG_NCH, TKG_THREADS>(%s, %s + ((size_t)%d * gridDim.x + blockIdx.x) * TKG_C2, tkm_lr, tkm_ll);\n",
                    acc, A(e, KA_PART, -1, 0), p);
        else
            bprintf(b, "  tkm_block_partial<TKG_VP, TKG_KCH, TKG_TPR, TKG_RPB, TKG_NCH>(%s, %s + ((size_t)%d * gridDim.x + blockIdx.x) * TKG_C2, tkm_pbuf, tkm_lr, tkm_ll);\n",
                    acc, A(e, KA_PART, -1, 0), p);
    }
}


/* cp.async of every input chunk of row block `rbn` (a variable of the
 * emitted code) into stage slot `slot_fmt` (a printf format with one int, or
 * a variable name when slot_val < 0) */
static void emit_stage_issue(Em *e, const FwdInput *rin, int nin, const char *slot_fmt, int slot_val) {
    Buf *b = e->b;
    char slot[24];
    if (slot_val >= 0) snprintf(slot, sizeof(slot), slot_fmt, slot_val);
    else snprintf(slot, sizeof(slot), "%s", slot_fmt);
    bprintf(b, "    const int rown = rbn * TKG_RPB + threadIdx.x / TKG_TPR;\n"
               "    const bool okn = rbn < TKG_NRB && rown < TKG_ROWS;\n");
    for (int i = 0; i < nin; i++)
        bprintf(b, "    _Pragma(\"unroll\") for (int k = 0; k < TKG_KCH; ++k) {\n"
                   "      const int tkm_ch = tkm_lr + k * TKG_TPR;\n"
                   "      tkm_cp<TKG_VP>(&TKM_STG(%s, %d, k), %s, (long long)rown * %s + %s + tkm_ch * TKG_VP,\n"
                   "                     okn && tkm_ch < TKG_NCH);\n    }\n",
                slot, i, rin[i].src, rin[i].stride, rin[i].col0);
}

/* backward of a group-closing RMSNorm from its input tx and dy = tg */
static void emit_rmsnorm_last_bwd(Em *e, const TkmNode *n) {
    Buf *b = e->b;
    const int j = local_of(e, n->id);
    const uint32_t f = node_flags(e->g, n->id);
    char gm[48];
    if (f & RES_PARAM_WEIGHT) snprintf(gm, sizeof(gm), "%s", pexpr(e, n, 0));
    else snprintf(gm, sizeof(gm), "make_float2(1.f, 1.f)");
    bprintf(b, "  { /* backward RMSNorm, one reduction */\n    const float eps = ");
    emit_float(b, n->fval);
    bprintf(b, ";\n    float2 m = make_float2(0.f, 0.f);\n");
    pairs_begin(b);
    bprintf(b, "          const float2 x = tx[k][q], gy = tg[k][q], gm = %s;\n"
               "          m.x += x.x * x.x + x.y * x.y;\n"
               "          m.y += gy.x * gm.x * x.x + gy.y * gm.y * x.y;\n",
            gm);
    pairs_end(b);
    bprintf(b, "    m = tkm_row_sum2<TKG_TPR, TKG_RPB>(m, tkm_red2);\n"
               "    const float istd = rsqrtf(m.x * TKG_INV_C + eps), m2 = istd * m.y * TKG_INV_C;\n");
    pairs_begin(b);
    bprintf(b, "          const float2 x = tx[k][q], gy = tg[k][q], gm = %s;\n"
               "          const float2 xh = make_float2(x.x * istd, x.y * istd);\n",
            gm);
    if (f & RES_PARAM_WEIGHT)
        bprintf(b, "          TKM_ACC(tacc_w_%d).x += gy.x * xh.x; TKM_ACC(tacc_w_%d).y += gy.y * xh.y;\n", j, j);
    bprintf(b, "          tg[k][q] = make_float2(istd * (gy.x * gm.x - xh.x * m2), istd * (gy.y * gm.y - xh.y * m2));\n");
    pairs_end(b);
    bprintf(b, "  }\n");
}

static void emit_plasma_bwd(Em *e) {
    Buf *b = e->b;
    const Lists *L = &e->L;
    const int din_acc = e->plan->group_din_acc[e->pg->id] > 0;
    set_args(e, 1);
    /* measured on the norm and twin backward kernels: accumulators in shared
     * memory plus parameters in registers beat every other combination */
    e->acc_smem = acc_smem_bytes(e) <= 64 * 1024;
    e->param_regs = 1;
    bprintf(b, e->acc_smem ? "#define TKM_ACC(a) a[(k * TKG_VP + q) * TKG_THREADS + threadIdx.x]\n"
                           : "#define TKM_ACC(a) a[k][q]\n");
    kernel_head(e, "bwd", 0);
    if (range_has_norm(e, 0, L->n))
        bprintf(b, "  __shared__ float tkm_red[TKM_RED_SLOTS(TKG_TPR, TKG_RPB)];\n"
                   "  __shared__ float2 tkm_red2[TKM_RED_SLOTS(TKG_TPR, TKG_RPB)];\n");
    declare_accs(e);
    if (e->param_regs) emit_param_preload(e);
    const char *in = A(e, KA_IN, -1, 0);
    /* every input of the row is requested before any row statistics */
    const int last = L->n - 1;
    const int skip = (L->nc > 0 && e->g->nodes[L->ids[last]].cat != CAT_NORM) ? last : -1;
    FwdInput rin[16];
    int nin = 0;
    const int need_x = bwd_needs_input(e->g, e->pg);
    if (e->pg->is_twin_epilogue) {
        rin[nin++] = (FwdInput){"txl", in, "(2 * TKG_C2)", "0"};
        rin[nin++] = (FwdInput){"txr", in, "(2 * TKG_C2)", "TKG_C2"};
    } else if (need_x) {
        rin[nin++] = (FwdInput){"tx", in, "TKG_C2", "0"};
    }
    rin[nin++] = (FwdInput){"tg", A(e, KA_DOUT, -1, 0), "TKG_C2", "0"};
    for (int i = 0; i < L->n && nin < 16 && need_x; i++) {
        const TkmNode *nd = &e->g->nodes[L->ids[i]];
        if (nd->op != OP_ADD || i == skip) continue;
        FwdInput f = {"", A(e, KA_BRANCH, nd->id, 0), "TKG_C2", "0"};
        snprintf(f.arr, sizeof(f.arr), "tbr_%d", i);
        rin[nin++] = f;
    }
    /* TKG_STAGE_BYTES > 0 (per storage type, tkm_group_bwd_stage_bytes):
     * rows are staged TKG_NSLOT row blocks ahead by cp.async into dynamic
     * shared-memory slots private to each thread, so that their loads are in
     * flight while the current row computes, without holding registers. */
    bprintf(b, "#if TKG_STAGE_BYTES > 0\n"
               "  extern __shared__ uint4 tkm_dyn[];\n"
               "#define TKM_STG(s, a, k) tkm_dyn[(((s) * %d + (a)) * TKG_KCH + (k)) * TKG_THREADS + threadIdx.x]\n",
            nin);
    for (int ahead = 0; ahead < stage_slots(1); ahead++) {
        bprintf(b, "  {\n    const int rbn = blockIdx.x + %d * gridDim.x;\n", ahead);
        emit_stage_issue(e, rin, nin, "%d", ahead);
        bprintf(b, "  }\n  tkm_cp_commit();\n");
    }
    bprintf(b, "#endif\n  int tkm_it = 0; (void)tkm_it;\n");
    bprintf(b, "  for (int tkm_rb = blockIdx.x; tkm_rb < TKG_NRB; tkm_rb += gridDim.x, ++tkm_it) {\n"
               "  const int row = tkm_rb * TKG_RPB + threadIdx.x / TKG_TPR;\n"
               "  const bool tkm_row_ok = row < TKG_ROWS;\n");
    declare_stats(e);
    const int alias_add = first_aliased_add(e);
    if (alias_add >= 0)
        bprintf(b, "  float2 tdbr[TKG_KCH][TKG_VP];\n"
                   "  _Pragma(\"unroll\") for (int k = 0; k < TKG_KCH; ++k) _Pragma(\"unroll\") for (int q = 0; q < TKG_VP; ++q)\n"
                   "    tdbr[k][q] = make_float2(0.f, 0.f);\n");
    bprintf(b, "#if TKG_STAGE_BYTES > 0\n  const int tkm_sl = tkm_it %% TKG_NSLOT;\n  tkm_cp_wait<TKG_NSLOT - 1>();\n");
    for (int i = 0; i < nin; i++) {
        decl_array(b, rin[i].arr);
        bprintf(b, "  _Pragma(\"unroll\") for (int k = 0; k < TKG_KCH; ++k) tkm_lds<TKG_VP>(&TKM_STG(tkm_sl, %d, k), %s[k]);\n",
                i, rin[i].arr);
    }
    bprintf(b, "  {\n    const int rbn = tkm_rb + TKG_NSLOT * gridDim.x;\n");
    emit_stage_issue(e, rin, nin, "tkm_sl", -1);
    bprintf(b, "  }\n  tkm_cp_commit();\n#else\n");
    for (int i = 0; i < nin; i++) load_array(b, rin[i].arr, rin[i].src, rin[i].stride, rin[i].col0);
    bprintf(b, "#endif\n");
    if (e->pg->is_twin_epilogue) {
        emit_replay(e, 0, L->nl, "txl", 0);
        emit_replay(e, L->nl, L->nl + L->nr, "txr", 0);
        decl_array(b, "tx");
        bprintf(b, "  _Pragma(\"unroll\") for (int k = 0; k < TKG_KCH; ++k) _Pragma(\"unroll\") for (int q = 0; q < TKG_VP; ++q)\n"
                   "    tx[k][q] = make_float2(txl[k][q].x * txr[k][q].x, txl[k][q].y * txr[k][q].y);\n");
    }
    const TkmNode *lastn = &e->g->nodes[L->ids[L->n - 1]];
    int nnorm = 0;
    for (int i = L->nl + L->nr; i < L->n; i++) nnorm += e->g->nodes[L->ids[i]].cat == CAT_NORM;
    if (!e->pg->is_twin_epilogue && lastn->op == OP_RMSNORM && nnorm == 1) {
        /* RMSNorm closes the group: its dy is dout, so sum(x^2) and
         * sum(dy * gain * x) come from one row reduction (mean(dy gain xh) =
         * istd * mean(dy gain x)) instead of the replay's and the backward's
         * two dependent ones */
        emit_replay(e, L->nl + L->nr, L->n - 1, "tx", 0);
        emit_rmsnorm_last_bwd(e, lastn);
        emit_bwd_range(e, L->nl + L->nr, L->n - 1, "tg");
    } else {
        if (need_x) emit_replay(e, L->nl + L->nr, L->n, "tx", 1);
        emit_bwd_range(e, L->nl + L->nr, L->n, "tg");
    }
    const char *din = A(e, KA_DIN, -1, 0);
    if (e->pg->is_twin_epilogue) {
        decl_array(b, "tgl");
        decl_array(b, "tgr");
        bprintf(b, "  _Pragma(\"unroll\") for (int k = 0; k < TKG_KCH; ++k) _Pragma(\"unroll\") for (int q = 0; q < TKG_VP; ++q) {\n"
                   "    tgl[k][q] = make_float2(tg[k][q].x * txr[k][q].x, tg[k][q].y * txr[k][q].y);\n"
                   "    tgr[k][q] = make_float2(tg[k][q].x * txl[k][q].x, tg[k][q].y * txl[k][q].y);\n  }\n");
        emit_bwd_range(e, 0, L->nl, "tgl");
        emit_bwd_range(e, L->nl, L->nl + L->nr, "tgr");
        store_array(b, din, "(2 * TKG_C2)", "0", "tgl", din_acc);
        store_array(b, din, "(2 * TKG_C2)", "TKG_C2", "tgr", din_acc);
    } else if (alias_add >= 0) {
        /* the residual branches that feed back into the group input, summed
         * with it; the first planned of these writes decides overwrite or
         * accumulate */
        bprintf(b, "  _Pragma(\"unroll\") for (int k = 0; k < TKG_KCH; ++k) _Pragma(\"unroll\") for (int q = 0; q < TKG_VP; ++q) {\n"
                   "    tg[k][q].x += tdbr[k][q].x; tg[k][q].y += tdbr[k][q].y;\n  }\n");
        store_array(b, din, "TKG_C2", "0", "tg", e->plan->add_branch_acc[alias_add] > 0);
    } else {
        store_array(b, din, "TKG_C2", "0", "tg", din_acc);
    }
    bprintf(b, "  }\n");
    bprintf(b, "#if TKG_STAGE_BYTES > 0\n  tkm_cp_wait<0>();  /* no copy into shared memory outlives the block */\n"
               "#undef TKM_STG\n#endif\n");
    emit_partials(e, 0);
    bprintf(b, "}\n#undef TKM_ACC\n\n");
}

/* QKV prep (reference src/tkm_codegen.c:211-295, rule src/tkm_registry.c:688-770):
 * bias over every channel, then per 64-wide Q/K head an RMS normalisation
 * with a per-channel gain (QKNorm, eps 1e-5), then RoPE on the Q and K heads:
 * pair i of a head rotates by pos * inv_freq[i], pos = row % S.  The cos/sin
 * table [S][D/2] is computed by the runtime in double precision. */
static void emit_qkv_prep(Em *e) {
    Buf *b = e->b;
    const TkmNode *n = &e->g->nodes[e->pg->node_ids[0]];
    const int hd2 = n->head_dim / 2, qk2 = (n->q_c + n->k_c) / 2, S = e->pg->H * e->pg->W;
    const int din_acc = e->plan->group_din_acc[e->pg->id] > 0;
    e->acc_smem = 0;
    e->param_regs = 0;
    bprintf(b, "#define TKG_HD2 %d\n#define TKG_QK2 %d\n#define TKG_SEQ %d\n#define TKG_CPH (TKG_HD2 / TKG_VP)\n", hd2, qk2,
            S > 0 ? S : 1);

    /* forward: persistent over row blocks; the next row block's inputs and
     * cos/sin pairs are requested before the current one is computed, the
     * per-channel bias and gains are loaded once */
    set_args(e, 0);
    kernel_head(e, "fwd", 0);
    bprintf(b, "  float2 tqb[TKG_KCH][TKG_VP], tqg[TKG_KCH][TKG_VP];\n"
               "  _Pragma(\"unroll\") for (int k = 0; k < TKG_KCH; ++k) {\n"
               "    const int tkm_ch = tkm_lr + k * TKG_TPR;\n"
               "    _Pragma(\"unroll\") for (int q = 0; q < TKG_VP; ++q) {\n"
               "      tqb[k][q] = tkm_ch < TKG_NCH ? __ldg(&%s[tkm_ch * TKG_VP + q]) : make_float2(0.f, 0.f);\n",
            A(e, KA_PARAM, n->id, 2));
    if (n->has_qknorm)
        bprintf(b, "      tqg[k][q] = (tkm_ch < TKG_NCH && tkm_ch * TKG_VP < TKG_QK2) ? __ldg(&%s[tkm_ch * TKG_VP + q])"
                   " : make_float2(1.f, 1.f);\n",
                A(e, KA_PARAM, n->id, 0));
    else
        bprintf(b, "      tqg[k][q] = make_float2(1.f, 1.f);\n");
    bprintf(b, "    }\n  }\n"
               "  float2 tx_nx[TKG_KCH][TKG_VP], tcs_nx[TKG_KCH][TKG_VP];\n"
               "  int tkm_rb = blockIdx.x;\n"
               "#define TKM_QKV_NEXT(rbv) {\\\n"
               "    const int rown = (rbv) * TKG_RPB + threadIdx.x / TKG_TPR;\\\n"
               "    const bool okn = (rbv) < TKG_NRB && rown < TKG_ROWS;\\\n"
               "    const int posn = rown %% TKG_SEQ; (void)posn;\\\n"
               "    _Pragma(\"unroll\") for (int k = 0; k < TKG_KCH; ++k) {\\\n"
               "      const int tkm_ch = tkm_lr + k * TKG_TPR;\\\n"
               "      if (okn && tkm_ch < TKG_NCH) tkm_ld<TKG_VP>(%s, (long long)rown * TKG_C2 + tkm_ch * TKG_VP, tx_nx[k]);\\\n"
               "      else tkm_zero<TKG_VP>(tx_nx[k]);\\\n"
               "      _Pragma(\"unroll\") for (int q = 0; q < TKG_VP; ++q) {\\\n"
               "        const int tid = tkm_ch * TKG_VP + q;\\\n",
            A(e, KA_IN, -1, 0));
    if (n->has_rope)
        bprintf(b, "        tcs_nx[k][q] = (okn && tkm_ch < TKG_NCH && tid < TKG_QK2)"
                   " ? __ldg(&%s[(size_t)posn * TKG_HD2 + (tid %% TKG_HD2)]) : make_float2(1.f, 0.f);\\\n",
                A(e, KA_ROPE, -1, 0));
    else
        bprintf(b, "        tcs_nx[k][q] = make_float2(1.f, 0.f); (void)tid;\\\n");
    bprintf(b, "      }\\\n    }\\\n  }\n"
               "  TKM_QKV_NEXT(tkm_rb)\n"
               "  for (; tkm_rb < TKG_NRB; tkm_rb += gridDim.x) {\n"
               "  const int row = tkm_rb * TKG_RPB + threadIdx.x / TKG_TPR;\n"
               "  const bool tkm_row_ok = row < TKG_ROWS;\n");
    decl_array(b, "tx");
    decl_array(b, "tcs");
    copy_array(b, "tx", "tx_nx");
    copy_array(b, "tcs", "tcs_nx");
    bprintf(b, "  TKM_QKV_NEXT(tkm_rb + gridDim.x)\n"
               "  _Pragma(\"unroll\") for (int k = 0; k < TKG_KCH; ++k) {\n"
               "    const int tkm_ch = tkm_lr + k * TKG_TPR;\n"
               "    float ss = 0.f;\n"
               "    _Pragma(\"unroll\") for (int q = 0; q < TKG_VP; ++q) {\n"
               "      tx[k][q].x += tqb[k][q].x; tx[k][q].y += tqb[k][q].y;\n"
               "      ss += tx[k][q].x * tx[k][q].x + tx[k][q].y * tx[k][q].y;\n"
               "    }\n");
    if (n->has_qknorm) {
        bprintf(b, "    const float istd = rsqrtf(tkm_group_sum<TKG_CPH>(ss) * ");
        emit_float(b, 1.0 / n->head_dim);
        bprintf(b, " + 1e-5f);\n"
                   "    const bool tkm_qk = tkm_ch * TKG_VP < TKG_QK2;\n"
                   "    _Pragma(\"unroll\") for (int q = 0; q < TKG_VP; ++q) if (tkm_qk)\n"
                   "      tx[k][q] = make_float2(tx[k][q].x * istd * tqg[k][q].x, tx[k][q].y * istd * tqg[k][q].y);\n");
    } else {
        bprintf(b, "    (void)ss; (void)tkm_ch; (void)tqg;\n");
    }
    if (n->has_rope)
        bprintf(b, "    _Pragma(\"unroll\") for (int q = 0; q < TKG_VP; ++q) {\n"
                   "      const float2 v = tx[k][q], cs = tcs[k][q];\n"
                   "      tx[k][q] = make_float2(v.x * cs.x - v.y * cs.y, v.x * cs.y + v.y * cs.x);\n"
                   "    }\n");
    bprintf(b, "  }\n");
    store_array(b, A(e, KA_OUT, -1, 0), "TKG_C2", "0", "tx", 0);
    bprintf(b, "  }\n#undef TKM_QKV_NEXT\n}\n\n");

    set_args(e, 1);
    kernel_head(e, "bwd", 0);
    decl_array(b, "tacc_b_0");
    zero_array(b, "tacc_b_0");
    if (n->has_qknorm) {
        decl_array(b, "tacc_w_0");
        zero_array(b, "tacc_w_0");
    }
    bprintf(b, "  for (int tkm_rb = blockIdx.x; tkm_rb < TKG_NRB; tkm_rb += gridDim.x) {\n"
               "  const int row = tkm_rb * TKG_RPB + threadIdx.x / TKG_TPR;\n"
               "  const bool tkm_row_ok = row < TKG_ROWS;\n"
               "  const int pos = row %% TKG_SEQ; (void)pos;\n");
    load_array(b, "tg", A(e, KA_DOUT, -1, 0), "TKG_C2", "0");
    if (n->has_rope) {
        pairs_begin(b);
        bprintf(b, "          if (tid < TKG_QK2) {\n"
                   "            const float2 cs = %s[(size_t)pos * TKG_HD2 + (tid %% TKG_HD2)];\n"
                   "            const float2 d = tg[k][q];\n"
                   "            tg[k][q] = make_float2(d.x * cs.x + d.y * cs.y, d.y * cs.x - d.x * cs.y);\n"
                   "          }\n",
                A(e, KA_ROPE, -1, 0));
        pairs_end(b);
    }
    if (n->has_qknorm) {
        load_array(b, "tx", A(e, KA_IN, -1, 0), "TKG_C2", "0");
        bprintf(b, "  _Pragma(\"unroll\") for (int k = 0; k < TKG_KCH; ++k) {\n"
                   "    const int tkm_ch = tkm_lr + k * TKG_TPR;\n"
                   "    const bool in_row = tkm_row_ok && tkm_ch < TKG_NCH;\n"
                   "    const bool qk = in_row && tkm_ch * TKG_VP < TKG_QK2;\n"
                   "    float ss = 0.f, m2 = 0.f;\n"
                   "    float2 xh[TKG_VP], gm[TKG_VP];\n"
                   "    _Pragma(\"unroll\") for (int q = 0; q < TKG_VP; ++q) {\n"
                   "      const int tid = tkm_ch * TKG_VP + q;\n"
                   "      const float2 bb = in_row ? %s[tid] : make_float2(0.f, 0.f);\n"
                   "      xh[q] = make_float2(tx[k][q].x + bb.x, tx[k][q].y + bb.y);\n"
                   "      ss += xh[q].x * xh[q].x + xh[q].y * xh[q].y;\n"
                   "      gm[q] = qk ? %s[tid] : make_float2(1.f, 1.f);\n"
                   "    }\n"
                   "    const float istd = rsqrtf(tkm_group_sum<TKG_CPH>(ss) * ",
                A(e, KA_PARAM, n->id, 2), A(e, KA_PARAM, n->id, 0));
        emit_float(b, 1.0 / n->head_dim);
        bprintf(b, " + 1e-5f);\n"
                   "    _Pragma(\"unroll\") for (int q = 0; q < TKG_VP; ++q) {\n"
                   "      xh[q].x *= istd; xh[q].y *= istd;\n"
                   "      m2 += tg[k][q].x * gm[q].x * xh[q].x + tg[k][q].y * gm[q].y * xh[q].y;\n"
                   "    }\n"
                   "    m2 = tkm_group_sum<TKG_CPH>(m2) * ");
        emit_float(b, 1.0 / n->head_dim);
        bprintf(b, ";\n"
                   "    if (qk) {\n"
                   "      _Pragma(\"unroll\") for (int q = 0; q < TKG_VP; ++q) {\n"
                   "        const float2 d = tg[k][q];\n"
                   "        tacc_w_0[k][q].x += d.x * xh[q].x; tacc_w_0[k][q].y += d.y * xh[q].y;\n"
                   "        tg[k][q] = make_float2(istd * (d.x * gm[q].x - xh[q].x * m2), istd * (d.y * gm[q].y - xh[q].y * m2));\n"
                   "      }\n    }\n  }\n");
    }
    pairs_begin(b);
    bprintf(b, "          tacc_b_0[k][q].x += tg[k][q].x; tacc_b_0[k][q].y += tg[k][q].y;\n");
    pairs_end(b);
    store_array(b, A(e, KA_DIN, -1, 0), "TKG_C2", "0", "tg", din_acc);
    bprintf(b, "  }\n");
    emit_partials(e, 1);
    bprintf(b, "}\n\n#undef TKG_HD2\n#undef TKG_QK2\n#undef TKG_SEQ\n#undef TKG_CPH\n");
}

/* finalize: d_param[c] = sum of the partial rows, two fixed-order stages
 * (stage 1 over segments of rows, stage 2 over the segment sums) */
static void emit_finalize(Em *e) {
    int nodes[64], which[64];
    const int np = tkm_group_params(e->g, e->pg, nodes, which);
    if (!np) return;
    Buf *b = e->b;
    bprintf(b, "extern \"C\" __global__ void __launch_bounds__(256) TKM_KNAME(fin)(float2* __restrict__ part, int nblk, int stage");
    for (int p = 0; p < np; p++) bprintf(b, ", float* __restrict__ d%d", p);
    bprintf(b, ") {\n  float* dst = nullptr;\n  switch (blockIdx.y) {\n");
    for (int p = 0; p < np; p++) bprintf(b, "    case %d: dst = d%d; break;\n", p, p);
    bprintf(b, "    default: return;\n  }\n  tkm_colsum_pairs(part + (size_t)blockIdx.y * nblk * TKG_C2, nblk, TKG_C2, stage, dst);\n}\n");
}

/* canonical code of one group (kernel names through TKM_KNAME) */
static void emit_group_body(const TkmGraph *g, const PlasmaGroup *pg, const TkmGradPlan *plan, Buf *b) {
    Em e;
    memset(&e, 0, sizeof(e));
    e.g = g;
    e.pg = pg;
    e.plan = plan;
    e.b = b;
    group_lists(g, pg, &e.L);
    emit_geom_macros(&e, 0);
    if (pg->is_qkv_prep) {
        emit_qkv_prep(&e);
    } else {
        emit_plasma_fwd(&e);
        undef_geom(b);
        emit_geom_macros(&e, 1);
        emit_plasma_bwd(&e);
    }
    emit_finalize(&e);
    undef_geom(b);
}

/* texts[i] = canonical code of group i; class_of[i] = first group with equal text */
static int build_classes(const TkmGraph *g, const TkmGradPlan *plan, char **texts, int *class_of) {
    int nclass = 0, rep[TKM_MAX_GROUPS];
    for (int i = 0; i < g->num_groups; i++) {
        Buf b = {0};
        if (!group_unsupported(g, &g->groups[i])) emit_group_body(g, &g->groups[i], plan, &b);
        texts[i] = b.s;
        if (b.oom) return -1;
        class_of[i] = -1;
        if (!texts[i]) continue;
        for (int c = 0; c < nclass; c++)
            if (!strcmp(texts[rep[c]], texts[i])) {
                class_of[i] = c;
                break;
            }
        if (class_of[i] < 0) {
            rep[nclass] = i;
            class_of[i] = nclass++;
        }
    }
    return nclass;
}

int tkm_codegen_classes(const TkmGraph *g, int *class_of) {
    TkmGradPlan *plan = (TkmGradPlan *)calloc(1, sizeof(TkmGradPlan));
    char **texts = (char **)calloc(TKM_MAX_GROUPS, sizeof(char *));
    int n = -1;
    if (plan && texts) {
        tkm_plan_grads(g, plan);
        n = build_classes(g, plan, texts, class_of);
    }
    if (texts)
        for (int i = 0; i < TKM_MAX_GROUPS; i++) free(texts[i]);
    free(texts);
    free(plan);
    return n;
}

char *tkm_codegen_cuda_string(const TkmGraph *g) {
    Buf out = {0};
    bprintf(&out, "%s\n", TKM_CODEGEN_MARKER);
    if (!g) return out.s;
    TkmGradPlan *plan = (TkmGradPlan *)calloc(1, sizeof(TkmGradPlan));
    char **texts = (char **)calloc(TKM_MAX_GROUPS, sizeof(char *));
    int class_of[TKM_MAX_GROUPS];
    if (!plan || !texts) {
        free(plan);
        free(texts);
        free(out.s);
        return NULL;
    }
    tkm_plan_grads(g, plan);
    const int nclass = build_classes(g, plan, texts, class_of);
    bprintf(&out, "/* %d plasma groups in %d kernel classes, batch %d.  Compiled behind the runtime's prelude,\n"
                  "   which defines TKM_ACT_BYTES (2: bf16 activations, 4: fp32). */\n\n",
            g->num_groups, nclass < 0 ? 0 : nclass, g->batch_size);
    for (int i = 0; i < g->num_groups; i++) {
        const PlasmaGroup *pg = &g->groups[i];
        bprintf(&out, "/* group %d: anchor #%d -> output #%d, C=%d%s%s", i, pg->anchor_id, pg->out_node_id, pg->C,
                pg->is_twin_epilogue ? ", twin epilogue" : "", pg->is_qkv_prep ? ", QKV prep" : "");
        const char *why = group_unsupported(g, pg);
        if (why) {
            bprintf(&out, " */\n#error \"plasma group %d: %s\"\n\n", i, why);
            continue;
        }
        if (class_of[i] >= 0 && texts[i] && i > 0) {
            int first = -1;
            for (int k = 0; k < i; k++)
                if (class_of[k] == class_of[i]) {
                    first = k;
                    break;
                }
            if (first >= 0) {
                bprintf(&out, "; kernels of class %d */\n\n", class_of[i]);
                continue;
            }
        }
        bprintf(&out, "; class %d */\n#define TKM_KNAME(part) tkm_c%d_##part\n%s#undef TKM_KNAME\n\n", class_of[i],
                class_of[i], texts[i] ? texts[i] : "");
    }
    for (int i = 0; i < TKM_MAX_GROUPS; i++) free(texts[i]);
    free(texts);
    free(plan);
    if (out.oom) {
        free(out.s);
        return NULL;
    }
    return out.s;
}
