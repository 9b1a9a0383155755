/*
 * tkm_graph.c -- .tkm DSL front end: parser (with the `block x N:` loop macro),
 * shape inference, fusion + plasma grouping with kernel-ABI binding, arena
 * planning, summary and registry verification.
 *
 * Behaviour follows the reference's src/tkm_core.c so that a .tkm file yields
 * the same TkmGraph (node ids, tags, arguments, dead flags, groups, kernel
 * signatures and arena offsets): the grammar of parse_statement_block /
 * parse_chain / parse_step / parse_args (tkm_core.c:15-247), the shape rules
 * of tkm_infer_shapes (:259-289), the group formation of tkm_optimize_and_bind
 * (:369-549) with build_group_abi (:333-367) and the sequential arena of
 * tkm_plan_memory (:551-577).  Malformed graphs produce an error message and
 * an empty graph instead of exit(1).
 */
#include <ctype.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "tkm_internal.h"

/* ------------------------------------------------------------ diagnostics */

static __thread char g_err[1024];

const char *tkm_last_error(void) { return g_err; }

void tkm_clear_error(void) { g_err[0] = 0; }

void tkm_set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    fprintf(stderr, "%s\n", g_err);
}

void tkm_graph_error(TkmGraph *g, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    fprintf(stderr, "%s\n", g_err);
    if (g) {
        g->num_nodes = 0;
        g->num_groups = 0;
    }
}

int tkm_verbose(void) {
    static int v = -1;
    if (v < 0) {
        const char *e = getenv("TKM_VERBOSE");
        v = (e && *e && strcmp(e, "0") != 0) ? 1 : 0;
    }
    return v;
}

void tkm_log(const char *fmt, ...) {
    if (!tkm_verbose()) return;
    va_list ap;
    va_start(ap, fmt);
    vprintf(fmt, ap);
    va_end(ap);
}

/* ----------------------------------------------------------------- lexing */

typedef struct {
    const char *p;
    TkmGraph *g;
    int failed;
} Lex;

static void lx_ws(Lex *L) {
    for (;;) {
        while (isspace((unsigned char)*L->p)) L->p++;
        if (*L->p != '#') return;
        while (*L->p && *L->p != '\n') L->p++;
    }
}

static int lx_word_char(char c) { return isalnum((unsigned char)c) || c == '_'; }

/* identifier (letters, digits, '_'), truncated to cap-1 characters */
static void lx_ident(Lex *L, char *out, size_t cap) {
    lx_ws(L);
    size_t n = 0;
    while (lx_word_char(*L->p)) {
        if (n + 1 < cap) out[n++] = *L->p;
        L->p++;
    }
    out[n] = 0;
}

static float lx_number(Lex *L) {
    lx_ws(L);
    char *end;
    float v = strtof(L->p, &end);
    L->p = end;
    return v;
}

static int lx_keyword(Lex *L, const char *kw) {
    lx_ws(L);
    const size_t n = strlen(kw);
    if (strncmp(L->p, kw, n) || lx_word_char(L->p[n])) return 0;
    L->p += n;
    return 1;
}

static int lx_arrow(Lex *L) {
    lx_ws(L);
    if (L->p[0] == '-' && L->p[1] == '>') {
        L->p += 2;
        return 1;
    }
    return 0;
}

static void lx_skip_char(Lex *L, char c) {
    lx_ws(L);
    if (*L->p == c) L->p++;
}

/* ------------------------------------------------------------------ nodes */

static int add_node(Lex *L, const TkmOpSpec *spec, int in0, int in1, int in2, const char *tag) {
    TkmGraph *g = L->g;
    if (g->num_nodes >= TKM_MAX_NODES) {
        tkm_graph_error(g, "[TKM Error] graph exceeds %d nodes", TKM_MAX_NODES);
        L->failed = 1;
        return -1;
    }
    const int id = g->num_nodes++;
    TkmNode *n = &g->nodes[id];
    memset(n, 0, sizeof(*n));
    n->id = id;
    n->spec_id = tkm_get_spec_index(spec);
    n->op = spec ? spec->op : OP_INPUT;
    n->cat = spec ? spec->cat : CAT_META;
    n->in0 = in0;
    n->in1 = in1;
    n->in2 = in2;
    n->plasma_grp = -1;
    n->out_buf_id = -1;
    n->k = 1;
    n->s = 1;
    n->p = 0;
    n->fval = spec ? spec->default_fval : 0.0f;
    n->fval2 = 4.0f;
    n->rope_theta = 10000.0f;
    n->rope_scale = 1.0f;
    n->rope_low_freq_factor = 1.0f;
    n->rope_high_freq_factor = 4.0f;
    n->rope_original_context_length = 8192.0f;
    n->rng_type = RNG_DEFAULT;
    snprintf(n->tag, sizeof(n->tag), "%s_%d", tag ? tag : (spec ? spec->dsl_name : "input"), id);
    return id;
}

static int is_true_word(const char *w) { return !strcmp(w, "true") || !strcmp(w, "causal") || !strcmp(w, "1"); }

static void set_keyed_arg(TkmNode *n, const char *key, float v) {
    static const struct { const char *key; int field; } keys[] = {
        {"c", 0}, {"out", 0}, {"k", 1}, {"s", 2}, {"p", 3}, {"q", 4}, {"kv", 5}, {"d", 6},
        {"theta", 7}, {"scale", 8}, {"low_freq_factor", 9}, {"high_freq_factor", 10},
        {"original_context_length", 11}, {"r", 12}, {"sigma", 12}, {"radius", 12},
    };
    for (size_t i = 0; i < sizeof(keys) / sizeof(keys[0]); i++) {
        if (strcmp(key, keys[i].key)) continue;
        switch (keys[i].field) {
            case 0: n->c_out = (int)v; return;
            case 1: n->k = (int)v; return;
            case 2: n->s = (int)v; return;
            case 3: n->p = (int)v; return;
            case 4: n->q_heads = (int)v; return;
            case 5: n->kv_heads = (int)v; return;
            case 6: n->head_dim = (int)v; return;
            case 7: n->rope_theta = v; return;
            case 8: n->rope_scale = v; return;
            case 9: n->rope_low_freq_factor = v; return;
            case 10: n->rope_high_freq_factor = v; return;
            case 11: n->rope_original_context_length = v; return;
            default: n->fval2 = v; return;
        }
    }
    n->fval = v; /* any other key (eps, alpha, gamma, cap, ...) sets the scalar */
}

/* "(a, key=value, ...)": positional 0 is the width of FC/Conv, the kernel of
 * the pools, else the scalar; positional 1 is the second scalar. */
static void parse_args(Lex *L, TkmNode *n) {
    lx_ws(L);
    if (*L->p != '(') return;
    L->p++;
    int pos = 0;
    while (*L->p && *L->p != ')') {
        lx_ws(L);
        const char *mark = L->p;
        char key[32];
        lx_ident(L, key, sizeof(key));
        lx_ws(L);
        if (*L->p == '=') {
            L->p++;
            if (!strcmp(key, "prng") || !strcmp(key, "rng")) {
                char name[32];
                lx_ident(L, name, sizeof(name));
                n->rng_type = tkm_parse_rng_name(name);
            } else if (!strcmp(key, "causal") || !strcmp(key, "mask")) {
                char word[32];
                lx_ident(L, word, sizeof(word));
                n->causal = is_true_word(word);
            } else {
                set_keyed_arg(n, key, lx_number(L));
            }
        } else {
            L->p = mark;
            const float v = lx_number(L);
            if (pos == 0) {
                if (n->op == OP_FC || n->op == OP_CONV) n->c_out = (int)v;
                else if (n->op == OP_MIXPOOL || n->op == OP_AVGPOOL) n->k = (int)v;
                else n->fval = v;
            } else if (pos == 1) {
                n->fval2 = v;
            }
            pos++;
        }
        lx_ws(L);
        if (*L->p == ',') L->p++;
        if (L->p == mark) L->p++; /* never stall on an unexpected character */
    }
    if (*L->p == ')') L->p++;
}

static int parse_chain(Lex *L, int in, const char *tag);

/* One step of a chain: an operator, `Identity`, or a `{ branches } -> Merge`. */
static int parse_step(Lex *L, int in, const char *tag) {
    if (L->failed) return in;
    lx_ws(L);
    if (*L->p == '{') {
        L->p++;
        int ends[8], nb = 0;
        for (;;) {
            lx_ws(L);
            if (!*L->p || *L->p == '}') break;
            char btag[32] = "br";
            const char *mark = L->p;
            lx_ident(L, btag, sizeof(btag));
            lx_ws(L);
            if (*L->p == ':') L->p++;
            else L->p = mark;
            const int end = parse_chain(L, in, btag);
            if (L->failed) return in;
            if (nb < 8) ends[nb++] = end;
            lx_ws(L);
            if (*L->p == ',' || *L->p == ';') L->p++;
            if (L->p == mark) L->p++;
        }
        if (*L->p == '}') L->p++;
        lx_arrow(L);
        char merge[32];
        lx_ident(L, merge, sizeof(merge));
        const TkmOpSpec *ms = tkm_find_spec_by_name(merge);
        if (!ms) {
            tkm_graph_error(L->g, "Unknown merge op '%s'", merge);
            L->failed = 1;
            return in;
        }
        const int id = add_node(L, ms, nb > 0 ? ends[0] : -1, nb > 1 ? ends[1] : -1, nb > 2 ? ends[2] : -1, tag);
        if (id >= 0) parse_args(L, &L->g->nodes[id]);
        return id;
    }

    char name[32];
    lx_ident(L, name, sizeof(name));
    if (!name[0] || !strcmp(name, "Identity")) return in;
    const TkmOpSpec *spec = tkm_find_spec_by_name(name);
    if (!spec) {
        tkm_graph_error(L->g, "[TKM Error] Unknown operator '%s' (not in the operator registry)", name);
        L->failed = 1;
        return in;
    }
    const int id = add_node(L, spec, in, -1, -1, tag);
    if (id < 0) return in;
    parse_args(L, &L->g->nodes[id]);
    /* FC and Conv carry their bias as a separate fluid node */
    if (spec->op == OP_CONV || spec->op == OP_FC) return add_node(L, tkm_find_spec_by_op(OP_BIAS), id, -1, -1, tag);
    return id;
}

static int parse_chain(Lex *L, int in, const char *tag) {
    int cur = parse_step(L, in, tag);
    while (!L->failed && lx_arrow(L)) cur = parse_step(L, cur, tag);
    return cur;
}

/* Statements: `input: HxWxC`, `prng: name`, `flow:`, `label: chain` and
 * `label x N: { statements }` (the body is re-parsed N times). */
static int parse_block(Lex *L, int tail, int until_brace) {
    while (!L->failed) {
        lx_ws(L);
        if (!*L->p) break;
        if (until_brace && *L->p == '}') {
            L->p++;
            break;
        }
        if (lx_keyword(L, "input")) {
            lx_skip_char(L, ':');
            int d[3] = {0, 0, 1};
            d[0] = (int)lx_number(L);
            lx_ws(L);
            if (*L->p == 'x' || *L->p == 'X') L->p++;
            d[1] = (int)lx_number(L);
            lx_ws(L);
            if (*L->p == 'x' || *L->p == 'X') {
                L->p++;
                d[2] = (int)lx_number(L);
            }
            tail = add_node(L, NULL, -1, -1, -1, "input");
            if (tail >= 0) {
                L->g->nodes[tail].H = d[0];
                L->g->nodes[tail].W = d[1];
                L->g->nodes[tail].C = d[2];
            }
            continue;
        }
        if (lx_keyword(L, "prng") || lx_keyword(L, "rng")) {
            lx_skip_char(L, ':');
            char name[32];
            lx_ident(L, name, sizeof(name));
            L->g->default_rng = tkm_parse_rng_name(name);
            continue;
        }
        if (lx_keyword(L, "flow")) {
            lx_skip_char(L, ':');
            continue;
        }
        char label[32];
        lx_ident(L, label, sizeof(label));
        if (!label[0]) break;
        lx_ws(L);
        int repeat = 1;
        if (*L->p == 'x' || *L->p == 'X' || *L->p == '*') {
            const char *mark = L->p++;
            lx_ws(L);
            if (isdigit((unsigned char)*L->p)) repeat = (int)lx_number(L);
            else L->p = mark;
        }
        lx_skip_char(L, ':');
        lx_ws(L);
        if (repeat > 1 && *L->p == '{') {
            const char *body = ++L->p;
            for (int r = 0; r < repeat && !L->failed; r++) {
                L->p = body;
                tail = parse_block(L, tail, 1);
            }
        } else {
            tail = parse_chain(L, tail, label);
        }
    }
    return tail;
}

void tkm_parse_dsl(TkmGraph *g, const char *dsl_text, int batch_size) {
    if (!g) return;
    memset(g, 0, sizeof(*g));
    tkm_clear_error();
    g->batch_size = batch_size;
    g->default_rng = RNG_WANG_XORSHIFT32;
    if (!dsl_text) {
        tkm_graph_error(g, "[TKM Error] no DSL text");
        return;
    }
    Lex L = {dsl_text, g, 0};
    parse_block(&L, -1, 0);
    for (int i = 0; i < g->num_nodes; i++)
        if (g->nodes[i].rng_type == RNG_DEFAULT) g->nodes[i].rng_type = g->default_rng;
}

/* ----------------------------------------------------------------- shapes */

static int valid_in(const TkmGraph *g, int id) { return id >= 0 && id < g->num_nodes; }

void tkm_infer_shapes(TkmGraph *g) {
    if (!g) return;
    for (int i = 0; i < g->num_nodes; i++) {
        TkmNode *n = &g->nodes[i];
        if (n->dead || n->op == OP_INPUT) continue;
        if (!valid_in(g, n->in0)) {
            tkm_graph_error(g, "[TKM Shape Error] Node #%d (%s) has no input", i, n->tag);
            return;
        }
        const TkmNode *a = &g->nodes[n->in0];
        n->H = a->H;
        n->W = a->W;
        n->C = a->C;
        switch (n->op) {
            case OP_CONV:
                if (n->s <= 0) {
                    tkm_graph_error(g, "[TKM Shape Error] Conv node #%d (%s) needs a positive stride", i, n->tag);
                    return;
                }
                n->H = (a->H + 2 * n->p - n->k) / n->s + 1;
                n->W = (a->W + 2 * n->p - n->k) / n->s + 1;
                n->C = n->c_out;
                break;
            case OP_MIXPOOL:
            case OP_AVGPOOL:
                if (n->k <= 0) {
                    tkm_graph_error(g, "[TKM Shape Error] pool node #%d (%s) needs a positive kernel", i, n->tag);
                    return;
                }
                n->H = a->H / n->k;
                n->W = a->W / n->k;
                break;
            case OP_FLATTEN:
                n->C = a->H * a->W * a->C;
                n->H = n->W = 1;
                break;
            case OP_FC:
            case OP_FC_TWIN_FUSED:
            case OP_FC_QKV_FUSED:
                n->C = n->c_out;
                break;
            case OP_QKNORM:
            case OP_MUL:
                if (n->c_out > 0) n->C = n->c_out;
                break;
            case OP_GQA_ATTN:
                n->C = n->q_heads * n->head_dim;
                break;
            case OP_ADD: {
                if (!valid_in(g, n->in1)) {
                    tkm_graph_error(g, "[TKM Shape Error] Add node #%d (%s) needs two branches", i, n->tag);
                    return;
                }
                const TkmNode *b = &g->nodes[n->in1];
                if (a->H != b->H || a->W != b->W || a->C != b->C) {
                    tkm_graph_error(g,
                                    "[TKM Shape Error] Node #%d (%s) branch mismatch: [%dx%dx%d] vs [%dx%dx%d]", i,
                                    n->tag, a->H, a->W, a->C, b->H, b->W, b->C);
                    return;
                }
                break;
            }
            default:
                break;
        }
    }
}

/* ------------------------------------------------------- group kernel ABI */

static void sig_arg(TkmKernelSig *s, TkmArgKind kind, int node, int suffix, const char *ctype, const char *name) {
    if (s->num_args >= TKM_MAX_KARGS) return;
    TkmKernelArg *a = &s->args[s->num_args++];
    a->kind = kind;
    a->node_id = node;
    snprintf(a->c_type, sizeof(a->c_type), "%s", ctype);
    if (suffix) snprintf(a->c_name, sizeof(a->c_name), "%s_%d", name, node);
    else snprintf(a->c_name, sizeof(a->c_name), "%s", name);
}

static void bind_fwd(TkmKernelSig *s, const TkmNode *n) {
    const TkmOpSpec *sp = tkm_find_spec_by_node(n);
    if (!sp) return;
    const uint32_t f = sp->res_flags;
    if (f & RES_PARAM_BIAS) sig_arg(s, KARG_BIAS, n->id, 1, "const float2* __restrict__", "b_vec");
    if (f & RES_PARAM_WEIGHT) sig_arg(s, KARG_WEIGHT_VEC, n->id, 1, "const float2* __restrict__", "w_vec");
    if (f & RES_PARAM_BETA) sig_arg(s, KARG_BETA, n->id, 1, "const float2* __restrict__", "beta_vec");
    if (f & RES_SAVE_ISTD) sig_arg(s, KARG_SAVE_ISTD, n->id, 1, "float* __restrict__", "save_istd");
    if (f & RES_SAVE_XHAT) sig_arg(s, KARG_SAVE_XHAT, n->id, 1, "__half2* __restrict__", "save_xhat");
    if (f & RES_SAVE_MASK) sig_arg(s, KARG_SAVE_MASK, n->id, 1, "uint16_t* __restrict__", "save_mask");
    if (f & RES_RNG_SEED) sig_arg(s, KARG_STEP_SEED, n->id, 1, "const uint32_t* __restrict__", "d_seed");
    if (f & RES_BRANCH_IN) sig_arg(s, KARG_BRANCH_IN, n->in1, 1, "const __half2* __restrict__", "branch_in");
}

static void bind_bwd(TkmKernelSig *s, const TkmNode *n) {
    const TkmOpSpec *sp = tkm_find_spec_by_node(n);
    if (!sp) return;
    const uint32_t f = sp->res_flags;
    if (f & RES_BRANCH_IN) sig_arg(s, KARG_DBRANCH_OUT, n->in1, 1, "__half2* __restrict__", "dbranch_out");
    if (f & RES_SAVE_MASK) sig_arg(s, KARG_SAVE_MASK, n->id, 1, "const uint16_t* __restrict__", "save_mask");
    if (f & RES_SAVE_XHAT) sig_arg(s, KARG_SAVE_XHAT, n->id, 1, "const __half2* __restrict__", "save_xhat");
    if (f & RES_SAVE_ISTD) sig_arg(s, KARG_SAVE_ISTD, n->id, 1, "const float* __restrict__", "save_istd");
    if (f & RES_PARAM_WEIGHT) {
        sig_arg(s, KARG_WEIGHT_VEC, n->id, 1, "const float2* __restrict__", "w_vec");
        sig_arg(s, KARG_DWEIGHT_VEC, n->id, 1, "float* __restrict__", "dw_vec");
    }
    if (f & RES_PARAM_BETA) {
        sig_arg(s, KARG_BETA, n->id, 1, "const float2* __restrict__", "beta_vec");
        sig_arg(s, KARG_DBETA, n->id, 1, "float* __restrict__", "dbeta_vec");
    }
    if (f & RES_PARAM_BIAS) {
        sig_arg(s, KARG_BIAS, n->id, 1, "const float2* __restrict__", "b_vec");
        sig_arg(s, KARG_DBIAS, n->id, 1, "float* __restrict__", "db_vec");
    }
}

/* Kernel signature record of a group, as stored in the public PlasmaGroup
 * (reference src/tkm_core.c:333-367).  The launch shape recorded here is the
 * reference's; this build's generated kernels take these arguments in this
 * order followed by private trailing arguments, and are launched with the
 * geometry of tkm_row_geom(). */
static void bind_group(TkmGraph *g, PlasmaGroup *pg) {
    TkmKernelSig *fs = &pg->fwd_sig, *bs = &pg->bwd_sig;
    memset(fs, 0, sizeof(*fs));
    memset(bs, 0, sizeof(*bs));
    snprintf(fs->func_name, sizeof(fs->func_name), "tkm_plasma_fwd_g%d", pg->id);
    snprintf(bs->func_name, sizeof(bs->func_name), "tkm_plasma_bwd_g%d", pg->id);
    if (pg->is_coord_group) {
        fs->grid_x = bs->grid_x = g->batch_size;
        fs->block_x = bs->block_x = 256;
        sig_arg(fs, KARG_IN_MAIN, pg->anchor_id, 0, "const __half* __restrict__", "in_img");
        sig_arg(fs, KARG_OUT_MAIN, pg->out_node_id, 0, "__half* __restrict__", "out_img");
        sig_arg(fs, KARG_STEP_SEED, pg->out_node_id, 0, "const uint32_t* __restrict__", "d_seed");
        sig_arg(bs, KARG_DOUT_MAIN, pg->out_node_id, 0, "const __half* __restrict__", "dout_img");
        sig_arg(bs, KARG_DIN_MAIN, pg->anchor_id, 0, "__half* __restrict__", "din_img");
        return;
    }
    if (pg->C % 2) {
        tkm_graph_error(g,
                        "[TKM Shape Error] PlasmaGroup #%d has odd channel count %d; the plasma kernels work on "
                        "channel pairs and require an even channel count.",
                        pg->id, pg->C);
        return;
    }
    const int rows = g->batch_size * pg->H * pg->W, c2 = pg->C / 2;
    const int small = !pg->is_qkv_prep && c2 > 0 && c2 <= 32 && 256 % c2 == 0;
    const int per_block = small ? 256 / c2 : 16;
    fs->grid_x = bs->grid_x = (rows + per_block - 1) / per_block;
    if (small && bs->grid_x > 256) bs->grid_x = 256;
    fs->block_x = bs->block_x = 256;

    sig_arg(fs, KARG_IN_MAIN, pg->anchor_id, 0, "const __half2* __restrict__", "in_0");
    sig_arg(fs, KARG_OUT_MAIN, pg->out_node_id, 0, "__half2* __restrict__", "out_0");
    sig_arg(bs, KARG_DOUT_MAIN, pg->out_node_id, 0, "const __half2* __restrict__", "dout_0");
    sig_arg(bs, KARG_IN_MAIN, pg->anchor_id, 0, "const __half2* __restrict__", "replay_in_0");
    sig_arg(bs, KARG_DIN_MAIN, pg->anchor_id, 0, "__half2* __restrict__", "din_0");
    if (pg->is_twin_epilogue) {
        const TkmNode *m = &g->nodes[pg->node_ids[0]];
        for (int i = 0; i < m->left_len; i++) bind_fwd(fs, &g->nodes[m->left_nodes[i]]);
        for (int i = 0; i < m->right_len; i++) bind_fwd(fs, &g->nodes[m->right_nodes[i]]);
        for (int i = 0; i < m->left_len; i++) bind_bwd(bs, &g->nodes[m->left_nodes[i]]);
        for (int i = 0; i < m->right_len; i++) bind_bwd(bs, &g->nodes[m->right_nodes[i]]);
    }
    for (int i = 0; i < pg->count; i++) bind_fwd(fs, &g->nodes[pg->node_ids[i]]);
    for (int i = pg->count - 1; i >= 0; i--) bind_bwd(bs, &g->nodes[pg->node_ids[i]]);
}

/* ------------------------------------------------------ optimize and bind */

static int check_node(TkmGraph *g, int i) {
    const TkmNode *n = &g->nodes[i];
    if (n->dead) return 1;
    if (n->op == OP_GQA_ATTN) {
        const int ok = (n->head_dim == 64 || n->head_dim == 128) && n->q_heads > 0 && n->kv_heads > 0 &&
                       n->q_heads % n->kv_heads == 0 && valid_in(g, n->in0) && valid_in(g, n->in1) &&
                       valid_in(g, n->in2) && n->q_heads * n->head_dim == g->nodes[n->in0].C &&
                       n->kv_heads * n->head_dim == g->nodes[n->in1].C &&
                       n->kv_heads * n->head_dim == g->nodes[n->in2].C;
        if (!ok) {
            tkm_graph_error(g,
                            "[TKM Shape Error] GQA node #%d (%s) requires head_dim 64 or 128, divisible query/KV "
                            "heads, and Q/K/V widths matching the configured heads.",
                            i, n->tag);
            return 0;
        }
    }
    if (n->op == OP_ROPE &&
        (!(n->rope_theta > 0.0f) || !(n->rope_scale >= 1.0f) || !(n->rope_low_freq_factor > 0.0f) ||
         !(n->rope_high_freq_factor > n->rope_low_freq_factor) || !(n->rope_original_context_length > 0.0f))) {
        tkm_graph_error(g,
                        "[TKM Shape Error] RoPE node #%d (%s) requires theta>0, scale>=1, "
                        "0<low_freq_factor<high_freq_factor, and original_context_length>0.",
                        i, n->tag);
        return 0;
    }
    if ((n->op == OP_MIXPOOL || n->op == OP_AVGPOOL) && n->C % 2) {
        tkm_graph_error(g, "[TKM Shape Error] %s node #%d (%s) has odd channel count %d.",
                        n->op == OP_MIXPOOL ? "MixPool" : "AvgPool", i, n->tag, n->C);
        return 0;
    }
    const TkmOpSpec *sp = tkm_find_spec_by_node(n);
    if (sp && (sp->res_flags & RES_AUG_COLOR) && n->C != 3) {
        tkm_graph_error(g, "[TKM Shape Error] Color augmentation node #%d (%s) requires exactly 3 channels, got %d.",
                        i, n->tag, n->C);
        return 0;
    }
    return 1;
}

/* first live node after `cur` whose main input is `cur` */
static int next_consumer(const TkmGraph *g, int cur) {
    for (int k = cur + 1; k < g->num_nodes; k++)
        if (!g->nodes[k].dead && g->nodes[k].in0 == cur) return k;
    return -1;
}

static PlasmaGroup *new_group(TkmGraph *g, const TkmNode *n) {
    if (g->num_groups >= TKM_MAX_GROUPS) {
        tkm_graph_error(g, "[TKM Error] graph exceeds %d plasma groups", TKM_MAX_GROUPS);
        return NULL;
    }
    PlasmaGroup *pg = &g->groups[g->num_groups];
    memset(pg, 0, sizeof(*pg));
    pg->id = g->num_groups++;
    pg->anchor_id = n->in0;
    pg->H = n->H;
    pg->W = n->W;
    pg->C = n->C;
    return pg;
}

static void join_group(PlasmaGroup *pg, TkmNode *cn) {
    if (pg->count < 16) pg->node_ids[pg->count++] = cn->id;
    pg->out_node_id = cn->id;
    cn->plasma_grp = pg->id;
}

void tkm_optimize_and_bind(TkmGraph *g) {
    if (!g || g->num_nodes <= 0) return;
    int nrules = 0;
    const TkmFusionRule *rules = tkm_get_fusion_rules(&nrules);

    tkm_infer_shapes(g);
    for (int i = 0; i < g->num_nodes; i++)
        if (!check_node(g, i)) return;

    for (int i = 0; i < g->num_nodes; i++) {
        if (g->nodes[i].dead) continue;
        for (int r = 0; r < nrules; r++)
            if (rules[r].match(g, i)) {
                rules[r].apply(g, i);
                break;
            }
    }
    if (g->num_nodes <= 0) return;
    tkm_infer_shapes(g);
    if (g->num_nodes <= 0) return;

    for (int i = 0; i < g->num_nodes; i++) g->nodes[i].users = 0;
    for (int i = 0; i < g->num_nodes; i++) {
        const TkmNode *n = &g->nodes[i];
        if (n->dead) continue;
        if (n->in0 >= 0) g->nodes[n->in0].users++;
        if (n->in1 >= 0) g->nodes[n->in1].users++;
        if (n->in2 >= 0) g->nodes[n->in2].users++;
    }

    g->num_groups = 0;
    for (int i = 0; i < g->num_nodes; i++) {
        TkmNode *n = &g->nodes[i];
        if (n->dead || n->plasma_grp >= 0) continue;
        PlasmaGroup *pg = NULL;
        if (n->cat == CAT_COORD) {
            /* coordinate bricks, then pixel/colour bricks, until a fan-out */
            if (!(pg = new_group(g, n))) return;
            pg->is_coord_group = 1;
            int seen_pixel = 0;
            for (int cur = i; cur >= 0;) {
                TkmNode *cn = &g->nodes[cur];
                if (cn->dead || cn->plasma_grp >= 0 || cn->cat != CAT_COORD) break;
                const TkmOpSpec *sp = tkm_find_spec_by_node(cn);
                const int pixel = sp && (sp->res_flags & (RES_AUG_PIXEL | RES_AUG_COLOR));
                if (seen_pixel && !pixel) break;
                seen_pixel |= pixel;
                if (cn->op == OP_BORDER_REFLECT) pg->use_reflect_border = 1;
                join_group(pg, cn);
                if (cn->users > 1) break;
                cur = next_consumer(g, cur);
            }
        } else if (n->op == OP_QKNORM && n->q_c > 0) {
            if (!(pg = new_group(g, n))) return;
            pg->is_qkv_prep = 1;
            join_group(pg, n);
        } else if (n->cat == CAT_NORM || n->cat == CAT_FLUID) {
            /* a chain of fluid operators with at most one normalisation */
            if (!(pg = new_group(g, n))) return;
            if (n->op == OP_MUL && n->left_len > 0) pg->is_twin_epilogue = 1;
            for (int cur = i; cur >= 0;) {
                TkmNode *cn = &g->nodes[cur];
                if (cn->dead || cn->plasma_grp >= 0) break;
                if (cn->cat != CAT_NORM && cn->cat != CAT_FLUID) break;
                if (cn->cat == CAT_NORM && pg->has_norm) break;
                join_group(pg, cn);
                if (cn->cat == CAT_NORM) pg->has_norm = 1;
                if (cn->users > 1) break;
                cur = next_consumer(g, cur);
            }
        }
        if (pg) {
            bind_group(g, pg);
            if (g->num_nodes <= 0) return;
        }
    }
}

/* ------------------------------------------------------------------ arena */

void tkm_plan_memory(TkmGraph *g) {
    if (!g) return;
    size_t off = 0, naive = 0;
    int slot = 0;
    for (int i = 0; i < g->num_nodes; i++) {
        TkmNode *n = &g->nodes[i];
        if (n->dead) continue;
        const size_t bytes = (((size_t)g->batch_size * n->H * n->W * n->C * 2) + 255) & ~(size_t)255;
        naive += bytes;
        if (n->plasma_grp >= 0 && g->groups[n->plasma_grp].out_node_id != i) {
            n->out_buf_id = -1; /* lives in registers inside its group */
            n->out_bytes = 0;
            continue;
        }
        n->out_bytes = bytes;
        n->out_buf_id = slot++;
        n->out_offset = off;
        off += bytes;
    }
    g->total_arena_bytes = off;
    g->naive_arena_bytes = naive;
}

/* ---------------------------------------------------------------- summary */

void tkm_dump_summary(const TkmGraph *g, FILE *out) {
    if (!g || !out) return;
    const double naive = g->naive_arena_bytes / 1048576.0, fused = g->total_arena_bytes / 1048576.0;
    fprintf(out, "  default PRNG  : %s\n", tkm_rng_name(g->default_rng));
    fprintf(out, "  arena (16-bit): unfused %.2f MB -> fused %.2f MB (%.1f%% saved)\n\n", naive, fused,
            naive > 0 ? 100.0 * (1.0 - fused / naive) : 0.0);
    fprintf(out, " %-4s %-20s %-14s %-10s %-16s %s\n", "id", "tag", "op", "inputs", "shape HxWxC", "storage");
    for (int i = 0; i < g->num_nodes; i++) {
        const TkmNode *n = &g->nodes[i];
        if (n->dead) continue;
        const TkmOpSpec *sp = tkm_find_spec_by_node(n);
        char shape[48], where[96], ins[24];
        snprintf(shape, sizeof(shape), "%dx%dx%d", n->H, n->W, n->C);
        snprintf(ins, sizeof(ins), "%d,%d", n->in0, n->in1);
        if (n->out_buf_id < 0)
            snprintf(where, sizeof(where), "registers (plasma group %d)", n->plasma_grp);
        else if (n->plasma_grp >= 0)
            snprintf(where, sizeof(where), "slot %d @%zu KB (plasma group %d output)", n->out_buf_id,
                     n->out_offset / 1024, n->plasma_grp);
        else
            snprintf(where, sizeof(where), "slot %d @%zu KB (anchor output)", n->out_buf_id, n->out_offset / 1024);
        fprintf(out, " #%-3d %-20s %-14s %-10s %-16s %s\n", n->id, n->tag, sp ? sp->dsl_name : "Input", ins, shape,
                where);
    }
    fprintf(out, "\n");
}

/* --------------------------------------------------------------- registry */

int tkm_verify_registry(void) {
    int errors = 0;
    for (int op = 0; op < OP_COUNT; op++) {
        if (op == OP_USER_FLUID) continue;
        if (!tkm_find_spec_by_op((TkmOpType)op)) {
            fprintf(stderr, "[Registry Error] operator enum %d has no registry entry\n", op);
            errors++;
        }
    }
    for (int i = 0; i < tkm_get_spec_count(); i++) {
        const TkmOpSpec *s = tkm_find_spec_by_index(i);
        const int has_fwd = s->fwd_cuda || s->fwd_expr, has_bwd = s->bwd_cuda || s->bwd_expr;
        if (s->cat == CAT_NORM && !(s->res_flags & RES_SAVE_XHAT)) {
            fprintf(stderr, "[Registry Error] normalisation '%s' must declare RES_SAVE_XHAT\n", s->dsl_name);
            errors++;
        }
        if (s->cat == CAT_FLUID && has_fwd != has_bwd) {
            fprintf(stderr, "[Registry Error] '%s' needs both a forward and a backward definition\n", s->dsl_name);
            errors++;
        }
        if ((s->fwd_cuda && s->fwd_expr) || (s->bwd_cuda && s->bwd_expr)) {
            fprintf(stderr, "[Registry Error] '%s' mixes a CUDA body and a formula in one direction\n", s->dsl_name);
            errors++;
        }
        if (s->fwd_expr || s->bwd_expr) {
            const float probes[3] = {-1.0f, 0.25f, 1.5f};
            for (int p = 0; p < 3; p++) {
                float v;
                if ((s->fwd_expr && !tkm_eval_math_expr(s->fwd_expr, probes[p], s->default_fval, &v)) ||
                    (s->bwd_expr && !tkm_eval_math_expr(s->bwd_expr, probes[p], s->default_fval, &v))) {
                    fprintf(stderr, "[Registry Error] '%s' has an invalid formula\n", s->dsl_name);
                    errors++;
                    break;
                }
            }
        }
    }
    return errors;
}
