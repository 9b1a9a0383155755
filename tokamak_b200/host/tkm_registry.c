/*
 * tkm_registry.c -- operator registry, scalar formula evaluator, PRNG names and
 * the four peephole fusion rules of the Tokamak engine.
 *
 * The table keeps the reference's contract (src/tkm_registry.c:43-466): the
 * same entries in the same order (spec indexes are stored in TkmNode.spec_id),
 * the same DSL names, categories, resource flags and default scalars, so a
 * .tkm file parses to the same node table.  The per-pair CUDA bodies are this
 * build's own; they run inside the snippet environment documented in
 * docs/CONTRIBUTING_OP.md of the reference (float2 v / dy / pre, fval, tid,
 * row, idx2, w_vec / b_vec / beta_vec, acc_dw / acc_db / acc_dbeta, save_mask,
 * rng) that tkm_codegen.c provides.
 *
 * Entries whose bodies are NULL are emitted natively by the code generator:
 * normalisations (a row reduction spans many pairs per thread there), the
 * residual Add (vector load of the branch), the fused QKV prep (QKNorm + RoPE)
 * and the twin-branch Mul.  Image augmentations (CAT_COORD) carry no bodies:
 * coordinate groups are outside this build's scope and are rejected at ignite.
 */
#include <ctype.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "tkm_internal.h"

/* ------------------------------------------------------------------ PRNGs */

const char *tkm_rng_name(TkmRngType r) {
    static const char *names[] = {"wang_xorshift32", "xorshift32", "wang_xorshift32", "pcg32", "philox"};
    return (r >= RNG_DEFAULT && r <= RNG_PHILOX) ? names[r] : names[0];
}

const char *tkm_rng_struct_name(TkmRngType r) {
    static const char *names[] = {"RngWangXorshift32", "RngXorshift32", "RngWangXorshift32", "RngPcg32",
                                  "RngPhilox"};
    return (r >= RNG_DEFAULT && r <= RNG_PHILOX) ? names[r] : names[0];
}

TkmRngType tkm_parse_rng_name(const char *s) {
    static const struct { const char *name; TkmRngType type; } aliases[] = {
        {"xorshift32", RNG_XORSHIFT32}, {"xorshift", RNG_XORSHIFT32},
        {"wang_xorshift32", RNG_WANG_XORSHIFT32}, {"wang", RNG_WANG_XORSHIFT32},
        {"pcg32", RNG_PCG32}, {"pcg", RNG_PCG32},
        {"philox", RNG_PHILOX}, {"philox4x32", RNG_PHILOX},
    };
    for (size_t i = 0; s && i < sizeof(aliases) / sizeof(aliases[0]); i++)
        if (!strcmp(s, aliases[i].name)) return aliases[i].type;
    return RNG_WANG_XORSHIFT32;
}

/* --------------------------------------------------------------- registry */

#define NOBODY NULL, NULL
#define AUG(op, name, flags, f) {op, name, CAT_COORD, flags, f, NOBODY, NULL, NULL}

static const TkmOpSpec REGISTRY[] = {
    {OP_NONE, "None", CAT_META, RES_NONE, 0.0f, NOBODY, NULL, NULL},
    {OP_INPUT, "Input", CAT_META, RES_NONE, 0.0f, NOBODY, NULL, NULL},

    {OP_CONV, "Conv", CAT_ANCHOR, RES_NONE, 0.0f, NOBODY, NULL, NULL},
    {OP_FC, "FC", CAT_ANCHOR, RES_NONE, 0.0f, NOBODY, NULL, NULL},
    {OP_FC_TWIN_FUSED, "FC_Twin2x", CAT_ANCHOR, RES_NONE, 0.0f, NOBODY, NULL, NULL},
    {OP_FC_QKV_FUSED, "FC_QKV3x", CAT_ANCHOR, RES_NONE, 0.0f, NOBODY, NULL, NULL},
    {OP_GQA_ATTN, "GQA", CAT_ANCHOR, RES_NONE, 0.0f, NOBODY, NULL, NULL},
    {OP_MIXPOOL, "MixPool", CAT_SPATIAL, RES_NONE, 0.85f, NOBODY, NULL, NULL},
    {OP_AVGPOOL, "AvgPool", CAT_SPATIAL, RES_NONE, 0.0f, NOBODY, NULL, NULL},
    {OP_FLATTEN, "Flatten", CAT_SPATIAL, RES_NONE, 0.0f, NOBODY, NULL, NULL},

    AUG(OP_BORDER_REFLECT, "BorderReflect", RES_NONE, 0.0f),
    AUG(OP_RAND_SHIFT, "RandShift", RES_RNG_SEED, 2.0f),
    AUG(OP_RAND_ROTATE, "RandRotate", RES_RNG_SEED, 10.0f),
    AUG(OP_RAND_SCALE, "RandScale", RES_RNG_SEED, 0.10f),
    AUG(OP_RAND_FLIPX, "RandFlipX", RES_RNG_SEED, 0.5f),
    AUG(OP_RAND_FLIPY, "RandFlipY", RES_RNG_SEED, 0.5f),
    AUG(OP_RAND_ELASTIC, "RandElastic", RES_RNG_SEED, 1.6f),
    AUG(OP_RAND_NOISE, "RandNoise", RES_RNG_SEED | RES_AUG_PIXEL, 0.03f),
    AUG(OP_RAND_CUTOUT, "RandCutout", RES_RNG_SEED | RES_AUG_PIXEL, 4.0f),
    AUG(OP_RAND_BRIGHTNESS, "RandBrightness", RES_RNG_SEED | RES_AUG_PIXEL, 0.15f),
    AUG(OP_RAND_CONTRAST, "RandContrast", RES_RNG_SEED | RES_AUG_PIXEL, 0.20f),
    AUG(OP_RAND_SATURATION, "RandSaturation", RES_RNG_SEED | RES_AUG_COLOR, 0.30f),
    AUG(OP_RAND_HUE, "RandHue", RES_RNG_SEED | RES_AUG_COLOR, 0.08f),
    AUG(OP_RAND_GRAYSCALE, "RandGrayscale", RES_RNG_SEED | RES_AUG_COLOR, 0.10f),
    AUG(OP_RAND_CHANNEL_SCALE, "RandChannelScale", RES_RNG_SEED | RES_AUG_COLOR, 0.15f),
    AUG(OP_RAND_SOLARIZE, "RandSolarize", RES_RNG_SEED | RES_AUG_PIXEL, 0.50f),
    AUG(OP_RAND_ERASING, "RandErasing", RES_RNG_SEED | RES_AUG_PIXEL, 8.0f),

    /* normalisations: emitted natively (row statistics over all pairs) */
    {OP_BN, "BN", CAT_NORM, RES_PARAM_WEIGHT | RES_PARAM_BETA | RES_SAVE_ISTD | RES_SAVE_XHAT, 1e-2f, NOBODY, NULL, NULL},
    {OP_LN, "LN", CAT_NORM, RES_PARAM_WEIGHT | RES_PARAM_BETA | RES_SAVE_ISTD | RES_SAVE_XHAT, 1e-5f, NOBODY, NULL, NULL},
    {OP_RMSNORM, "RMSNorm", CAT_NORM, RES_PARAM_WEIGHT | RES_SAVE_ISTD | RES_SAVE_XHAT, 1e-5f, NOBODY, NULL, NULL},
    {OP_L2NORM, "L2Norm", CAT_NORM, RES_SAVE_ISTD | RES_SAVE_XHAT, 1e-5f, NOBODY, NULL, NULL},
    {OP_QKNORM, "QKNorm", CAT_FLUID, RES_PARAM_BIAS | RES_PARAM_WEIGHT | RES_SAVE_ISTD | RES_SAVE_XHAT, 1e-5f,
     NOBODY, NULL, NULL},

    /* pointwise fluid operators: per channel pair */
    {OP_BIAS, "Bias", CAT_FLUID, RES_PARAM_BIAS, 0.0f,
     "const float2 bb = b_vec[tid]; v = make_float2(v.x + bb.x, v.y + bb.y);",
     "acc_db = make_float2(acc_db.x + dy.x, acc_db.y + dy.y);", NULL, NULL},
    {OP_SILU, "SiLU", CAT_FLUID, RES_NONE, 0.0f,
     "v = make_float2(v.x * tkm_sigmoid(v.x), v.y * tkm_sigmoid(v.y));",
     "const float s0 = tkm_sigmoid(pre.x), s1 = tkm_sigmoid(pre.y);\n"
     "dy.x *= s0 + pre.x * s0 * (1.0f - s0);\n"
     "dy.y *= s1 + pre.y * s1 * (1.0f - s1);", NULL, NULL},
    {OP_RELU, "ReLU", CAT_FLUID, RES_NONE, 0.0f,
     "v = make_float2(fmaxf(v.x, 0.0f), fmaxf(v.y, 0.0f));",
     "if (!(pre.x > 0.0f)) dy.x = 0.0f;\nif (!(pre.y > 0.0f)) dy.y = 0.0f;", NULL, NULL},
    {OP_RELU2, "ReLU2", CAT_FLUID, RES_NONE, 0.0f,
     "const float r0 = fmaxf(v.x, 0.0f), r1 = fmaxf(v.y, 0.0f); v = make_float2(r0 * r0, r1 * r1);",
     "dy.x *= pre.x > 0.0f ? pre.x + pre.x : 0.0f;\ndy.y *= pre.y > 0.0f ? pre.y + pre.y : 0.0f;", NULL, NULL},
    {OP_LEAKY_RELU, "LeakyReLU", CAT_FLUID, RES_NONE, 0.01f,
     "if (!(v.x > 0.0f)) v.x *= fval;\nif (!(v.y > 0.0f)) v.y *= fval;",
     "if (!(pre.x > 0.0f)) dy.x *= fval;\nif (!(pre.y > 0.0f)) dy.y *= fval;", NULL, NULL},
    {OP_ELU, "ELU", CAT_FLUID, RES_NONE, 1.0f,
     "if (!(v.x > 0.0f)) v.x = fval * expm1f(v.x);\nif (!(v.y > 0.0f)) v.y = fval * expm1f(v.y);",
     "if (!(pre.x > 0.0f)) dy.x *= fval * expf(pre.x);\nif (!(pre.y > 0.0f)) dy.y *= fval * expf(pre.y);", NULL,
     NULL},
    {OP_GELU, "GELU", CAT_FLUID, RES_NONE, 0.0f,
     "v = make_float2(tkm_gelu_tanh(v.x), tkm_gelu_tanh(v.y));",
     "dy = make_float2(dy.x * tkm_gelu_tanh_grad(pre.x), dy.y * tkm_gelu_tanh_grad(pre.y));", NULL, NULL},
    {OP_MISH, "Mish", CAT_FLUID, RES_NONE, 0.0f,
     "v = make_float2(v.x * tanhf(tkm_softplus20(v.x)), v.y * tanhf(tkm_softplus20(v.y)));",
     "const float t0 = tanhf(tkm_softplus20(pre.x)), t1 = tanhf(tkm_softplus20(pre.y));\n"
     "dy.x *= t0 + pre.x * (1.0f - t0 * t0) * tkm_sigmoid(pre.x);\n"
     "dy.y *= t1 + pre.y * (1.0f - t1 * t1) * tkm_sigmoid(pre.y);", NULL, NULL},
    {OP_HARDSWISH, "HardSwish", CAT_FLUID, RES_NONE, 0.0f,
     "v.x *= fminf(fmaxf(v.x + 3.0f, 0.0f), 6.0f) * (1.0f / 6.0f);\n"
     "v.y *= fminf(fmaxf(v.y + 3.0f, 0.0f), 6.0f) * (1.0f / 6.0f);",
     "dy.x *= pre.x <= -3.0f ? 0.0f : (pre.x >= 3.0f ? 1.0f : (2.0f * pre.x + 3.0f) * (1.0f / 6.0f));\n"
     "dy.y *= pre.y <= -3.0f ? 0.0f : (pre.y >= 3.0f ? 1.0f : (2.0f * pre.y + 3.0f) * (1.0f / 6.0f));", NULL, NULL},
    {OP_HARDSIGMOID, "HardSigmoid", CAT_FLUID, RES_NONE, 0.0f,
     "v.x = fminf(fmaxf((v.x + 3.0f) * (1.0f / 6.0f), 0.0f), 1.0f);\n"
     "v.y = fminf(fmaxf((v.y + 3.0f) * (1.0f / 6.0f), 0.0f), 1.0f);",
     "dy.x *= (pre.x > -3.0f && pre.x < 3.0f) ? (1.0f / 6.0f) : 0.0f;\n"
     "dy.y *= (pre.y > -3.0f && pre.y < 3.0f) ? (1.0f / 6.0f) : 0.0f;", NULL, NULL},
    {OP_TANH, "Tanh", CAT_FLUID, RES_NONE, 0.0f,
     "v = make_float2(tanhf(v.x), tanhf(v.y));",
     "const float t0 = tanhf(pre.x), t1 = tanhf(pre.y);\ndy.x *= 1.0f - t0 * t0;\ndy.y *= 1.0f - t1 * t1;", NULL, NULL},
    {OP_SIGMOID, "Sigmoid", CAT_FLUID, RES_NONE, 0.0f,
     "v = make_float2(tkm_sigmoid(v.x), tkm_sigmoid(v.y));",
     "const float s0 = tkm_sigmoid(pre.x), s1 = tkm_sigmoid(pre.y);\ndy.x *= s0 * (1.0f - s0);\n"
     "dy.y *= s1 * (1.0f - s1);", NULL, NULL},
    {OP_SWISH_BETA, "SwishBeta", CAT_FLUID, RES_NONE, 1.5f,
     "v = make_float2(v.x * tkm_sigmoid(fval * v.x), v.y * tkm_sigmoid(fval * v.y));",
     "const float s0 = tkm_sigmoid(fval * pre.x), s1 = tkm_sigmoid(fval * pre.y);\n"
     "dy.x *= s0 * (1.0f + fval * pre.x * (1.0f - s0));\n"
     "dy.y *= s1 * (1.0f + fval * pre.y * (1.0f - s1));", NULL, NULL},
    {OP_SIN, "Sin", CAT_FLUID, RES_NONE, 1.0f,
     "v = make_float2(sinf(fval * v.x), sinf(fval * v.y));",
     "dy.x *= fval * cosf(fval * pre.x);\ndy.y *= fval * cosf(fval * pre.y);", NULL, NULL},
    {OP_COSGATE, "CosGate", CAT_FLUID, RES_NONE, 0.0f,
     "v = make_float2(v.x * cosf(v.x), v.y * cosf(v.y));",
     "dy.x *= cosf(pre.x) - pre.x * sinf(pre.x);\ndy.y *= cosf(pre.y) - pre.y * sinf(pre.y);", NULL, NULL},
    {OP_SOFTCAP, "SoftCap", CAT_FLUID, RES_NONE, 30.0f,
     "v = make_float2(fval * tanhf(v.x / fval), fval * tanhf(v.y / fval));",
     "const float t0 = tanhf(pre.x / fval), t1 = tanhf(pre.y / fval);\ndy.x *= 1.0f - t0 * t0;\n"
     "dy.y *= 1.0f - t1 * t1;", NULL, NULL},
    {OP_CLAMP, "Clamp", CAT_FLUID, RES_NONE, 6.0f,
     "v = make_float2(fminf(fmaxf(v.x, -fval), fval), fminf(fmaxf(v.y, -fval), fval));",
     "if (!(pre.x > -fval && pre.x < fval)) dy.x = 0.0f;\nif (!(pre.y > -fval && pre.y < fval)) dy.y = 0.0f;",
     NULL, NULL},
    {OP_SCALE, "Scale", CAT_FLUID, RES_NONE, 1.0f,
     "v = make_float2(v.x * fval, v.y * fval);",
     "dy = make_float2(dy.x * fval, dy.y * fval);", NULL, NULL},
    {OP_LAYERSCALE, "LayerScale", CAT_FLUID, RES_PARAM_WEIGHT, 1e-4f,
     "const float2 ww = w_vec[tid]; v = make_float2(v.x * ww.x, v.y * ww.y);",
     "const float2 ww = w_vec[tid];\n"
     "acc_dw = make_float2(acc_dw.x + dy.x * pre.x, acc_dw.y + dy.y * pre.y);\n"
     "dy = make_float2(dy.x * ww.x, dy.y * ww.y);", NULL, NULL},
    {OP_DYT, "DyT", CAT_FLUID, RES_PARAM_WEIGHT, 0.5f,
     "const float2 ww = w_vec[tid]; v = make_float2(tanhf(fval * v.x) * ww.x, tanhf(fval * v.y) * ww.y);",
     "const float2 ww = w_vec[tid];\n"
     "const float t0 = tanhf(fval * pre.x), t1 = tanhf(fval * pre.y);\n"
     "acc_dw = make_float2(acc_dw.x + dy.x * t0, acc_dw.y + dy.y * t1);\n"
     "dy.x *= ww.x * fval * (1.0f - t0 * t0);\n"
     "dy.y *= ww.y * fval * (1.0f - t1 * t1);", NULL, NULL},
    {OP_PRELU, "PReLU", CAT_FLUID, RES_PARAM_WEIGHT, 0.25f,
     "const float2 ww = w_vec[tid];\n"
     "if (!(v.x > 0.0f)) v.x *= ww.x * fval;\n"
     "if (!(v.y > 0.0f)) v.y *= ww.y * fval;",
     "const float2 ww = w_vec[tid];\n"
     "if (!(pre.x > 0.0f)) { acc_dw.x += dy.x * pre.x * fval; dy.x *= ww.x * fval; }\n"
     "if (!(pre.y > 0.0f)) { acc_dw.y += dy.y * pre.y * fval; dy.y *= ww.y * fval; }", NULL, NULL},
    {OP_XATLU, "xATLU", CAT_FLUID, RES_PARAM_WEIGHT, 0.5f,
     "const float2 ww = w_vec[tid];\n"
     "v.x *= ww.x * tkm_sigmoid(v.x) + (1.0f - ww.x);\n"
     "v.y *= ww.y * tkm_sigmoid(v.y) + (1.0f - ww.y);",
     "const float2 ww = w_vec[tid];\n"
     "const float s0 = tkm_sigmoid(pre.x), s1 = tkm_sigmoid(pre.y);\n"
     "acc_dw = make_float2(acc_dw.x + dy.x * pre.x * (s0 - 1.0f), acc_dw.y + dy.y * pre.y * (s1 - 1.0f));\n"
     "dy.x *= (1.0f - ww.x) + ww.x * s0 * (1.0f + pre.x * (1.0f - s0));\n"
     "dy.y *= (1.0f - ww.y) + ww.y * s1 * (1.0f + pre.y * (1.0f - s1));", NULL, NULL},
    {OP_ROPE, "RoPE", CAT_FLUID, RES_NONE, 0.0f, NOBODY, NULL, NULL},
    {OP_DROP, "Drop", CAT_FLUID, RES_SAVE_MASK | RES_RNG_SEED, 0.1f,
     "const float keep = 1.0f - fval;\n"
     "const unsigned k0 = rng_uniform(&rng) < keep, k1 = rng_uniform(&rng) < keep;\n"
     "save_mask[idx2] = (uint16_t)(k0 | (k1 << 8));\n"
     "v = make_float2(k0 ? v.x / keep : 0.0f, k1 ? v.y / keep : 0.0f);",
     "const uint16_t mk = save_mask[idx2]; const float keep = 1.0f - fval;\n"
     "dy = make_float2((mk & 0xFFu) ? dy.x / keep : 0.0f, (mk >> 8) ? dy.y / keep : 0.0f);", NULL, NULL},
    {OP_ADD, "Add", CAT_FLUID, RES_BRANCH_IN, 0.0f, NOBODY, NULL, NULL},
    {OP_MUL, "Mul", CAT_FLUID, RES_NONE, 0.0f, NOBODY, NULL, NULL},
    {OP_SOFTMAX, "Softmax", CAT_ANCHOR, RES_NONE, 0.0f, NOBODY, NULL, NULL},
    {OP_SOFTMAX_CE, "SoftmaxCE", CAT_ANCHOR, RES_NONE, 0.0f, NOBODY, NULL, NULL},
    {OP_SOFTMAX_FOCAL, "SoftmaxFocal", CAT_ANCHOR, RES_NONE, 2.0f, NOBODY, NULL, NULL},
    {OP_SOFTMAX_MSE, "SoftmaxMSE", CAT_ANCHOR, RES_NONE, 0.0f, NOBODY, NULL, NULL},
    /* formula-only operators: scalar forward and derivative in x and fval */
    {OP_USER_FLUID, "Softplus", CAT_FLUID, RES_NONE, 0.0f, NOBODY, "log(1 + exp(x))", "1 / (1 + exp(-x))"},
    /* Snake (Lee et al., BigVGAN, ICLR 2023, arXiv:2206.04658): x + sin^2(a x)/a */
    {OP_USER_FLUID, "Snake", CAT_FLUID, RES_NONE, 1.0f, NOBODY, "x + sin(fval * x) * sin(fval * x) / fval",
     "1 + sin(2 * fval * x)"},
};

#define N_SPECS ((int)(sizeof(REGISTRY) / sizeof(REGISTRY[0])))

int tkm_get_spec_count(void) { return N_SPECS; }

const TkmOpSpec *tkm_find_spec_by_index(int index) {
    return (index >= 0 && index < N_SPECS) ? &REGISTRY[index] : NULL;
}

const TkmOpSpec *tkm_find_spec_by_op(TkmOpType op) {
    for (int i = 0; i < N_SPECS; i++)
        if (REGISTRY[i].op == op) return &REGISTRY[i];
    return NULL;
}

const TkmOpSpec *tkm_find_spec_by_name(const char *dsl_name) {
    if (!dsl_name) return NULL;
    for (int i = 0; i < N_SPECS; i++)
        if (!strcmp(REGISTRY[i].dsl_name, dsl_name)) return &REGISTRY[i];
    return NULL;
}

const TkmOpSpec *tkm_find_spec_by_node(const TkmNode *node) {
    if (!node) return NULL;
    /* formula operators share OP_USER_FLUID; their spec index disambiguates */
    return node->op == OP_USER_FLUID ? tkm_find_spec_by_index(node->spec_id) : tkm_find_spec_by_op(node->op);
}

int tkm_get_spec_index(const TkmOpSpec *spec) {
    if (!spec || spec < REGISTRY || spec >= REGISTRY + N_SPECS) return -1;
    return (int)(spec - REGISTRY);
}

/* ---------------------------------------------------- formula evaluator
 * Grammar (reference src/tkm_registry.c:490-616, same operator set):
 *   sum     := product (('+'|'-') product)*
 *   product := unary (('*'|'/') unary)*
 *   unary   := ('+'|'-') unary | primary
 *   primary := number | 'x' | 'fval' | 'pi' | '(' sum ')' | name '(' sum [',' sum] ')'
 * Evaluation is in single precision with libm's float functions. */

typedef struct {
    const char *s;
    float x, fval;
    int bad;
} Expr;

static void ex_ws(Expr *e) {
    while (isspace((unsigned char)*e->s)) e->s++;
}

static float ex_sum(Expr *e);

static float ex_call(Expr *e, const char *name, float a, float b, int nargs) {
    static const struct { const char *name; int nargs; int id; } fns[] = {
        {"exp", 1, 0}, {"log", 1, 1}, {"ln", 1, 1}, {"sqrt", 1, 2}, {"sin", 1, 3}, {"cos", 1, 4},
        {"tanh", 1, 5}, {"abs", 1, 6}, {"max", 2, 7}, {"min", 2, 8}, {"pow", 2, 9},
    };
    for (size_t i = 0; i < sizeof(fns) / sizeof(fns[0]); i++) {
        if (strcmp(name, fns[i].name) || nargs != fns[i].nargs) continue;
        switch (fns[i].id) {
            case 0: return expf(a);
            case 1: return logf(a);
            case 2: return sqrtf(a);
            case 3: return sinf(a);
            case 4: return cosf(a);
            case 5: return tanhf(a);
            case 6: return fabsf(a);
            case 7: return fmaxf(a, b);
            case 8: return fminf(a, b);
            default: return powf(a, b);
        }
    }
    e->bad = 1;
    return 0.0f;
}

static float ex_primary(Expr *e) {
    ex_ws(e);
    const char c = *e->s;
    if (c == '(') {
        e->s++;
        float v = ex_sum(e);
        ex_ws(e);
        if (*e->s == ')') e->s++;
        else e->bad = 1;
        return v;
    }
    if (isdigit((unsigned char)c) || c == '.') {
        char *end;
        float v = strtof(e->s, &end);
        if (end == e->s) e->bad = 1;
        e->s = end;
        return v;
    }
    if (isalpha((unsigned char)c) || c == '_') {
        char name[32];
        size_t n = 0;
        while (isalnum((unsigned char)*e->s) || *e->s == '_') {
            if (n + 1 < sizeof(name)) name[n++] = *e->s;
            e->s++;
        }
        name[n] = 0;
        ex_ws(e);
        if (*e->s != '(') {
            if (!strcmp(name, "x")) return e->x;
            if (!strcmp(name, "fval")) return e->fval;
            if (!strcmp(name, "pi")) return 3.14159265358979323846f;
            e->bad = 1;
            return 0.0f;
        }
        e->s++;
        float a = ex_sum(e), b = 0.0f;
        int nargs = 1;
        ex_ws(e);
        if (*e->s == ',') {
            e->s++;
            b = ex_sum(e);
            nargs = 2;
            ex_ws(e);
        }
        if (*e->s == ')') e->s++;
        else e->bad = 1;
        return ex_call(e, name, a, b, nargs);
    }
    e->bad = 1;
    return 0.0f;
}

static float ex_unary(Expr *e) {
    ex_ws(e);
    if (*e->s == '-') { e->s++; return -ex_unary(e); }
    if (*e->s == '+') { e->s++; return ex_unary(e); }
    return ex_primary(e);
}

static float ex_product(Expr *e) {
    float v = ex_unary(e);
    for (;;) {
        ex_ws(e);
        const char op = *e->s;
        if (e->bad || (op != '*' && op != '/')) return v;
        e->s++;
        const float r = ex_unary(e);
        v = op == '*' ? v * r : v / r;
    }
}

static float ex_sum(Expr *e) {
    float v = ex_product(e);
    for (;;) {
        ex_ws(e);
        const char op = *e->s;
        if (e->bad || (op != '+' && op != '-')) return v;
        e->s++;
        const float r = ex_product(e);
        v = op == '+' ? v + r : v - r;
    }
}

int tkm_eval_math_expr(const char *expr, float x, float fval, float *out_value) {
    if (!expr || !out_value) return 0;
    Expr e = {expr, x, fval, 0};
    const float v = ex_sum(&e);
    ex_ws(&e);
    if (e.bad || *e.s) return 0;
    *out_value = v;
    return 1;
}

/* ----------------------------------------------------------- fusion rules
 * The four peephole rules of the reference (src/tkm_registry.c:622-820): the
 * same match conditions and the same rewrites of the node table, because the
 * rewritten table is visible through the public TkmGraph. */

/* Walks back from `end` through fluid operators (and QKNorm) to an FC.  On
 * success returns 1 with the FC's id and the chain in forward order. */
static int fc_chain(const TkmGraph *g, int end, int *fc, int *chain, int *len) {
    int rev[TKM_MAX_CHAIN], n = 0;
    for (int cur = end; cur >= 0 && n < TKM_MAX_CHAIN; cur = g->nodes[cur].in0) {
        const TkmNode *nd = &g->nodes[cur];
        if (nd->op == OP_FC) {
            *fc = cur;
            *len = n;
            for (int i = 0; i < n; i++) chain[i] = rev[n - 1 - i];
            return 1;
        }
        if (nd->cat != CAT_FLUID && nd->op != OP_QKNORM) return 0;
        rev[n++] = cur;
    }
    return 0;
}

/* Marks end, its in0, ... dead up to (not including) stop. */
static void kill_back_to(TkmGraph *g, int end, int stop) {
    for (int cur = end; cur >= 0 && cur != stop; cur = g->nodes[cur].in0) g->nodes[cur].dead = 1;
}

static int twin_match(const TkmGraph *g, int id) {
    const TkmNode *n = &g->nodes[id];
    int lf, rf, lc[TKM_MAX_CHAIN], rc[TKM_MAX_CHAIN], ll, rl;
    if (n->op != OP_MUL || n->in0 < 0 || n->in1 < 0) return 0;
    if (!fc_chain(g, n->in0, &lf, lc, &ll) || !fc_chain(g, n->in1, &rf, rc, &rl)) return 0;
    return g->nodes[lf].in0 == g->nodes[rf].in0 && g->nodes[lf].c_out == g->nodes[rf].c_out;
}

static void twin_apply(TkmGraph *g, int id) {
    TkmNode *n = &g->nodes[id];
    int lf = -1, rf = -1;
    fc_chain(g, n->in0, &lf, n->left_nodes, &n->left_len);
    fc_chain(g, n->in1, &rf, n->right_nodes, &n->right_len);
    TkmNode *fc = &g->nodes[lf];
    const int src = fc->in0, half = fc->c_out;
    tkm_log("  [fusion] twin-branch: FC #%d + FC #%d -> one GEMM of %d columns + SwiGLU-style epilogue\n", lf, rf,
            2 * half);
    kill_back_to(g, n->in0, src);
    kill_back_to(g, n->in1, src);
    fc->dead = 0;
    fc->op = OP_FC_TWIN_FUSED;
    fc->cat = CAT_ANCHOR;
    fc->c_out = 2 * half;
    snprintf(fc->tag, sizeof(fc->tag), "twin_gemm2x_%d", fc->id);
    n->in0 = fc->id;
    n->in1 = -1;
    n->c_out = half;
}

static int qkv_match(const TkmGraph *g, int id) {
    const TkmNode *n = &g->nodes[id];
    int f[3], c[3][TKM_MAX_CHAIN], l[3];
    if (n->op != OP_GQA_ATTN || n->in0 < 0 || n->in1 < 0 || n->in2 < 0) return 0;
    const int ins[3] = {n->in0, n->in1, n->in2};
    for (int i = 0; i < 3; i++)
        if (!fc_chain(g, ins[i], &f[i], c[i], &l[i])) return 0;
    return g->nodes[f[0]].in0 == g->nodes[f[1]].in0 && g->nodes[f[1]].in0 == g->nodes[f[2]].in0;
}

static int same_rope(const TkmNode *a, const TkmNode *b) {
    return a->rope_theta == b->rope_theta && a->rope_scale == b->rope_scale &&
           a->rope_low_freq_factor == b->rope_low_freq_factor &&
           a->rope_high_freq_factor == b->rope_high_freq_factor &&
           a->rope_original_context_length == b->rope_original_context_length;
}

static void qkv_apply(TkmGraph *g, int id) {
    TkmNode *n = &g->nodes[id];
    int f[3], c[3][TKM_MAX_CHAIN], l[3];
    const int ins[3] = {n->in0, n->in1, n->in2};
    for (int i = 0; i < 3; i++) fc_chain(g, ins[i], &f[i], c[i], &l[i]);

    /* Q and K chains must agree on QKNorm and on the RoPE configuration */
    int has_norm[2] = {0, 0};
    const TkmNode *rope[2] = {NULL, NULL};
    for (int b = 0; b < 2; b++)
        for (int m = 0; m < l[b]; m++) {
            const TkmNode *cn = &g->nodes[c[b][m]];
            if (cn->op == OP_QKNORM) has_norm[b] = 1;
            if (cn->op == OP_ROPE) rope[b] = cn;
        }
    if (has_norm[0] != has_norm[1] || (!rope[0]) != (!rope[1]) || (rope[0] && !same_rope(rope[0], rope[1]))) {
        tkm_graph_error(g, "[TKM Shape Error] Fused GQA requires matching Q/K QKNorm and RoPE configurations.");
        return;
    }
    if (has_norm[0] && n->head_dim != 64) {
        tkm_graph_error(g, "[TKM Shape Error] QKNorm currently supports 64-dimensional GQA heads only.");
        return;
    }
    TkmNode *fq = &g->nodes[f[0]];
    const TkmNode *fk = &g->nodes[f[1]], *fv = &g->nodes[f[2]];
    const int total = fq->c_out + fk->c_out + fv->c_out;
    tkm_log("  [fusion] 3-way QKV: Q(%d)+K(%d)+V(%d) -> one GEMM of %d columns + QKV prep%s%s\n", fq->c_out,
            fk->c_out, fv->c_out, total, has_norm[0] ? " +QKNorm" : "", rope[0] ? " +RoPE" : "");
    const int src = fq->in0, prep_id = c[0][0];
    for (int i = 0; i < 3; i++) kill_back_to(g, ins[i], src);

    fq->dead = 0;
    fq->op = OP_FC_QKV_FUSED;
    fq->cat = CAT_ANCHOR;
    fq->q_c = fq->c_out;
    fq->k_c = fk->c_out;
    fq->v_c = fv->c_out;
    fq->c_out = total;

    /* the first node of the Q chain (its Bias) becomes the QKV-prep node */
    TkmNode *prep = &g->nodes[prep_id];
    prep->dead = 0;
    prep->op = OP_QKNORM;
    prep->cat = CAT_FLUID;
    prep->in0 = fq->id;
    prep->in1 = prep->in2 = -1;
    prep->q_c = fq->q_c;
    prep->k_c = fq->k_c;
    prep->v_c = fq->v_c;
    prep->c_out = total;
    prep->q_heads = n->q_heads;
    prep->kv_heads = n->kv_heads;
    prep->head_dim = n->head_dim;
    prep->has_qknorm = has_norm[0];
    prep->has_rope = rope[0] != NULL;
    if (rope[0]) {
        prep->rope_theta = rope[0]->rope_theta;
        prep->rope_scale = rope[0]->rope_scale;
        prep->rope_low_freq_factor = rope[0]->rope_low_freq_factor;
        prep->rope_high_freq_factor = rope[0]->rope_high_freq_factor;
        prep->rope_original_context_length = rope[0]->rope_original_context_length;
    }
    snprintf(prep->tag, sizeof(prep->tag), "qkv_prep_%d", prep->id);
    snprintf(fq->tag, sizeof(fq->tag), "qkv3x_gemm_%d", fq->id);
    n->in0 = prep->id;
    n->in1 = n->in2 = -1;
}

static int scale_fold_match(const TkmGraph *g, int id) {
    const TkmNode *n = &g->nodes[id];
    return n->op == OP_SCALE && n->in0 >= 0 && !g->nodes[n->in0].dead && g->nodes[n->in0].op == OP_SCALE;
}

static void scale_fold_apply(TkmGraph *g, int id) {
    TkmNode *n = &g->nodes[id];
    TkmNode *prev = &g->nodes[n->in0];
    tkm_log("  [fusion] scale fold: #%d x #%d -> Scale(%g)\n", prev->id, n->id, prev->fval * n->fval);
    prev->dead = 1;
    n->in0 = prev->in0;
    n->fval = prev->fval * n->fval;
}

static int noop_match(const TkmGraph *g, int id) {
    const TkmNode *n = &g->nodes[id];
    return (n->op == OP_DROP && fabsf(n->fval) < 1e-6f) || (n->op == OP_SCALE && fabsf(n->fval - 1.0f) < 1e-6f);
}

static void noop_apply(TkmGraph *g, int id) {
    TkmNode *n = &g->nodes[id];
    const int up = n->in0;
    tkm_log("  [fusion] no-op bypass: #%d (%s)\n", id, n->tag);
    n->dead = 1;
    for (int k = id + 1; k < g->num_nodes; k++) {
        TkmNode *m = &g->nodes[k];
        if (m->in0 == id) m->in0 = up;
        if (m->in1 == id) m->in1 = up;
        if (m->in2 == id) m->in2 = up;
    }
}

static const TkmFusionRule RULES[] = {
    {"Horizontal_Twin_Branch_Merge", twin_match, twin_apply},
    {"Horizontal_3Way_QKV_Merge", qkv_match, qkv_apply},
    {"Algebraic_Scale_Fold", scale_fold_match, scale_fold_apply},
    {"Dead_NoOp_Elimination", noop_match, noop_apply},
};

const TkmFusionRule *tkm_get_fusion_rules(int *out_count) {
    if (out_count) *out_count = (int)(sizeof(RULES) / sizeof(RULES[0]));
    return RULES;
}
