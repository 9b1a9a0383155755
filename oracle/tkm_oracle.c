/*
 * tkm_oracle.c -- CPU restatement of Tokamak's hot-path semantics (fp64 accumulate).
 *
 * TEST INFRASTRUCTURE ONLY: the parity checker for tokamak_b200's CUDA
 * kernels and the timed CPU baseline.  It is never linked into the product.
 * Citations are to BSODsystem32/Tokamak v4.1.0 (path:line within that project).
 */
#include "tkm_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

int tko_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* threads of the following parallel regions (n >= 1); a launcher may have
 * set OMP_NUM_THREADS=1 for a process that then times the oracle alone */
void tko_set_num_threads(int n) {
#ifdef _OPENMP
    if (n >= 1) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* ---------------------------------------------------------------- attention */

/* src/tkm_gpu.cu:302-438.  One (b, q-head, query) row at a time:
 * s_j = <q, k_j> * scale, masked (causal: j > i) rows contribute nothing,
 * m = max s_j, l = sum exp(s_j - m), o = sum exp(s_j - m) v_j / (l + 1e-8),
 * lse = m + ln(l + 1e-8). */
void tko_attn_fwd(const float *qkv, float *out, float *lse,
                  int B, int S, int Hq, int Hkv, int D, float scale, int causal) {
    const int G = Hq / Hkv;
    const long ld = (long)(Hq + 2 * Hkv) * D;
    const long ldo = (long)Hq * D;
    #pragma omp parallel
    {
        double *sc = (double *)malloc(sizeof(double) * (size_t)S);
        double *acc = (double *)malloc(sizeof(double) * (size_t)D);
        #pragma omp for schedule(dynamic, 1) collapse(2)
        for (int bh = 0; bh < B * Hq; bh++) {
            for (int i = 0; i < S; i++) {
                const int b = bh / Hq, h = bh % Hq, g = h / G;
                const float *q = qkv + ((long)b * S + i) * ld + (long)h * D;
                const int jend = causal ? i + 1 : S;
                double m = -INFINITY;
                for (int j = 0; j < jend; j++) {
                    const float *k = qkv + ((long)b * S + j) * ld + (long)(Hq + g) * D;
                    double dot = 0.0;
                    for (int d = 0; d < D; d++) dot += (double)q[d] * (double)k[d];
                    sc[j] = dot * (double)scale;
                    if (sc[j] > m) m = sc[j];
                }
                double l = 0.0;
                for (int d = 0; d < D; d++) acc[d] = 0.0;
                for (int j = 0; j < jend; j++) {
                    const float *v = qkv + ((long)b * S + j) * ld + (long)(Hq + Hkv + g) * D;
                    double p = exp(sc[j] - m);
                    l += p;
                    for (int d = 0; d < D; d++) acc[d] += p * (double)v[d];
                }
                float *o = out + ((long)b * S + i) * ldo + (long)h * D;
                for (int d = 0; d < D; d++) o[d] = (float)(acc[d] / (l + 1e-8));
                if (lse) lse[(long)bh * S + i] = (float)(m + log(l + 1e-8));
            }
        }
        free(sc);
        free(acc);
    }
}

/* Documented-math backward of the forward above (the reference's dQ path,
 * src/tkm_gpu.cu:503-564, extended with dK = dS^T Q and dV = P^T dO).
 * Parallel over (b, kv head) so that the GQA sum into dK/dV is race free. */
void tko_attn_bwd(const float *qkv, const float *out, const float *dout,
                  const float *lse, float *dqkv,
                  int B, int S, int Hq, int Hkv, int D, float scale, int causal) {
    const int G = Hq / Hkv;
    const long ld = (long)(Hq + 2 * Hkv) * D;
    const long ldo = (long)Hq * D;
    #pragma omp parallel
    {
        double *dk = (double *)malloc(sizeof(double) * (size_t)S * D);
        double *dv = (double *)malloc(sizeof(double) * (size_t)S * D);
        double *dq = (double *)malloc(sizeof(double) * (size_t)D);
        #pragma omp for schedule(dynamic, 1)
        for (int bg = 0; bg < B * Hkv; bg++) {
            const int b = bg / Hkv, g = bg % Hkv;
            memset(dk, 0, sizeof(double) * (size_t)S * D);
            memset(dv, 0, sizeof(double) * (size_t)S * D);
            for (int hh = 0; hh < G; hh++) {
                const int h = g * G + hh;
                for (int i = 0; i < S; i++) {
                    const float *q = qkv + ((long)b * S + i) * ld + (long)h * D;
                    const float *o = out + ((long)b * S + i) * ldo + (long)h * D;
                    const float *dO = dout + ((long)b * S + i) * ldo + (long)h * D;
                    double Di = 0.0;
                    for (int d = 0; d < D; d++) Di += (double)o[d] * (double)dO[d];
                    const double L = lse[((long)b * Hq + h) * S + i];
                    for (int d = 0; d < D; d++) dq[d] = 0.0;
                    const int jend = causal ? i + 1 : S;
                    for (int j = 0; j < jend; j++) {
                        const float *k = qkv + ((long)b * S + j) * ld + (long)(Hq + g) * D;
                        const float *v = qkv + ((long)b * S + j) * ld + (long)(Hq + Hkv + g) * D;
                        double s = 0.0, dp = 0.0;
                        for (int d = 0; d < D; d++) {
                            s += (double)q[d] * (double)k[d];
                            dp += (double)dO[d] * (double)v[d];
                        }
                        const double p = exp(s * (double)scale - L);
                        const double ds = p * (dp - Di) * (double)scale;
                        double *dkj = dk + (long)j * D, *dvj = dv + (long)j * D;
                        for (int d = 0; d < D; d++) {
                            dq[d] += ds * (double)k[d];
                            dkj[d] += ds * (double)q[d];
                            dvj[d] += p * (double)dO[d];
                        }
                    }
                    float *dqr = dqkv + ((long)b * S + i) * ld + (long)h * D;
                    for (int d = 0; d < D; d++) dqr[d] = (float)dq[d];
                }
            }
            for (int j = 0; j < S; j++) {
                float *dkr = dqkv + ((long)b * S + j) * ld + (long)(Hq + g) * D;
                float *dvr = dqkv + ((long)b * S + j) * ld + (long)(Hq + Hkv + g) * D;
                for (int d = 0; d < D; d++) {
                    dkr[d] = (float)dk[(long)j * D + d];
                    dvr[d] = (float)dv[(long)j * D + d];
                }
            }
        }
        free(dk);
        free(dv);
        free(dq);
    }
}

/* ------------------------------------------------------------ row kernels */

void tko_add_rmsnorm_fwd(const float *x, const float *r, float *s, float *y,
                         const float *gamma, float *istd, int rows, int C, float eps) {
    #pragma omp parallel for schedule(static)
    for (int i = 0; i < rows; i++) {
        const float *xr = x + (long)i * C;
        const float *rr = r ? r + (long)i * C : NULL;
        double ss = 0.0;
        for (int c = 0; c < C; c++) {
            /* s is rounded to fp32 the way a stored residual stream would be */
            float v = rr ? xr[c] + rr[c] : xr[c];
            if (s) s[(long)i * C + c] = v;
            ss += (double)v * (double)v;
        }
        double is = 1.0 / sqrt(ss / (double)C + (double)eps);
        if (istd) istd[i] = (float)is;
        for (int c = 0; c < C; c++) {
            float v = rr ? xr[c] + rr[c] : xr[c];
            y[(long)i * C + c] = (float)((double)v * is * (double)gamma[c]);
        }
    }
}

void tko_add_rmsnorm_bwd(const float *dy, const float *s, const float *gamma,
                         const float *istd, const float *ds_skip, float *dx,
                         float *dgamma, int rows, int C) {
    double *dg = (double *)calloc((size_t)C, sizeof(double));
    #pragma omp parallel
    {
        double *dgl = (double *)calloc((size_t)C, sizeof(double));
        #pragma omp for schedule(static)
        for (int i = 0; i < rows; i++) {
            const float *dyr = dy + (long)i * C, *sr = s + (long)i * C;
            const double is = istd[i];
            double m2 = 0.0;
            for (int c = 0; c < C; c++) {
                double xh = (double)sr[c] * is;
                m2 += (double)dyr[c] * (double)gamma[c] * xh;
                dgl[c] += (double)dyr[c] * xh;
            }
            m2 /= (double)C;
            for (int c = 0; c < C; c++) {
                double xh = (double)sr[c] * is;
                double v = is * ((double)dyr[c] * (double)gamma[c] - xh * m2);
                if (ds_skip) v += ds_skip[(long)i * C + c];
                dx[(long)i * C + c] = (float)v;
            }
        }
        #pragma omp critical
        for (int c = 0; c < C; c++) dg[c] += dgl[c];
        free(dgl);
    }
    if (dgamma)
        for (int c = 0; c < C; c++) dgamma[c] += (float)dg[c];
    free(dg);
}

static double sigm(double a) { return 1.0 / (1.0 + exp(-a)); }

void tko_swiglu_fwd(const float *gu, const float *bg, const float *bu, float *h,
                    int rows, int F) {
    #pragma omp parallel for schedule(static)
    for (int i = 0; i < rows; i++) {
        for (int c = 0; c < F; c++) {
            double a = (double)gu[(long)i * 2 * F + c] + (bg ? bg[c] : 0.0);
            double b = (double)gu[(long)i * 2 * F + F + c] + (bu ? bu[c] : 0.0);
            h[(long)i * F + c] = (float)(a * sigm(a) * b);
        }
    }
}

void tko_swiglu_bwd(const float *dh, const float *gu, const float *bg, const float *bu,
                    float *dgu, float *dbg, float *dbu, int rows, int F) {
    double *sg = (double *)calloc((size_t)F, sizeof(double));
    double *su = (double *)calloc((size_t)F, sizeof(double));
    #pragma omp parallel
    {
        double *lg = (double *)calloc((size_t)F, sizeof(double));
        double *lu = (double *)calloc((size_t)F, sizeof(double));
        #pragma omp for schedule(static)
        for (int i = 0; i < rows; i++) {
            for (int c = 0; c < F; c++) {
                double a = (double)gu[(long)i * 2 * F + c] + (bg ? bg[c] : 0.0);
                double b = (double)gu[(long)i * 2 * F + F + c] + (bu ? bu[c] : 0.0);
                double d = dh[(long)i * F + c];
                double sa = sigm(a);
                double da = d * b * sa * (1.0 + a * (1.0 - sa));
                double db = d * a * sa;
                dgu[(long)i * 2 * F + c] = (float)da;
                dgu[(long)i * 2 * F + F + c] = (float)db;
                lg[c] += da;
                lu[c] += db;
            }
        }
        #pragma omp critical
        for (int c = 0; c < F; c++) { sg[c] += lg[c]; su[c] += lu[c]; }
        free(lg);
        free(lu);
    }
    if (dbg) for (int c = 0; c < F; c++) dbg[c] += (float)sg[c];
    if (dbu) for (int c = 0; c < F; c++) dbu[c] += (float)su[c];
    free(sg);
    free(su);
}

/* src/tkm_codegen.c:43-70, evaluated in fp64. */
static double rope_inv_freq(int lane, int hd, double theta, double scale,
                            double low_ff, double high_ff, double orig_ctx) {
    double inv = exp(-log(theta) * (double)lane / (double)hd);
    if (scale > 1.0) {
        double wavelen = 6.283185307179586 / inv;
        double low_wavelen = orig_ctx / low_ff;
        double high_wavelen = orig_ctx / high_ff;
        if (wavelen > low_wavelen) inv /= scale;
        else if (wavelen >= high_wavelen) {
            double smooth = (orig_ctx / wavelen - low_ff) / (high_ff - low_ff);
            inv *= 1.0 - smooth * (1.0 - 1.0 / scale);
        }
    }
    return inv;
}

void tko_qkv_prep_fwd(const float *in, const float *bias, const float *qk_gain,
                      float *out, float *save_istd,
                      int rows, int S, int Hq, int Hkv, int D,
                      int has_qknorm, int has_rope, float theta, float rope_scale,
                      float low_ff, float high_ff, float orig_ctx) {
    const int C = (Hq + 2 * Hkv) * D, nqk = Hq + Hkv;
    #pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; r++) {
        const int pos = r % S;
        for (int hd = 0; hd < Hq + 2 * Hkv; hd++) {
            double v[256];
            for (int d = 0; d < D; d++) {
                int c = hd * D + d;
                v[d] = (double)in[(long)r * C + c] + (bias ? bias[c] : 0.0);
            }
            if (hd < nqk) {
                if (has_qknorm) {
                    double ss = 0.0;
                    for (int d = 0; d < D; d++) ss += v[d] * v[d];
                    double is = 1.0 / sqrt(ss / (double)D + 1e-5);
                    if (save_istd) save_istd[(long)r * nqk + hd] = (float)is;
                    for (int d = 0; d < D; d++) v[d] = v[d] * is * (qk_gain ? qk_gain[hd * D + d] : 1.0);
                }
                if (has_rope) {
                    for (int i = 0; i < D / 2; i++) {
                        double f = (double)pos * rope_inv_freq(i, D, theta, rope_scale, low_ff, high_ff, orig_ctx);
                        double sn = sin(f), cs = cos(f);
                        double x0 = v[2 * i], x1 = v[2 * i + 1];
                        v[2 * i] = x0 * cs - x1 * sn;
                        v[2 * i + 1] = x0 * sn + x1 * cs;
                    }
                }
            }
            for (int d = 0; d < D; d++) out[(long)r * C + hd * D + d] = (float)v[d];
        }
    }
}

void tko_qkv_prep_bwd(const float *dout, const float *in, const float *bias,
                      const float *qk_gain, const float *save_istd,
                      float *din, float *dbias, float *dgain,
                      int rows, int S, int Hq, int Hkv, int D,
                      int has_qknorm, int has_rope, float theta, float rope_scale,
                      float low_ff, float high_ff, float orig_ctx) {
    const int C = (Hq + 2 * Hkv) * D, nqk = Hq + Hkv;
    double *db = (double *)calloc((size_t)C, sizeof(double));
    double *dgm = (double *)calloc((size_t)C, sizeof(double));
    #pragma omp parallel
    {
        double *ldb = (double *)calloc((size_t)C, sizeof(double));
        double *ldg = (double *)calloc((size_t)C, sizeof(double));
        #pragma omp for schedule(static)
        for (int r = 0; r < rows; r++) {
            const int pos = r % S;
            for (int hd = 0; hd < Hq + 2 * Hkv; hd++) {
                double dy[256];
                for (int d = 0; d < D; d++) dy[d] = dout[(long)r * C + hd * D + d];
                if (hd < nqk) {
                    if (has_rope) {
                        for (int i = 0; i < D / 2; i++) {
                            double f = (double)pos * rope_inv_freq(i, D, theta, rope_scale, low_ff, high_ff, orig_ctx);
                            double sn = sin(f), cs = cos(f);
                            double y0 = dy[2 * i], y1 = dy[2 * i + 1];
                            dy[2 * i] = y0 * cs + y1 * sn;
                            dy[2 * i + 1] = -y0 * sn + y1 * cs;
                        }
                    }
                    if (has_qknorm) {
                        double is = save_istd[(long)r * nqk + hd];
                        double xh[256], m2 = 0.0;
                        for (int d = 0; d < D; d++) {
                            int c = hd * D + d;
                            xh[d] = ((double)in[(long)r * C + c] + (bias ? bias[c] : 0.0)) * is;
                            double gm = qk_gain ? qk_gain[c] : 1.0;
                            ldg[c] += dy[d] * xh[d];
                            m2 += dy[d] * gm * xh[d];
                        }
                        m2 /= (double)D;
                        for (int d = 0; d < D; d++) {
                            double gm = qk_gain ? qk_gain[hd * D + d] : 1.0;
                            dy[d] = is * (dy[d] * gm - xh[d] * m2);
                        }
                    }
                }
                for (int d = 0; d < D; d++) {
                    int c = hd * D + d;
                    ldb[c] += dy[d];
                    din[(long)r * C + c] += (float)dy[d];
                }
            }
        }
        #pragma omp critical
        for (int c = 0; c < C; c++) { db[c] += ldb[c]; dgm[c] += ldg[c]; }
        free(ldb);
        free(ldg);
    }
    if (dbias) for (int c = 0; c < C; c++) dbias[c] += (float)db[c];
    if (dgain) for (int c = 0; c < nqk * D; c++) dgain[c] += (float)dgm[c];
    free(db);
    free(dgm);
}

void tko_softmax_fwd(const float *x, float *p, int rows, int C) {
    #pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; r++) {
        const float *xr = x + (long)r * C;
        double m = -INFINITY, s = 0.0;
        for (int c = 0; c < C; c++) if (xr[c] > m) m = xr[c];
        for (int c = 0; c < C; c++) s += exp((double)xr[c] - m);
        for (int c = 0; c < C; c++) p[(long)r * C + c] = (float)(exp((double)xr[c] - m) / s);
    }
}

void tko_softmax_bwd(const float *p, const float *dp, float *dx, int rows, int C) {
    #pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; r++) {
        double dot = 0.0;
        for (int c = 0; c < C; c++) dot += (double)p[(long)r * C + c] * (double)dp[(long)r * C + c];
        for (int c = 0; c < C; c++) {
            long k = (long)r * C + c;
            dx[k] += (float)((double)p[k] * ((double)dp[k] - dot));
        }
    }
}

/* src/tkm_gpu.cu:632-682, one row at a time. */
float tko_softmax_loss(const float *logits, const int32_t *labels, float *dlogits,
                       int *correct, int rows, int C, int kind, float gamma) {
    double total = 0.0;
    int corr = 0;
    const double inv_rows = 1.0 / (double)rows;
    #pragma omp parallel for schedule(static) reduction(+:total, corr)
    for (int r = 0; r < rows; r++) {
        const float *x = logits + (long)r * C;
        double m = -INFINITY;
        int pred = 0;
        for (int c = 0; c < C; c++) if (x[c] > m) { m = x[c]; pred = c; }
        double s = 0.0;
        for (int c = 0; c < C; c++) s += exp((double)x[c] - m);
        const int y = labels ? labels[r] : 0;
        if (pred == y) corr++;
        double pt = exp((double)x[y] - m) / s;
        if (pt < 1e-7) pt = 1e-7;
        double fw = pow(1.0 - pt, (double)gamma);
        double fgs = kind == 1 ? fw - (double)gamma * pt * pow(1.0 - pt, (double)gamma - 1.0) * log(pt) : 1.0;
        double bdot = 0.0;
        if (kind == 2)
            for (int c = 0; c < C; c++) {
                double pc = exp((double)x[c] - m) / s;
                bdot += pc * (pc - (c == y ? 1.0 : 0.0));
            }
        if (kind == 0) total += -log(pt) * inv_rows;
        else if (kind == 1) total += -fw * log(pt) * inv_rows;
        for (int c = 0; c < C; c++) {
            double pc = exp((double)x[c] - m) / s;
            double t = c == y ? 1.0 : 0.0, g;
            if (kind == 0) g = pc - t;
            else if (kind == 1) g = fgs * (pc - t);
            else {
                double diff = pc - t;
                total += diff * diff / (double)C * inv_rows;
                g = 2.0 / (double)C * pc * (diff - bdot);
            }
            if (dlogits) dlogits[(long)r * C + c] = (float)(g * inv_rows);
        }
    }
    if (correct) *correct = corr;
    return (float)total;
}

void tko_sgd(float *p, float *v, const float *g, long n, float lr, float momentum,
             float wd, int apply_wd) {
    #pragma omp parallel for schedule(static)
    for (long i = 0; i < n; i++) {
        float gi = g[i];
        if (apply_wd) gi = fmaf(wd, p[i], gi);
        float vi = fmaf(momentum, v[i], gi);
        p[i] = fmaf(-lr, fmaf(momentum, vi, gi), p[i]);
        v[i] = vi;
    }
}
