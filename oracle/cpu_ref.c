/* cpu_ref.c -- THE ORACLE (test infrastructure only; see cpu_ref.h).
 *
 * A plain-C fp64 restatement of coherence-kernel's Form recipes for the quantized dequant /
 * matvec / MoE path, in the reference's own operation order so every fp64 value is bit-identical
 * to what the reference runtime (fkwu) computes.  Only tests/, the smoke check and bench.py's CPU
 * baseline leg call it.  Built with -ffp-contract=off: a fused multiply-add would change the
 * rounding the reference's separate mul and add perform.
 */
#include "cpu_ref.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ---------------------------------------------------------------- f16 / bf16 decode
 * form/form-stdlib/f16-decode.fk:28-57.  fd-value: mantissa = bits mod 2^mb, exponent field =
 * (bits / 2^mb) mod 2^eb, sign = bits / 2^(eb+mb); normal -> 2^(e-bias) * (1 + mant/2^mb),
 * subnormal -> 2^(1-bias) * mant/2^mb; a set sign bit gives 0.0 - magnitude.  Powers of two are
 * exact (format-arith.fk:17-19 fq-pow2), so ldexp is the same value. */
static double fd_value(uint32_t bits, int eb, int mb) {
    uint32_t mant = bits % (1u << mb);
    uint32_t ex = (bits >> mb) % (1u << eb);
    uint32_t sgn = bits >> (eb + mb);
    int bias = (1 << (eb - 1)) - 1;
    double frac = (1.0 * (double)mant) / ldexp(1.0, mb);
    double mag = (ex == 0) ? ldexp(1.0, 1 - bias) * frac : ldexp(1.0, (int)ex - bias) * (1.0 + frac);
    return sgn == 1 ? 0.0 - mag : mag;
}
double ckr_f16(uint32_t bits) { return fd_value(bits & 0xFFFFu, 5, 10); }
double ckr_bf16(uint32_t bits) { return fd_value(bits & 0xFFFFu, 8, 7); }

/* ---------------------------------------------------------------- Q8_0
 * form/form-stdlib/q8-0-msl.fk:53-70: block = idx/32 at 34-byte stride; d = fd-f16 of the LE
 * u16 at +0; q = two's-complement byte at +2+i (q6k-s8); w = d * q. */
double ckr_q80_at(const uint8_t *src, int64_t base, int64_t idx) {
    int64_t b = base + (idx / 32) * 34;
    int64_t i = idx - (idx / 32) * 32;
    double d = ckr_f16((uint32_t)src[b] + 256u * (uint32_t)src[b + 1]);
    int q = (int)src[b + 2 + i];
    if (q >= 128) q -= 256;
    return d * (double)q;
}

/* ---------------------------------------------------------------- Q4_K
 * form/form-stdlib/q4k-msl.fk:55-86 (q4m-flat-at) over q4k-dequant.fk:19-43's unpack:
 * block = idx/256 at 144-byte stride; d f16 @+0, dmin f16 @+2, scales[12] @+4, qs[128] @+16;
 * i = idx mod 256, c = i/64, half = (i mod 64)/32, l = i mod 32, j = 2c + half;
 * get_scale_min_k4 for (sc, m); nib = low nibble of qs[32c+l] when half = 0 else the high one;
 * w = (d * sc) * nib - dmin * m. */
static inline int q4k_scale(const uint8_t *s, int j) {
    return j < 4 ? (s[j] % 64) : ((s[j + 4] % 16) + (s[j - 4] / 64) * 16);
}
static inline int q4k_min(const uint8_t *s, int j) {
    return j < 4 ? (s[j + 4] % 64) : ((s[j + 4] / 16) + (s[j] / 64) * 16);
}
uint32_t ckr_q4k_codes(const uint8_t *src, int64_t base, int64_t idx) {
    const uint8_t *b = src + base + (idx / 256) * 144;
    int i = (int)(idx % 256);
    int c = i / 64, within = i % 64, hf = within / 32, l = within % 32, j = 2 * c + hf;
    int qbyte = b[16 + c * 32 + l];
    int nib = hf == 0 ? qbyte % 16 : qbyte / 16;
    return (uint32_t)q4k_scale(b + 4, j) | ((uint32_t)q4k_min(b + 4, j) << 8) | ((uint32_t)nib << 16);
}
double ckr_q4k_at(const uint8_t *src, int64_t base, int64_t idx) {
    const uint8_t *b = src + base + (idx / 256) * 144;
    uint32_t codes = ckr_q4k_codes(src, base, idx);
    double d = ckr_f16((uint32_t)b[0] + 256u * (uint32_t)b[1]);
    double dmin = ckr_f16((uint32_t)b[2] + 256u * (uint32_t)b[3]);
    double sc = (double)(codes & 0xFF), m = (double)((codes >> 8) & 0xFF), nib = (double)(codes >> 16);
    return (d * sc) * nib - dmin * m;
}

void ckr_q80_dequant(const uint8_t *qb, int64_t off, int64_t n, double *w) {
    for (int64_t i = 0; i < n; i++) w[i] = ckr_q80_at(qb, 0, off + i);
}

/* Block-wise Q4_K dequant of the flat range [off, off+n): the same values as q4m-flat-at (the
 * same d, dmin, sc, m, nib and the same two products and subtraction), decoded once per
 * sub-block instead of once per weight. */
void ckr_q4k_dequant(const uint8_t *qb, int64_t off, int64_t n, double *w) {
    int64_t idx = off, end = off + n;
    while (idx < end) {
        const uint8_t *b = qb + (idx / 256) * 144;
        double d = ckr_f16((uint32_t)b[0] + 256u * (uint32_t)b[1]);
        double dmin = ckr_f16((uint32_t)b[2] + 256u * (uint32_t)b[3]);
        int i = (int)(idx % 256);
        while (i < 256 && idx < end) {
            int c = i / 64, hf = (i % 64) / 32, j = 2 * c + hf;
            double dsc = d * (double)q4k_scale(b + 4, j);
            double dm = dmin * (double)q4k_min(b + 4, j);
            int l0 = i % 32;
            for (int l = l0; l < 32 && idx < end; l++, i++, idx++) {
                int qbyte = b[16 + c * 32 + l];
                int nib = hf == 0 ? qbyte % 16 : qbyte / 16;
                w[idx - off] = dsc * (double)nib - dm;
            }
        }
    }
}

/* ---------------------------------------------------------------- Q6_K
 * form/form-stdlib/q6k-msl.fk:62-81 (q6m-flat-at) over q6k-dequant.fk:29-61's decomposition:
 * block = idx/256 at 210-byte stride; ql[128] @+0, qh[64] @+128, scales[16] (signed) @+192,
 * d f16 @+208.  i = idx mod 256, h = i/128, wi = i mod 128, l = wi mod 32, g = wi/32, is = l/16;
 * nib = low nibble of ql[64h + l + 32 (g mod 2)] for g < 2 else the high one; hi = (qh[32h + l]
 * / 4^g) mod 4; q = nib + 16 hi - 32; sc = s8(scales[8h + is + 2g]); w = (d * sc) * q. */
uint32_t ckr_q6k_codes(const uint8_t *src, int64_t base, int64_t idx) {
    const uint8_t *b = src + base + (idx / 256) * 210;
    int i = (int)(idx % 256);
    int h = i / 128, wi = i % 128, l = wi % 32, g = wi / 32, is = l / 16;
    int qlb = b[64 * h + l + 32 * (g % 2)];
    int nib = g / 2 == 0 ? qlb % 16 : qlb / 16;
    static const int pow4[4] = {1, 4, 16, 64};
    int hi = (b[128 + 32 * h + l] / pow4[g]) % 4;
    int scb = b[192 + 8 * h + is + 2 * g];
    /* the 6-bit code q + 32 (0..63) in bits 0..7 and the scale byte in bits 8..15 */
    return (uint32_t)(nib + 16 * hi) | ((uint32_t)scb << 8);
}
double ckr_q6k_at(const uint8_t *src, int64_t base, int64_t idx) {
    const uint8_t *b = src + base + (idx / 256) * 210;
    uint32_t codes = ckr_q6k_codes(src, base, idx);
    int q = (int)(codes & 0xFF) - 32;
    int sc = (int)((codes >> 8) & 0xFF);
    if (sc >= 128) sc -= 256;
    double d = ckr_f16((uint32_t)b[208] + 256u * (uint32_t)b[209]);
    return (d * (double)sc) * (double)q;
}
void ckr_q6k_dequant(const uint8_t *qb, int64_t off, int64_t n, double *w) {
    for (int64_t i = 0; i < n; i++) w[i] = ckr_q6k_at(qb, 0, off + i);
}

/* ---------------------------------------------------------------- the right fold
 * form/form-stdlib/transformer-block.fk:25-26 tb-dot: a0*b0 + (a1*b1 + (... + (an*bn + 0.0))). */
double ckr_dot(const double *a, const double *b, int64_t n) {
    double acc = 0.0;
    for (int64_t j = n - 1; j >= 0; j--) {
        double p = a[j] * b[j];
        acc = p + acc;
    }
    return acc;
}

/* four independent right folds at once (the same per-row order; only the interleaving differs) */
static void dot4(const double *r0, const double *r1, const double *r2, const double *r3,
                 const double *x, int64_t n, double *out) {
    double a0 = 0.0, a1 = 0.0, a2 = 0.0, a3 = 0.0;
    for (int64_t j = n - 1; j >= 0; j--) {
        double xj = x[j];
        a0 = r0[j] * xj + a0;
        a1 = r1[j] * xj + a1;
        a2 = r2[j] * xj + a2;
        a3 = r3[j] * xj + a3;
    }
    out[0] = a0; out[1] = a1; out[2] = a2; out[3] = a3;
}

void ckr_q80_matvec(const uint8_t *qb, const double *x, double *y, int64_t rows, int64_t cols) {
    double *w = (double *)malloc(sizeof(double) * (size_t)cols);
    for (int64_t r = 0; r < rows; r++) {
        ckr_q80_dequant(qb, r * cols, cols, w);
        y[r] = ckr_dot(w, x, cols);
    }
    free(w);
}

void ckr_q6k_matvec(const uint8_t *qb, const double *x, double *y, int64_t rows, int64_t cols) {
    double *w = (double *)malloc(sizeof(double) * (size_t)cols);
    for (int64_t r = 0; r < rows; r++) {
        ckr_q6k_dequant(qb, r * cols, cols, w);
        y[r] = ckr_dot(w, x, cols);
    }
    free(w);
}

void ckr_q4k_matvec(const uint8_t *qb, const double *x, double *y, int64_t rows, int64_t cols) {
    double *w = (double *)malloc(sizeof(double) * (size_t)cols);
    for (int64_t r = 0; r < rows; r++) {
        ckr_q4k_dequant(qb, r * cols, cols, w);
        y[r] = ckr_dot(w, x, cols);
    }
    free(w);
}

/* ---------------------------------------------------------------- threads */
typedef void (*ckr_job_fn)(void *ctx, int64_t i0, int64_t i1);
typedef struct { ckr_job_fn fn; void *ctx; int64_t i0, i1; } ckr_job;
static void *ckr_job_main(void *p) {
    ckr_job *j = (ckr_job *)p;
    j->fn(j->ctx, j->i0, j->i1);
    return NULL;
}
static void ckr_parallel(ckr_job_fn fn, void *ctx, int64_t n, int nthreads) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    if ((int64_t)nthreads > n) nthreads = (int)(n > 0 ? n : 1);
    if (nthreads == 1) { fn(ctx, 0, n); return; }
    pthread_t th[256];
    ckr_job jobs[256];
    for (int t = 0; t < nthreads; t++) {
        jobs[t].fn = fn; jobs[t].ctx = ctx;
        jobs[t].i0 = n * t / nthreads; jobs[t].i1 = n * (t + 1) / nthreads;
        pthread_create(&th[t], NULL, ckr_job_main, &jobs[t]);
    }
    for (int t = 0; t < nthreads; t++) pthread_join(th[t], NULL);
}

typedef struct {
    const uint8_t *qb; const double *x; double *y;
    int64_t rows, cols, r0, r1;
} mm_ctx;
static void mm_job(void *p, int64_t t0, int64_t t1) {
    mm_ctx *c = (mm_ctx *)p;
    double *w = (double *)malloc(sizeof(double) * (size_t)c->cols);
    for (int64_t r = c->r0; r < c->r1; r++) {
        ckr_q4k_dequant(c->qb, r * c->cols, c->cols, w);
        for (int64_t t = t0; t < t1; t++) c->y[t * c->rows + r] = ckr_dot(w, c->x + t * c->cols, c->cols);
    }
    free(w);
}
void ckr_q4k_matmul(const uint8_t *qb, const double *x, double *y, int64_t rows, int64_t cols,
                    int64_t ntok, int64_t r0, int64_t r1, int nthreads) {
    mm_ctx c = {qb, x, y, rows, cols, r0, r1};
    ckr_parallel(mm_job, &c, ntok, nthreads);
}

/* ---------------------------------------------------------------- scalar numerics */

/* transformer-numerics.fk:16-24.  tn-exp-acc: 14 Taylor terms, term' = term*(x/n), acc' = acc +
 * term*(x/n); tn-exp-reduce halves x until |x| <= 0.5 (tn-abs), then squares back k times. */
double ckr_exp(double x) {
    int k = 0;
    for (;;) {
        double ax = x < 0.0 ? 0.0 - x : x;
        if (ax <= 0.5) break;
        x = x / 2.0;
        k = k + 1;
    }
    double n = 1.0, term = 1.0, acc = 1.0;
    while (!(n > 14.0)) {
        double t = term * (x / n);
        acc = acc + t;
        term = t;
        n = n + 1.0;
    }
    for (int i = 0; i < k; i++) acc = acc * acc;
    return acc;
}

/* transformer-numerics.fk:32-34: Newton from v itself, 50 fixed iterations. */
double ckr_sqrt(double v) {
    if (v <= 0.0) return 0.0;
    double g = v;
    for (int n = 50; n > 0; n--) g = 0.5 * (g + v / g);
    return g;
}

/* llama-numerics.fk:40-50 ln-rmsnorm: o_i = (x_i * (1 / rms)) * g_i, rms = tn-sqrt(ms + eps), ms =
 * the left-fold sum of x_i * x_i divided by the float-counted length (tn-flen). */
void ckr_rmsnorm(const double *x, const double *g, int64_t n, double eps, double *out) {
    double acc = 0.0;
    for (int64_t i = 0; i < n; i++) acc = acc + x[i] * x[i];
    double flen = 0.0;
    for (int64_t i = 0; i < n; i++) flen = 1.0 + flen;
    double s = 1.0 / ckr_sqrt(acc / flen + eps);
    for (int64_t i = 0; i < n; i++) out[i] = (x[i] * s) * g[i];
}

/* trig.fk:40-53 fln: e*LN2 + ln-m(mantissa), ln-m(m) = 2*(z + sum_j z^(2j+3)/(2j+3)), 14 terms. */
double ckr_ln(double x) {
    double xf = x * 1.0;
    long long e = 0;
    double a = xf;
    if (a >= 1.0) { while (a >= 2.0) { a = a * 0.5; e = e + 1; } }
    else { while (a < 1.0) { a = a * 2.0; e = e - 1; } }
    double m = xf;
    for (;;) {
        if (m >= 2.0) m = m * 0.5;
        else if (m < 1.0) m = m * 2.0;
        else break;
    }
    double z = (m - 1.0) / (m + 1.0);
    double z2 = z * z, zpow = z, acc = 0.0;
    for (long long j = 0; j < 14; j++) {
        double np = zpow * z2;
        acc = acc + np / ((double)(2 * (j + 1)) + 1.0);
        zpow = np;
    }
    double lnm = 2.0 * (z + acc);
    return (double)e * 0.6931471805599453 + lnm;
}

double ckr_sigmoid(double x) { return 1.0 / (1.0 + ckr_exp(0.0 - x)); }
double ckr_silu(double x) { return x * ckr_sigmoid(x); }

/* ---------------------------------------------------------------- routers */

/* moe-msl.fk:73-106.  mm-softmax: mx = mm-max over the tail starting from the head (strict >),
 * e_i = tn-exp(x_i - mx), sum = left fold from 0.0, p_i = e_i * (1/sum).  mm-topk: k rounds of
 * mm-argmax-free (the first free index is taken, then strict > replaces it), best first. */
void ckr_route_softmax(const double *logits, int ne, int nsel, int renorm, int32_t *ids,
                       double *wts, double *probs) {
    double p[1024];
    unsigned char taken[1024];
    double mx = logits[0];
    for (int i = 1; i < ne; i++) if (logits[i] > mx) mx = logits[i];
    double s = 0.0;
    for (int i = 0; i < ne; i++) { p[i] = ckr_exp(logits[i] - mx); s = s + p[i]; }
    double inv = 1.0 / s;
    for (int i = 0; i < ne; i++) { p[i] = p[i] * inv; taken[i] = 0; }
    for (int k = 0; k < nsel; k++) {
        int best = -1;
        double bv = 0.0;
        for (int i = 0; i < ne; i++) {
            if (taken[i]) continue;
            if (best == -1 || p[i] > bv) { best = i; bv = p[i]; }
        }
        taken[best] = 1;
        ids[k] = best;
        wts[k] = p[best];
    }
    if (renorm) {
        double ws = 0.0;
        for (int k = 0; k < nsel; k++) ws = ws + wts[k];
        double winv = 1.0 / ws;
        for (int k = 0; k < nsel; k++) wts[k] = wts[k] * winv;
    }
    if (probs) memcpy(probs, p, sizeof(double) * (size_t)ne);
}

/* dsv4-forward.fk:72-81 dsv4-argmax / dsv4-topk: repeated argmax (strict >, the first maximum
 * wins), each winner overwritten with -1e9, the list built by cons so the LAST pick comes first.
 * Writes the picks in that list order to out[0..k). */
static void dsv4_topk(double *scores, int n, int k, int32_t *out) {
    for (int r = 0; r < k; r++) {
        double best = scores[0];
        int bi = 0;
        for (int i = 1; i < n; i++) if (scores[i] > best) { best = scores[i]; bi = i; }
        scores[bi] = -1000000000.0;
        out[k - 1 - r] = bi;
    }
}

/* dsv4-forward.fk:105-111 (dsv4-routed-moe's weights): tn-sum of the gathered probs (left fold
 * from 0.0), floored at 2^-14, each weight times (wscale / s). */
static void dsv4_weights(const double *probs, const int32_t *sel, int k, double wscale, double *wts) {
    double s0 = 0.0;
    for (int i = 0; i < k; i++) s0 = s0 + probs[sel[i]];
    double s = s0 < 0.00006103515625 ? 0.00006103515625 : s0;
    double sc = wscale / s;
    for (int i = 0; i < k; i++) wts[i] = probs[sel[i]] * sc;
}

void ckr_route_dsv4(const double *logits, const double *bias, int ne, int nused, double wscale,
                    int32_t *ids, double *wts) {
    double probs[1024], score[1024];
    for (int i = 0; i < ne; i++) {
        /* dsv4-forward.fk:65-69: sqrt(fln(1 + tn-exp(z))) */
        probs[i] = ckr_sqrt(ckr_ln(1.0 + ckr_exp(logits[i])));
        score[i] = probs[i] + bias[i];
    }
    dsv4_topk(score, ne, nused, ids);
    dsv4_weights(probs, ids, nused, wscale, wts);
}

void ckr_route_sigmoid_group(const double *logits, const double *bias, int ne, int ngroups,
                             int topk_groups, int nused, double wscale, int32_t *ids, double *wts,
                             double *margin) {
    double probs[1024], score[1024], masked[1024], gscore[64], tmp[1024];
    int gs = ne / ngroups;
    for (int i = 0; i < ne; i++) {
        probs[i] = ckr_sigmoid(logits[i]);
        score[i] = probs[i] + bias[i];
    }
    /* group score: tn-sum over the dsv4-gather of the group's dsv4-topk-2 (second, best) */
    for (int g = 0; g < ngroups; g++) {
        int32_t two[2];
        memcpy(tmp, score + g * gs, sizeof(double) * (size_t)gs);
        dsv4_topk(tmp, gs, 2, two);
        gscore[g] = (0.0 + score[g * gs + two[0]]) + score[g * gs + two[1]];
    }
    int32_t gsel[64];
    memcpy(tmp, gscore, sizeof(double) * (size_t)ngroups);
    dsv4_topk(tmp, ngroups, topk_groups, gsel);
    unsigned char gon[64];
    memset(gon, 0, sizeof(gon));
    for (int i = 0; i < topk_groups; i++) gon[gsel[i]] = 1;
    for (int i = 0; i < ne; i++) masked[i] = gon[i / gs] ? score[i] : -1000000000.0;
    memcpy(tmp, masked, sizeof(double) * (size_t)ne);
    dsv4_topk(tmp, ne, nused, ids);
    dsv4_weights(probs, ids, nused, wscale, wts);
    if (margin) {
        double gmin = 1e300, gmax = -1e300, emin = 1e300, emax = -1e300;
        for (int g = 0; g < ngroups; g++) {
            if (gon[g]) { if (gscore[g] < gmin) gmin = gscore[g]; }
            else if (gscore[g] > gmax) gmax = gscore[g];
        }
        unsigned char on[1024];
        memset(on, 0, (size_t)ne);
        for (int i = 0; i < nused; i++) on[ids[i]] = 1;
        for (int i = 0; i < ne; i++) {
            if (!gon[i / gs]) continue;
            if (on[i]) { if (score[i] < emin) emin = score[i]; }
            else if (score[i] > emax) emax = score[i];
        }
        double mg = (topk_groups < ngroups) ? gmin - gmax : 1e300;
        double me = emin - emax;
        *margin = mg < me ? mg : me;
    }
}

/* ---------------------------------------------------------------- the MoE layer */
typedef struct {
    const ckr_moe_cfg *cfg;
    const uint8_t *w_gate, *w_up, *w_down, *s_gate, *s_up, *s_down;
    const float *router_w, *bias;
    const uint16_t *x_bf16;
    const int64_t *tok;
    int32_t *ids;
    double *wts, *out, *margin;
} moe_ctx;

static int64_t q4k_bytes(int64_t n) { return (n / 256) * 144; }

/* one token's logits: tb-matvec of the fp32 router rows with x (transformer-block.fk:27) */
static void router_logits(const moe_ctx *c, const double *x, double *logits, double *wrow4) {
    const ckr_moe_cfg *cfg = c->cfg;
    int64_t H = cfg->hidden;
    int e = 0;
    for (; e + 4 <= cfg->n_experts; e += 4) {
        for (int q = 0; q < 4; q++)
            for (int64_t j = 0; j < H; j++) wrow4[q * H + j] = (double)c->router_w[(int64_t)(e + q) * H + j];
        dot4(wrow4, wrow4 + H, wrow4 + 2 * H, wrow4 + 3 * H, x, H, logits + e);
    }
    for (; e < cfg->n_experts; e++) {
        for (int64_t j = 0; j < H; j++) wrow4[j] = (double)c->router_w[(int64_t)e * H + j];
        logits[e] = ckr_dot(wrow4, x, H);
    }
}

/* out = down * mid, mid_r = silu(gate_r . x) * (up_r . x) * w  (dsv4-mid with the clamp off;
 * w = 1.0 reproduces ln-swiglu for the softmax layer). */
static void expert_out(const uint8_t *g, const uint8_t *u, const uint8_t *d, int64_t H, int64_t I,
                       const double *x, double w, double *y, double *wrow, double *mid) {
    for (int64_t r = 0; r < I; r++) {
        ckr_q4k_dequant(g, r * H, H, wrow);
        double gv = ckr_dot(wrow, x, H);
        ckr_q4k_dequant(u, r * H, H, wrow);
        double uv = ckr_dot(wrow, x, H);
        mid[r] = (ckr_silu(gv) * uv) * w;
    }
    for (int64_t r = 0; r < H; r++) {
        ckr_q4k_dequant(d, r * I, I, wrow);
        y[r] = ckr_dot(wrow, mid, I);
    }
}

static void moe_job(void *p, int64_t i0, int64_t i1) {
    moe_ctx *c = (moe_ctx *)p;
    const ckr_moe_cfg *cfg = c->cfg;
    int64_t H = cfg->hidden, I = cfg->inter;
    int64_t big = H > I ? H : I;
    double *x = (double *)malloc(sizeof(double) * (size_t)H);
    double *wrow = (double *)malloc(sizeof(double) * (size_t)big * 4);
    double *mid = (double *)malloc(sizeof(double) * (size_t)I);
    double *y = (double *)malloc(sizeof(double) * (size_t)H);
    double logits[1024];
    int64_t eb_gu = q4k_bytes(I * H), eb_d = q4k_bytes(H * I);
    for (int64_t i = i0; i < i1; i++) {
        int64_t t = c->tok ? c->tok[i] : i;
        for (int64_t j = 0; j < H; j++) x[j] = ckr_bf16(c->x_bf16[t * H + j]);
        router_logits(c, x, logits, wrow);
        double bias[1024];
        for (int e = 0; e < cfg->n_experts; e++) bias[e] = c->bias ? (double)c->bias[e] : 0.0;
        int32_t *ids = c->ids + i * cfg->nsel;
        double *wts = c->wts + i * cfg->nsel;
        double mg = 0.0;
        if (cfg->mode == 3) {
            ckr_route_softmax(logits, cfg->n_experts, cfg->nsel, 0, ids, wts, NULL);
            /* k/k+1 logit gap: softmax is monotonic, so this is the decision margin */
            double kth = 1e300, next = -1e300;
            unsigned char on[1024];
            memset(on, 0, sizeof(on));
            for (int k = 0; k < cfg->nsel; k++) on[ids[k]] = 1;
            for (int e = 0; e < cfg->n_experts; e++) {
                if (on[e]) { if (logits[e] < kth) kth = logits[e]; }
                else if (logits[e] > next) next = logits[e];
            }
            mg = kth - next;
        } else {
            ckr_route_sigmoid_group(logits, bias, cfg->n_experts, cfg->ngroups, cfg->topk_groups,
                                    cfg->nsel, cfg->wscale, ids, wts, &mg);
        }
        if (c->margin) c->margin[i] = mg;
        if (!c->out) continue;
        double *acc = c->out + i * H;
        for (int64_t r = 0; r < H; r++) acc[r] = 0.0;
        if (cfg->mode == 3) {
            /* moe-mix (moe-gate.fk:32-37): ascending expert index, a zero gate skips, acc + g*y */
            for (int e = 0; e < cfg->n_experts; e++) {
                double g = 0.0;
                for (int k = 0; k < cfg->nsel; k++) if (ids[k] == e) g = wts[k];
                if (g == 0.0) continue;
                expert_out(c->w_gate + e * eb_gu, c->w_up + e * eb_gu, c->w_down + e * eb_d, H, I, x,
                           1.0, y, wrow, mid);
                for (int64_t r = 0; r < H; r++) acc[r] = acc[r] + g * y[r];
            }
        } else {
            /* dsv4-moe-acc (dsv4-forward.fk:100-103): selection-list order, acc + E(x; w) */
            for (int k = 0; k < cfg->nsel; k++) {
                int e = ids[k];
                expert_out(c->w_gate + e * eb_gu, c->w_up + e * eb_gu, c->w_down + e * eb_d, H, I, x,
                           wts[k], y, wrow, mid);
                for (int64_t r = 0; r < H; r++) acc[r] = acc[r] + y[r];
            }
        }
        /* shared experts, weight 1.0, added after the routed sum (dsv4-ffn-half, dsv4-forward.fk:155) */
        for (int s = 0; s < cfg->n_shared; s++) {
            expert_out(c->s_gate + s * eb_gu, c->s_up + s * eb_gu, c->s_down + s * eb_d, H, I, x, 1.0,
                       y, wrow, mid);
            for (int64_t r = 0; r < H; r++) acc[r] = acc[r] + y[r];
        }
    }
    free(x); free(wrow); free(mid); free(y);
}

int ckr_moe_layer(const ckr_moe_cfg *cfg, const uint8_t *w_gate, const uint8_t *w_up,
                  const uint8_t *w_down, const uint8_t *s_gate, const uint8_t *s_up,
                  const uint8_t *s_down, const float *router_w, const float *bias,
                  const uint16_t *x_bf16, const int64_t *tok, int64_t ntok, int32_t *ids,
                  double *wts, double *out, int nthreads) {
    if (cfg->n_experts < 1 || cfg->n_experts > 1024 || cfg->nsel < 1 || cfg->nsel > cfg->n_experts) return -1;
    if (cfg->mode != 3 && cfg->mode != 4) return -1;
    if (cfg->mode == 4 && (cfg->ngroups < 1 || cfg->ngroups > 64 || cfg->n_experts % cfg->ngroups)) return -1;
    if ((cfg->hidden * cfg->inter) % 256) return -1;
    moe_ctx c = {cfg, w_gate, w_up, w_down, s_gate, s_up, s_down, router_w, bias, x_bf16, tok,
                 ids, wts, out, NULL};
    ckr_parallel(moe_job, &c, ntok, nthreads);
    return 0;
}

int ckr_moe_route(const ckr_moe_cfg *cfg, const float *router_w, const float *bias,
                  const uint16_t *x_bf16, int64_t ntok, int32_t *ids, double *wts,
                  double *margin, int nthreads) {
    if (cfg->n_experts < 1 || cfg->n_experts > 1024 || cfg->nsel < 1 || cfg->nsel > cfg->n_experts) return -1;
    if (cfg->mode != 3 && cfg->mode != 4) return -1;
    if (cfg->mode == 4 && (cfg->ngroups < 1 || cfg->ngroups > 64 || cfg->n_experts % cfg->ngroups)) return -1;
    moe_ctx c = {cfg, NULL, NULL, NULL, NULL, NULL, NULL, router_w, bias, x_bf16, NULL,
                 ids, wts, NULL, margin};
    ckr_parallel(moe_job, &c, ntok, nthreads);
    return 0;
}
