/* cpu_ref.h -- the oracle: a plain-C, fp64 restatement of coherence-kernel's Form recipes for the
 * quantized dequant / matvec / MoE path.  TEST INFRASTRUCTURE ONLY: the tests, the smoke check and
 * the CPU-baseline leg of bench.py call it as the checker; the product path never links it.
 *
 * Every function follows one Form recipe of the reference, in the same operation order, so that its
 * fp64 result is bit-identical to what the reference's own runtime (fkwu) prints for the same inputs.
 * The citation beside each declaration is the recipe it restates (paths inside the reference tree).
 */
#ifndef CK_ORACLE_CPU_REF_H
#define CK_ORACLE_CPU_REF_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* form/form-stdlib/f16-decode.fk:28-57 (fd-value at eb=5, mb=10), and eb=8 mb=7 for bf16 */
double ckr_f16(uint32_t bits);
double ckr_bf16(uint32_t bits);

/* form/form-stdlib/q8-0-msl.fk:53-72 (q80-flat-at): weight at a flat index, 34-byte blocks */
double ckr_q80_at(const uint8_t *src, int64_t base, int64_t idx);
/* llama-numerics.fk:40-50 ln-rmsnorm over n values with gain g */
void ckr_rmsnorm(const double *x, const double *g, int64_t n, double eps, double *out);
/* form/form-stdlib/q6k-msl.fk:62-81 (q6m-flat-at): weight at a flat index, 210-byte superblocks;
 * ckr_q6k_codes: the 6-bit code q + 32 (bits 0..7) and the raw scale byte (bits 8..15);
 * ckr_q6k_dequant: the flat range [off, off+n); ckr_q6k_matvec: the right fold per row. */
double ckr_q6k_at(const uint8_t *src, int64_t base, int64_t idx);
uint32_t ckr_q6k_codes(const uint8_t *src, int64_t base, int64_t idx);
void ckr_q6k_dequant(const uint8_t *qb, int64_t off, int64_t n, double *w);
void ckr_q6k_matvec(const uint8_t *qb, const double *x, double *y, int64_t rows, int64_t cols);
/* form/form-stdlib/q4k-msl.fk:55-86 (q4m-flat-at): weight at a flat index, 144-byte superblocks */
double ckr_q4k_at(const uint8_t *src, int64_t base, int64_t idx);
/* The decoded integer fields of a Q4_K weight (q4k-dequant.fk:19-43): 6-bit scale, 6-bit min and
 * 4-bit code, packed as scale | min<<8 | code<<16. */
uint32_t ckr_q4k_codes(const uint8_t *src, int64_t base, int64_t idx);

void ckr_q80_dequant(const uint8_t *qb, int64_t off, int64_t n, double *w);
void ckr_q4k_dequant(const uint8_t *qb, int64_t off, int64_t n, double *w);

/* form/form-stdlib/transformer-block.fk:25-26 (tb-dot): x0*w0 + (x1*w1 + (... + (xn*wn + 0.0))) */
double ckr_dot(const double *a, const double *b, int64_t n);

/* tb-matvec (transformer-block.fk:27-28) over dequantized rows: row r is the flat range
 * [r*cols, (r+1)*cols) of the tensor, so rows may straddle blocks (q4k-msl.fk:73-86). */
void ckr_q80_matvec(const uint8_t *qb, const double *x, double *y, int64_t rows, int64_t cols);
void ckr_q4k_matvec(const uint8_t *qb, const double *x, double *y, int64_t rows, int64_t cols);
/* one tb-matvec per token: x[t*cols + j], y[t*rows + r] (qk-matmul-batch.fk:117-121).
 * rows [r0, r1) only, so a large matrix can be sampled; nthreads splits the tokens. */
void ckr_q4k_matmul(const uint8_t *qb, const double *x, double *y, int64_t rows, int64_t cols,
                    int64_t ntok, int64_t r0, int64_t r1, int nthreads);

/* scalar numerics */
double ckr_exp(double x);     /* transformer-numerics.fk:16-24 tn-exp */
double ckr_sqrt(double v);    /* transformer-numerics.fk:32-34 tn-sqrt */
double ckr_ln(double x);      /* trig.fk:40-54 fln */
double ckr_sigmoid(double x); /* llama-numerics.fk:29 ln-sigmoid */
double ckr_silu(double x);    /* llama-numerics.fk:30 ln-silu */

/* Softmax router (moe-msl.fk:73-106): mm-softmax, mm-topk (best first; strict '>' keeps the lower
 * index), mm-gather; renorm=1 adds mm-route-weights' renormalization.  probs (ne) is optional. */
void ckr_route_softmax(const double *logits, int ne, int nsel, int renorm, int32_t *ids,
                       double *wts, double *probs);
/* DeepSeek-style router (dsv4-forward.fk:65-112, dsv4-router-msl.fk dr-weights): probs =
 * sqrt(softplus(logit)); selection on probs+bias by dsv4-topk (ids come out LAST-selected first);
 * weights from the unbiased probs, sum floored at 2^-14, times wscale. */
void ckr_route_dsv4(const double *logits, const double *bias, int ne, int nused, double wscale,
                    int32_t *ids, double *wts);
/* Sigmoid, group-limited router, composed from the same primitives: probs = ln-sigmoid(logit);
 * score = probs + bias; group score = tn-sum of the group's dsv4-topk-2 scores; dsv4-topk over the
 * group scores picks topk_groups groups; experts outside them are set to -1e9 (dsv4-set-nth's
 * sentinel) and dsv4-topk picks nused experts; weights as in ckr_route_dsv4 (floor, wscale).
 * margin (optional) receives the smallest gap between a chosen and a rejected candidate at either
 * decision (groups, then experts) -- the quantity a fast path must exceed to be trusted. */
void ckr_route_sigmoid_group(const double *logits, const double *bias, int ne, int ngroups,
                             int topk_groups, int nused, double wscale, int32_t *ids, double *wts,
                             double *margin);

/* One MoE layer over a list of tokens.
 *   mode 3: softmax router, top-nsel, no renormalization; experts combined moe-mix style
 *           (moe-gate.fk:22-36: ascending expert index, acc + g*E(x)); then each shared expert
 *           (weight 1.0) added in index order.
 *   mode 4: sigmoid group-limited router (ckr_route_sigmoid_group); experts combined dsv4 style
 *           (dsv4-forward.fk:92-112: mid = silu(g)*u*w, acc + E(x) in selection order); then the
 *           shared expert(s) added (dsv4-ffn-half's tb-vec-add moe shared).
 * Weights: gate/up are [inter x hidden] Q4_K, down is [hidden x inter] Q4_K, expert e's tensor at
 * byte offset e*bytes of each array; shared experts likewise in their own arrays.
 * router_w is fp32 [ne x hidden]; bias fp32 [ne] (mode 4); x is bf16 bits [*, hidden].
 * For each token tok[i]: ids[i*nsel..], wts[i*nsel..] and out[i*hidden..] (fp64). */
typedef struct {
    int64_t hidden, inter;
    int32_t n_experts, n_shared, nsel, mode;
    int32_t ngroups, topk_groups;
    double wscale;
} ckr_moe_cfg;

int ckr_moe_layer(const ckr_moe_cfg *cfg, const uint8_t *w_gate, const uint8_t *w_up,
                  const uint8_t *w_down, const uint8_t *s_gate, const uint8_t *s_up,
                  const uint8_t *s_down, const float *router_w, const float *bias,
                  const uint16_t *x_bf16, const int64_t *tok, int64_t ntok, int32_t *ids,
                  double *wts, double *out, int nthreads);

/* Router only (all tokens): the ids and weights ckr_moe_layer would choose, and each token's
 * decision margin (mode 4) or the logit gap at the k/k+1 boundary (mode 3). */
int ckr_moe_route(const ckr_moe_cfg *cfg, const float *router_w, const float *bias,
                  const uint16_t *x_bf16, int64_t ntok, int32_t *ids, double *wts,
                  double *margin, int nthreads);

#ifdef __cplusplus
}
#endif
#endif
