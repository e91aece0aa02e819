// route_exact.cu -- the exact fp64 re-route of near-tie tokens.
//
// A token whose fast-path decision margin is below tau (a chosen/rejected gap at the group or the
// expert step, or the gap between two chosen experts whose list order it decides) is routed again
// here with the reference's own numerics, so its expert ids and their list order are the
// reference's bit for bit:
//   logits  tb-dot's right fold (transformer-block.fk:25-26): acc = w*x + acc over j descending,
//           each product exact in fp64 (fp32 w times bf16 x), each add rounded once
//   mode 4  ln-sigmoid over tn-exp (llama-numerics.fk:29, transformer-numerics.fk:16-24), score =
//           prob + bias, group score = tn-sum of dsv4-topk-2, dsv4-topk over groups and then over
//           the masked scores (dsv4-forward.fk:72-81), weights = probs * (wscale / max(sum, 2^-14))
//   mode 3  mm-softmax (max, tn-exp, left-fold sum, * 1/sum) and mm-topk (moe-msl.fk:73-99)
// Explicit round-to-nearest intrinsics keep the compiler from contracting a multiply and an add.
//
// Two kernels: k_exact_logits spreads (token, expert) right folds over the whole GPU (each fold is a
// 7168-long dependent chain, so many chains must be in flight) -- tiled over 16 tokens x 64 experts
// when more than 128 tokens are flagged, one chain per lane fed by a cp.async ring
// (k_exact_logits_few) when at most 128 are; k_exact_select is one CTA per token.
#include "ck_common.cuh"
#include "ck_launch.h"

namespace ck {

CK_DEV double ref_exp(double x) {
    int k = 0;
    for (;;) {
        const double ax = x < 0.0 ? 0.0 - x : x;
        if (ax <= 0.5) break;
        x = __ddiv_rn(x, 2.0);
        ++k;
    }
    double n = 1.0, term = 1.0, acc = 1.0;
    while (!(n > 14.0)) {
        const double tt = __dmul_rn(term, __ddiv_rn(x, n));
        acc = __dadd_rn(acc, tt);
        term = tt;
        n = __dadd_rn(n, 1.0);
    }
    for (int i = 0; i < k; ++i) acc = __dmul_rn(acc, acc);
    return acc;
}
CK_DEV double ref_sigmoid(double x) { return __ddiv_rn(1.0, __dadd_rn(1.0, ref_exp(__dsub_rn(0.0, x)))); }

constexpr int XL_TOK = 16;   // flagged tokens per work item
constexpr int XL_EXP = 64;   // experts per work item
constexpr int XL_J = 32;     // columns per shared-memory tile
constexpr int XL_TPT = 4;    // tokens (independent fold chains) per thread

// out[f * ne + e] = right fold of router row e with flagged token f's activations, fp64.
// The product of an fp32 weight and a bf16 activation has at most 32 significant bits, so it is
// exact in fp64 and fma(w, x, acc) rounds once exactly as acc + (w * x) does: one DFMA per term.
// 256 threads = 64 experts x 4 token groups; each thread folds 4 tokens.  The W and x tiles are
// converted to double once per tile into shared memory, double-buffered: the next tile's global
// loads are in registers while the current tile is folded.
// Few flagged tokens (a decode step): the tiled form below would leave most of the GPU idle and fold
// padding, so each warp takes one (token, 32 experts) item and every lane one fold chain.  A chain
// is a dependent sequence of DFMAs, so its inputs must arrive far ahead: each lane copies its
// router row's next columns eight at a time (two 16-byte cp.async) into a per-warp ring of
// XF_NB stages in shared memory, lane 0 copies the token's eight activations beside them, and the
// chain consumes stage i while stages i+1 .. i+XF_NB-1 are in flight.  Same fold, same bits.
constexpr uint32_t XL_FEW = 128;  // 8 items per token: one item per warp at two CTAs per SM
constexpr int XF_NB = 24;       // ring stages per warp (8 columns each)
constexpr int XF_WARPS = 4;     // warps per CTA in the few-token form
struct XfRing {
    float4 w[XF_NB][32][2];     // [stage][lane][columns 8j .. 8j+3, 8j+4 .. 8j+7]
    uint4 x[XF_NB];             // the token's eight bf16 activations of the stage
};
CK_DEV void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
CK_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
CK_DEV void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

CK_DEV void exact_logits_few(const uint16_t *__restrict__ x, const float *__restrict__ W,
                             const uint32_t *__restrict__ flag_list, uint32_t nflag, double *__restrict__ out,
                             uint32_t ne, uint32_t hidden, XfRing &r) {
    const int lane = threadIdx.x & 31;
    const uint32_t neg = (ne + 31) / 32, nwarp = gridDim.x * (blockDim.x >> 5);
    const int nst = (int)hidden / 8;
    for (uint32_t item = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); item < nflag * neg; item += nwarp) {
        const uint32_t f = item / neg, e = (item % neg) * 32 + lane;
        const bool live = e < ne;
        const float *wr = W + (size_t)(live ? e : 0) * hidden;
        const uint16_t *xr = x + (size_t)flag_list[f] * hidden;
        // stage s holds columns 8 (nst-1-s) .. +7 (the fold runs from the last column down)
        auto issue = [&](int s) {
            if (s < nst) {
                const int j = 8 * (nst - 1 - s), b = s % XF_NB;
                cp_async16(&r.w[b][lane][0], wr + j);
                cp_async16(&r.w[b][lane][1], wr + j + 4);
                if (lane == 0) cp_async16(&r.x[b], xr + j);
            }
            cp_async_commit();  // an empty group past the end keeps the wait count uniform
        };
        __syncwarp();  // the previous item's reads of the ring are done
        for (int s = 0; s < XF_NB - 1; ++s) issue(s);
        double acc = 0.0;
        for (int s = 0; s < nst; ++s) {
            issue(s + XF_NB - 1);
            cp_async_wait<XF_NB - 1>();
            __syncwarp();
            const int b = s % XF_NB;
            const float4 lo = r.w[b][lane][0], hi = r.w[b][lane][1];
            const uint4 xv = r.x[b];
            acc = __fma_rn((double)hi.w, (double)__uint_as_float(xv.w & 0xFFFF0000u), acc);
            acc = __fma_rn((double)hi.z, (double)__uint_as_float(xv.w << 16), acc);
            acc = __fma_rn((double)hi.y, (double)__uint_as_float(xv.z & 0xFFFF0000u), acc);
            acc = __fma_rn((double)hi.x, (double)__uint_as_float(xv.z << 16), acc);
            acc = __fma_rn((double)lo.w, (double)__uint_as_float(xv.y & 0xFFFF0000u), acc);
            acc = __fma_rn((double)lo.z, (double)__uint_as_float(xv.y << 16), acc);
            acc = __fma_rn((double)lo.y, (double)__uint_as_float(xv.x & 0xFFFF0000u), acc);
            acc = __fma_rn((double)lo.x, (double)__uint_as_float(xv.x << 16), acc);
            __syncwarp();  // every lane has read stage b before issue() refills it next iteration
        }
        cp_async_wait<0>();
        if (live) out[(size_t)f * ne + e] = acc;
    }
}
__global__ void __launch_bounds__(XF_WARPS * 32) k_exact_logits_few(const uint16_t *__restrict__ x,
                                                                    const float *__restrict__ W,
                                                                    const uint32_t *__restrict__ flag_list,
                                                                    const uint32_t *__restrict__ flag_count,
                                                                    double *__restrict__ out, uint32_t ne,
                                                                    uint32_t hidden) {
    grid_dep_trigger_small();
    grid_dep_wait();
    extern __shared__ __align__(16) uint8_t xf_smem[];
    const uint32_t nflag = *flag_count;
    if (nflag > XL_FEW) return;  // the tiled kernel takes them
    XfRing &r = reinterpret_cast<XfRing *>(xf_smem)[threadIdx.x >> 5];
    exact_logits_few(x, W, flag_list, nflag, out, ne, hidden, r);
}

__global__ void __launch_bounds__(256) k_exact_logits(const uint16_t *__restrict__ x, const float *__restrict__ W,
                                                      const uint32_t *__restrict__ flag_list,
                                                      const uint32_t *__restrict__ flag_count, double *__restrict__ out,
                                                      uint32_t ne, uint32_t hidden) {
    grid_dep_trigger_small();
    grid_dep_wait();
    __shared__ double wt[2][XL_EXP][XL_J + 1];
    __shared__ __align__(16) double xt[2][XL_TOK][XL_J];
    const uint32_t nflag = *flag_count;
    if (nflag <= XL_FEW) return;  // k_exact_logits_few takes them
    const int tid = threadIdx.x;
    const int el = tid & (XL_EXP - 1);
    const int q = tid / XL_EXP;  // 0..3: this thread folds tokens 4q .. 4q+3 of the item
    const uint32_t ntg = (nflag + XL_TOK - 1) / XL_TOK, neg = (ne + XL_EXP - 1) / XL_EXP;
    const int ntile = (int)(hidden / XL_J);
    constexpr int WPT = XL_EXP * XL_J / 256;  // W floats each thread stages per tile (8)
    constexpr int XPT = XL_TOK * XL_J / 256;  // x values each thread stages per tile (2)
    for (uint32_t item = blockIdx.x; item < ntg * neg; item += gridDim.x) {
        const uint32_t f0 = (item / neg) * XL_TOK, e0 = (item % neg) * XL_EXP;
        const float *wrow[WPT];
        const uint16_t *xrow[XPT];
#pragma unroll
        for (int k = 0; k < WPT; ++k) {
            const uint32_t e = e0 + (uint32_t)((tid + 256 * k) / XL_J);
            wrow[k] = e < ne ? W + (size_t)e * hidden : nullptr;
        }
#pragma unroll
        for (int k = 0; k < XPT; ++k) {
            const uint32_t f = min(f0 + (uint32_t)((tid + 256 * k) / XL_J), nflag - 1);
            xrow[k] = x + (size_t)flag_list[f] * hidden;
        }
        const int jc = tid % XL_J;
        float wv[WPT];
        uint16_t xv[XPT];
        auto fetch = [&](int tile) {  // tile t covers columns hidden - 32 (t + 1) .. hidden - 32 t - 1
            const int j0 = (int)hidden - XL_J * (tile + 1);
#pragma unroll
            for (int k = 0; k < WPT; ++k) wv[k] = wrow[k] ? __ldg(wrow[k] + j0 + jc) : 0.0f;
#pragma unroll
            for (int k = 0; k < XPT; ++k) xv[k] = __ldg(xrow[k] + j0 + jc);
        };
        auto stage = [&](int b) {
#pragma unroll
            for (int k = 0; k < WPT; ++k) wt[b][(tid + 256 * k) / XL_J][jc] = (double)wv[k];
#pragma unroll
            for (int k = 0; k < XPT; ++k) xt[b][(tid + 256 * k) / XL_J][jc] = (double)bf16_bits_to_float(xv[k]);
        };
        fetch(0);
        stage(0);
        __syncthreads();
        double a[XL_TPT];
#pragma unroll
        for (int t = 0; t < XL_TPT; ++t) a[t] = 0.0;
        for (int tile = 0; tile < ntile; ++tile) {
            const int b = tile & 1;
            if (tile + 1 < ntile) fetch(tile + 1);
#pragma unroll
            for (int jj = XL_J - 2; jj >= 0; jj -= 2) {  // columns jj + 1, then jj: descending j
                const double w1 = wt[b][el][jj + 1], w0 = wt[b][el][jj];
#pragma unroll
                for (int t = 0; t < XL_TPT; ++t) {
                    const double2 xx = *reinterpret_cast<const double2 *>(&xt[b][XL_TPT * q + t][jj]);
                    a[t] = __fma_rn(w1, xx.y, a[t]);
                    a[t] = __fma_rn(w0, xx.x, a[t]);
                }
            }
            if (tile + 1 < ntile) stage(b ^ 1);
            __syncthreads();
        }
        const uint32_t e = e0 + el;
        if (e < ne) {
#pragma unroll
            for (int t = 0; t < XL_TPT; ++t) {
                const uint32_t f = f0 + XL_TPT * q + t;
                if (f < nflag) out[(size_t)f * ne + e] = a[t];
            }
        }
    }
}

// (value, index) maximum over the warp: the larger value, the lower index on a tie -- the
// first-maximum rule of a left-to-right scan with strict '>'
CK_DEV void warp_argmax_d(double &v, int &i) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const double ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, i, o);
        if (ov > v || (ov == v && oi < i)) { v = ov; i = oi; }
    }
}

constexpr int XS_MAXR = 8;  // up to 256 experts: lane holds e = lane + 32 r
// Warp 0's part of k_exact_select: the selection over the fp64 terms in `sprob`.
CK_DEV void select_token(const double *sprob, const float *__restrict__ bias, int32_t *__restrict__ ids,
                         float *__restrict__ wts, uint32_t t, const RouteParams &p, int lane) {
    const int ne = (int)p.ne, k = (int)p.nsel;
    const double NEG = -1000000000.0;  // dsv4-set-nth's sentinel
    double v[XS_MAXR], pr[XS_MAXR];
    int sel[16];
    double w[16];
    if (p.mode == 4) {
#pragma unroll
        for (int r = 0; r < XS_MAXR; ++r) {
            const int e = lane + 32 * r;
            pr[r] = e < ne ? sprob[e] : 0.0;
            v[r] = e < ne ? __dadd_rn(pr[r], (double)bias[e]) : -3.0e300;
        }
        // group scores: dsv4-topk-2 of the group (first max, then the first max of the rest),
        // tn-sum over (second, best) = (0 + second) + best
        const int gs = ne / (int)p.ngroups;
        double gsc[32];
        for (int g = 0; g < (int)p.ngroups; ++g) {
            double b1 = -3.0e300;
            int i1 = 1 << 30;
#pragma unroll
            for (int r = 0; r < XS_MAXR; ++r) {
                const int e = lane + 32 * r;
                if (e < ne && e / gs == g && (v[r] > b1 || (v[r] == b1 && e < i1))) { b1 = v[r]; i1 = e; }
            }
            warp_argmax_d(b1, i1);
            double b2 = -3.0e300;
            int i2 = 1 << 30;
#pragma unroll
            for (int r = 0; r < XS_MAXR; ++r) {
                const int e = lane + 32 * r;
                if (e < ne && e / gs == g && e != i1 && (v[r] > b2 || (v[r] == b2 && e < i2))) { b2 = v[r]; i2 = e; }
            }
            warp_argmax_d(b2, i2);
            gsc[g] = __dadd_rn(__dadd_rn(0.0, b2), b1);
        }
        unsigned gon = 0;
        for (int r = 0; r < (int)p.topk_groups; ++r) {
            double best = -3.0e300;
            int bi = 0;
            for (int g = 0; g < (int)p.ngroups; ++g)
                if (!(gon >> g & 1) && gsc[g] > best) { best = gsc[g]; bi = g; }
            gon |= 1u << bi;
        }
#pragma unroll
        for (int r = 0; r < XS_MAXR; ++r) {
            const int e = lane + 32 * r;
            if (e < ne && !(gon >> (e / gs) & 1)) v[r] = NEG;
        }
        // dsv4-topk over the masked scores: the picks listed last-first
        for (int r = 0; r < k; ++r) {
            double b = -3.0e300;
            int bi = 1 << 30;
#pragma unroll
            for (int rr = 0; rr < XS_MAXR; ++rr) {
                const int e = lane + 32 * rr;
                if (e < ne && v[rr] > b) { b = v[rr]; bi = e; }
            }
            warp_argmax_d(b, bi);
            sel[k - 1 - r] = bi;
#pragma unroll
            for (int rr = 0; rr < XS_MAXR; ++rr)
                if (lane + 32 * rr == bi) v[rr] = NEG;
        }
        double s0 = 0.0;
        for (int i = 0; i < k; ++i) {
            double pe = 0.0;
#pragma unroll
            for (int rr = 0; rr < XS_MAXR; ++rr)
                if (lane + 32 * rr == sel[i]) pe = pr[rr];
            pe = __shfl_sync(0xffffffffu, pe, sel[i] & 31);
            w[i] = pe;
            s0 = __dadd_rn(s0, pe);
        }
        const double s = s0 < 0.00006103515625 ? 0.00006103515625 : s0;
        const double scl = __ddiv_rn((double)p.wscale, s);
        for (int i = 0; i < k; ++i) w[i] = __dmul_rn(w[i], scl);
    } else {
        // mm-softmax: mm-max over the tail from the head, tn-exp of (l - max) (both above), the sum
        // as a left fold in index order, p = e * (1/sum); mm-topk keeps the first index on a tie
        const double *buf = sprob;
        double s = 0.0;
        for (int e = 0; e < ne; ++e) s = __dadd_rn(s, buf[e]);
        const double inv = __ddiv_rn(1.0, s);
#pragma unroll
        for (int r = 0; r < XS_MAXR; ++r) {
            const int e = lane + 32 * r;
            v[r] = e < ne ? __dmul_rn(buf[e], inv) : -3.0e300;
        }
        for (int r = 0; r < k; ++r) {
            double b = -3.0e300;
            int bi = 1 << 30;
#pragma unroll
            for (int rr = 0; rr < XS_MAXR; ++rr) {
                const int e = lane + 32 * rr;
                if (e < ne && v[rr] > b) { b = v[rr]; bi = e; }
            }
            warp_argmax_d(b, bi);
            sel[r] = bi;
            w[r] = b;
#pragma unroll
            for (int rr = 0; rr < XS_MAXR; ++rr)
                if (lane + 32 * rr == bi) v[rr] = -3.0e300;
        }
    }
    if (lane == 0)
        for (int i = 0; i < k; ++i) {
            ids[(size_t)t * k + i] = sel[i];
            wts[(size_t)t * k + i] = (float)w[i];
        }
}


// One CTA per flagged token: the 256 threads evaluate the expensive fp64 terms (ln-sigmoid, or
// the softmax's tn-exp) one expert each into shared memory, then warp 0 makes the selection.
__global__ void __launch_bounds__(256) k_exact_select(const double *__restrict__ lg, const float *__restrict__ bias,
                                                      int32_t *__restrict__ ids, float *__restrict__ wts,
                                                      const uint32_t *__restrict__ flag_list,
                                                      const uint32_t *__restrict__ flag_count, RouteParams p) {
    grid_dep_trigger_small();
    grid_dep_wait();
    __shared__ double sbuf[256], sprob[256];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const uint32_t nflag = *flag_count;
    const int ne = (int)p.ne;
    for (uint32_t f = blockIdx.x; f < nflag; f += gridDim.x) {
        const uint32_t t = flag_list[f];
        const double *L = lg + (size_t)f * ne;
        const int te = threadIdx.x;
        if (p.mode == 4) {
            if (te < ne) sprob[te] = ref_sigmoid(L[te]);
        } else {
            // mm-max over the tail from the head (every thread scans the same row), then tn-exp
            if (te < ne) sbuf[te] = L[te];
            __syncthreads();
            double mx = sbuf[0];
            for (int e = 1; e < ne; ++e)
                if (sbuf[e] > mx) mx = sbuf[e];
            if (te < ne) sprob[te] = ref_exp(__dsub_rn(sbuf[te], mx));
        }
        __syncthreads();
        if (wib == 0) select_token(sprob, bias, ids, wts, t, p, lane);
        __syncthreads();  // the shared rows are reused by the next token
    }
}

// The middle tier of a large batch's route: fp64 logits of the flagged tokens accurate to a few
// roundings of sum|w x|, without the reference's sequential fold.  The tiles are those of
// k_exact_logits, but every thread keeps eight interleaved partial sums per token (column j feeds
// partial j mod 8) of the exact fp64 products, so a chain is hidden / 8 terms long and a thread has
// 32 independent chains in flight; the eight are summed in a fixed order at the end (deterministic).
// The error against the exact dot is at most (hidden / 8 + 3) * 2^-53 * sum|w x|, and the
// reference's own fold differs from it by at most hidden * 2^-53 * sum|w x|: the fp64 selection that
// follows flags a token for the sequential fold only when its margin is below 16 * 2^-40 of its
// largest sum|w x| -- in practice only exact ties.  sum|w x| (fp32) is written beside each logit.
// Block 0 also clears the count of the list that selection fills.
__global__ void __launch_bounds__(256) k_accurate_logits(const uint16_t *__restrict__ x, const float *__restrict__ W,
                                                         const uint32_t *__restrict__ flag_list,
                                                         const uint32_t *__restrict__ flag_count,
                                                         double *__restrict__ out, float *__restrict__ out_abs,
                                                         uint32_t *__restrict__ next_count, uint32_t ne,
                                                         uint32_t hidden) {
    grid_dep_trigger_small();
    grid_dep_wait();
    if (blockIdx.x == 0 && threadIdx.x == 0) *next_count = 0u;
    __shared__ float wt[2][XL_EXP][XL_J + 1];
    __shared__ __align__(16) float xt[2][XL_TOK][XL_J];
    const uint32_t nflag = *flag_count;
    const int tid = threadIdx.x;
    const int el = tid & (XL_EXP - 1);
    const int q = tid / XL_EXP;
    const uint32_t ntg = (nflag + XL_TOK - 1) / XL_TOK, neg = (ne + XL_EXP - 1) / XL_EXP;
    const int ntile = (int)(hidden / XL_J);
    constexpr int WPT = XL_EXP * XL_J / 256;
    constexpr int XPT = XL_TOK * XL_J / 256;
    constexpr int NP = 8;
    for (uint32_t item = blockIdx.x; item < ntg * neg; item += gridDim.x) {
        const uint32_t f0 = (item / neg) * XL_TOK, e0 = (item % neg) * XL_EXP;
        const float *wrow[WPT];
        const uint16_t *xrow[XPT];
#pragma unroll
        for (int k = 0; k < WPT; ++k) {
            const uint32_t e = e0 + (uint32_t)((tid + 256 * k) / XL_J);
            wrow[k] = e < ne ? W + (size_t)e * hidden : nullptr;
        }
#pragma unroll
        for (int k = 0; k < XPT; ++k) {
            const uint32_t f = min(f0 + (uint32_t)((tid + 256 * k) / XL_J), nflag - 1);
            xrow[k] = x + (size_t)flag_list[f] * hidden;
        }
        const int jc = tid % XL_J;
        float wv[WPT];
        uint16_t xv[XPT];
        auto fetch = [&](int tile) {
            const int j0 = XL_J * tile;
#pragma unroll
            for (int k = 0; k < WPT; ++k) wv[k] = wrow[k] ? __ldg(wrow[k] + j0 + jc) : 0.0f;
#pragma unroll
            for (int k = 0; k < XPT; ++k) xv[k] = __ldg(xrow[k] + j0 + jc);
        };
        auto stage = [&](int b) {
#pragma unroll
            for (int k = 0; k < WPT; ++k) wt[b][(tid + 256 * k) / XL_J][jc] = wv[k];
#pragma unroll
            for (int k = 0; k < XPT; ++k) xt[b][(tid + 256 * k) / XL_J][jc] = bf16_bits_to_float(xv[k]);
        };
        fetch(0);
        stage(0);
        __syncthreads();
        double a[XL_TPT][NP];
        float ab[XL_TPT];
#pragma unroll
        for (int t = 0; t < XL_TPT; ++t) {
            ab[t] = 0.0f;
#pragma unroll
            for (int i = 0; i < NP; ++i) a[t][i] = 0.0;
        }
        for (int tile = 0; tile < ntile; ++tile) {
            const int b = tile & 1;
            if (tile + 1 < ntile) fetch(tile + 1);
#pragma unroll
            for (int j = 0; j < XL_J; ++j) {
                const float w = wt[b][el][j];
                const double wd = (double)w;
#pragma unroll
                for (int t = 0; t < XL_TPT; ++t) {
                    const float xf = xt[b][XL_TPT * q + t][j];
                    a[t][j % NP] = __fma_rn(wd, (double)xf, a[t][j % NP]);  // the product is exact in fp64
                    ab[t] = fmaf(fabsf(w), fabsf(xf), ab[t]);
                }
            }
            if (tile + 1 < ntile) stage(b ^ 1);
            __syncthreads();
        }
        const uint32_t e = e0 + el;
        if (e < ne) {
#pragma unroll
            for (int t = 0; t < XL_TPT; ++t) {
                const uint32_t f = f0 + XL_TPT * q + t;
                if (f < nflag) {
                    const double s = ((a[t][0] + a[t][1]) + (a[t][2] + a[t][3])) +
                                     ((a[t][4] + a[t][5]) + (a[t][6] + a[t][7]));
                    out[(size_t)f * ne + e] = s;
                    out_abs[(size_t)f * ne + e] = ab[t] * 1.0001f;  // covers the fp32 sum's own rounding
                }
            }
        }
    }
}

int launch_accurate_logits(const uint16_t *x, const float *w, const uint32_t *flag_list, const uint32_t *flag_count,
                           double *out, float *out_abs, uint32_t *next_count, uint32_t ne, uint32_t hidden,
                           cudaStream_t s) {
    if (ne > 256 || hidden % XL_J != 0 || (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(w) & 15))
        return CK_ERR_SHAPE;
    int dev = 0, nsm = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    const cudaError_t e = launch_pdl(k_accurate_logits, dim3(nsm * 2), dim3(256), 0, s, x, w, flag_list, flag_count,
                                     out, out_abs, next_count, ne, hidden);
    return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

int launch_route_exact(const uint16_t *x, const float *w, const float *bias, int32_t *ids, float *wts,
                       const uint32_t *flag_list, const uint32_t *flag_count, double *scratch,
                       const RouteParams &p, cudaStream_t s) {
    if (p.ne > 256 || p.hidden % XL_J != 0 || (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(w) & 15) || p.nsel > 16 || (p.mode == 4 && p.ngroups > 32)) return CK_ERR_SHAPE;
    int dev = 0, nsm = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    static unsigned long long few_attr = 0;
    if (attr_pending(few_attr)) {
        const cudaError_t e = cudaFuncSetAttribute(k_exact_logits_few, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   (int)(XF_WARPS * sizeof(XfRing)));
        if (e != cudaSuccess) return (int)e;
        attr_mark(few_attr);
    }
    // both forms are launched; each returns at once unless the flagged count is its own
    cudaError_t e = launch_pdl(k_exact_logits_few, dim3(2 * nsm), dim3(XF_WARPS * 32), XF_WARPS * sizeof(XfRing), s, x,
                               w, flag_list, flag_count, scratch, p.ne, p.hidden);
    if (e == cudaSuccess)
        e = launch_pdl(k_exact_logits, dim3(nsm * 2), dim3(256), 0, s, x, w, flag_list, flag_count, scratch, p.ne,
                       p.hidden);
    if (e == cudaSuccess)
        e = launch_pdl(k_exact_select, dim3(nsm * 2), dim3(256), 0, s, scratch, bias, ids, wts, flag_list, flag_count,
                       p);
    return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

}  // namespace ck
