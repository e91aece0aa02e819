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
// The logits: k_exact_logits spreads (token, expert) right folds over the whole GPU -- tiled over
// 16 tokens x 64 experts when more than 128 tokens are flagged, one chain per lane fed by a cp.async
// ring (k_exact_logits_few) when at most 128 are; k_exact_select is one CTA per token.
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

// out[f * ne + e] = right fold of router row e with flagged token f's activations, fp64.
// The product of an fp32 weight and a bf16 activation has at most 32 significant bits, so it is
// exact in fp64 and fma(w, x, acc) rounds once exactly as acc + (w * x) does: one DFMA per term,
// j descending.  A fold is a dependent chain of `hidden` DFMAs (about 9 cycles a step), so many
// chains must run at once and their operands must be in registers when the chain reaches them.
// This GPU converts fp32 to fp64 at a quarter of its DFMA rate, so an operand shared by several
// chains is converted once.
//
// Many flagged tokens (k_exact_logits): the router is first converted to fp64 (k_router_f64,
// skipped otherwise).  A work item is 16 tokens x 64 experts on a CTA of four warps; warp q folds
// tokens 4q .. 4q+3 and lane l experts l and l + 32, eight chains per thread (16 x 32 and four
// chains when the 64-expert items would leave more than half the CTAs without one).  Tiles of 32 columns
// (the last tile first) arrive by cp.async in a ring of XT_NS stages; the router rows are read from
// the ring with 16-byte loads at a 34-double pitch (conflict-free per quarter warp), the tile's
// activations are converted into one of two fp64 buffers a tile ahead.  One CTA barrier per tile.
// Few flagged tokens (a decode step, or a rank's share of a batch; k_exact_logits_few): a work
// item is 4 tokens x 32 experts on a CTA of four warps, warp q folding token q, lane l expert l --
// enough warps to fill the GPU, each folding one chain.  Stages of 32 columns go through a CTA-wide
// cp.async ring of XF_NB stages: the 32 experts' fp32 row pieces (eight threads to a piece, so each
// copy instruction moves whole lines; a thread per row would keep 32 scattered sectors in flight
// per instruction and run into the SM's limit on outstanding requests) and the four tokens'
// activations, converted to fp64 once, two stages ahead.  The router is shared by the item's four
// tokens through the ring (one read of it from L2 per four tokens), and each lane converts its 32
// router values of the next stage while it folds the current one (converting them once per CTA
// into shared memory instead measured slower).  It is launched without programmatic dependent
// launch: launched early, beside the kernels before it, its CTAs were placed so that up to 51
// flagged tokens took twice the time that 65 did.
constexpr int XL_J = 32;          // columns per tile
constexpr int XT_TOK = 16;        // flagged tokens per work item
constexpr int XT_EXP = 64;        // experts per work item
constexpr int XT_NS = 6;          // cp.async ring stages
constexpr int XT_THREADS = 128;
constexpr int XT_WP = XL_J + 2;   // router row pitch in the ring, in doubles
struct XtSmem {
    double w[XT_NS][XT_EXP][XT_WP];     // router rows of the tile (fp64)
    uint16_t x[XT_NS][XT_TOK][XL_J];    // activations of the tile, as copied
    double xd[2][XT_TOK][XL_J];         // converted
};
constexpr uint32_t XL_FEW = 128;  // at most this many flagged tokens take the few-token form
constexpr int XF_C = 32;          // columns per stage
constexpr int XF_NB = 8;          // ring stages
constexpr int XF_W = 4;           // warps per CTA = tokens per work item
struct XfRing {
    float4 w[XF_NB][32][XF_C / 4 + 1];  // [stage][expert][column quad], one pad quad: conflict-free per quarter warp
    uint4 x[XF_NB][XF_W][XF_C / 8];     // [stage][token][8 columns]
    double xd[XF_NB][XF_W][XF_C];       // [stage][token][column]
};
CK_DEV void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
CK_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
CK_DEV void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// The router in fp64 (n4 groups of four values), for the tiled form.
__global__ void __launch_bounds__(256) k_router_f64(const float4 *__restrict__ w, double2 *__restrict__ wd, size_t n4,
                                                    const uint32_t *__restrict__ flag_count) {
    grid_dep_trigger_small();
    grid_dep_wait();
    if (*flag_count <= XL_FEW) return;  // only the tiled form reads it
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
        const float4 v = __ldg(w + i);
        wd[2 * i] = make_double2(v.x, v.y);
        wd[2 * i + 1] = make_double2(v.z, v.w);
    }
}

__global__ void __launch_bounds__(XF_W * 32) k_exact_logits_few(const uint16_t *__restrict__ x,
                                                                const float *__restrict__ W,
                                                                const uint32_t *__restrict__ flag_list,
                                                                const uint32_t *__restrict__ flag_count,
                                                                double *__restrict__ out, uint32_t ne, uint32_t hidden) {
    extern __shared__ __align__(16) uint8_t xf_smem[];
    XfRing &r = *reinterpret_cast<XfRing *>(xf_smem);
    const uint32_t nflag = *flag_count;
    if (nflag == 0 || nflag > XL_FEW) return;  // nothing flagged, or the tiled kernel takes them
    const int tid = threadIdx.x, lane = tid & 31, wq = tid >> 5;
    const uint32_t ntg = (nflag + XF_W - 1) / XF_W, neg = (ne + 31) / 32;
    const int nst = (int)hidden / XF_C;
    for (uint32_t item = blockIdx.x; item < ntg * neg; item += gridDim.x) {
        const uint32_t f0 = (item / neg) * XF_W, e = (item % neg) * 32 + lane, f = f0 + wq;
        const bool live = e < ne && f < nflag;
        // a stage's router piece is 32 rows of XF_C / 4 16-byte chunks: thread i copies chunk
        // (i + 128 k) % CPR of row (i + 128 k) / CPR (rows past ne repeat the last row); threads below
        // XF_W * XPR copy chunk i % XPR of token i / XPR's activations (tokens past nflag repeat the
        // last one)
        constexpr int CPR = XF_C / 4, CPT = 32 * CPR / (XF_W * 32), XPR = XF_C / 8;
        const float *wr[CPT];
#pragma unroll
        for (int k = 0; k < CPT; ++k) {
            const uint32_t i = (uint32_t)(tid + XF_W * 32 * k);
            wr[k] = W + (size_t)min((item % neg) * 32 + i / CPR, ne - 1) * hidden + 4 * (i % CPR);
        }
        const uint16_t *xr = x + (size_t)flag_list[min(f0 + (uint32_t)(tid / XPR % XF_W), nflag - 1)] * hidden +
                             8 * (tid % XPR);
        // stage s holds columns XF_C (nst-1-s) .. + XF_C - 1 (the fold runs from the last column down)
        auto issue = [&](int s) {
            if (s < nst) {
                const int j = XF_C * (nst - 1 - s), b = s % XF_NB;
#pragma unroll
                for (int k = 0; k < CPT; ++k) {
                    const int i = tid + XF_W * 32 * k;
                    cp_async16(&r.w[b][i / CPR][i % CPR], wr[k] + j);
                }
                if (tid < XF_W * XPR) cp_async16(&r.x[b][tid / XPR][tid % XPR], xr + j);
            }
            cp_async_commit();  // an empty group past the end keeps the wait count uniform
        };
        auto convert_x = [&](int s) {  // the stage's XF_C * XF_W activations, one per thread
            if (s < nst && tid < XF_C * XF_W) {
                const int b = s % XF_NB, t = tid / XF_C, c = tid % XF_C;
                const uint16_t h = reinterpret_cast<const uint16_t *>(&r.x[b][t][0])[c];
                r.xd[b][t][c] = (double)bf16_bits_to_float(h);
            }
        };
        auto load_w = [&](int s, double (&wv)[XF_C]) {  // the lane's XF_C router values, in fp64
            const int b = s % XF_NB;
#pragma unroll
            for (int c = 0; c < XF_C / 4; ++c) {
                const float4 v = r.w[b][lane][c];
                wv[4 * c] = v.x;
                wv[4 * c + 1] = v.y;
                wv[4 * c + 2] = v.z;
                wv[4 * c + 3] = v.w;
            }
        };
        double acc = 0.0;
        // one stage: refill, wait, convert two stages ahead, load the next stage's router values,
        // then fold this stage (column 15 first)
        auto step = [&](int s, const double (&wc)[XF_C], double (&wn)[XF_C]) {
            issue(s + XF_NB - 1);        // into the slot of stage s - 1, read in an earlier step
            cp_async_wait<XF_NB - 3>();  // stages up to s + 2 have landed
            __syncthreads();             // every thread's copies and conversions are visible
            convert_x(s + 2);
            if (s + 1 < nst) load_w(s + 1, wn);
            const double2 *xv = reinterpret_cast<const double2 *>(r.xd[s % XF_NB][wq]);
#pragma unroll
            for (int c = XF_C / 2 - 1; c >= 0; --c) {
                const double2 xx = xv[c];
                acc = __fma_rn(wc[2 * c + 1], xx.y, acc);
                acc = __fma_rn(wc[2 * c], xx.x, acc);
            }
        };
        __syncthreads();  // the previous item's reads of the ring are done
        for (int s = 0; s < XF_NB - 1; ++s) issue(s);
        cp_async_wait<XF_NB - 3>();  // stages 0 and 1 have landed
        __syncthreads();
        convert_x(0);
        convert_x(1);
        double wa[XF_C], wb[XF_C];
        load_w(0, wa);
        int s = 0;
        for (; s + 1 < nst; s += 2) {
            step(s, wa, wb);
            step(s + 1, wb, wa);
        }
        if (s < nst) step(s, wa, wb);
        cp_async_wait<0>();
        if (live) out[(size_t)f * ne + e] = acc;
    }
}

// One work item set of the tiled form: NE2 experts per lane (XT_TOK tokens x 32 NE2 experts per
// item).  NE2 = 2 shares each activation load between two experts; NE2 = 1 halves the items' size,
// for batches whose items would leave most SMs idle.
template <int NE2>
CK_DEV void exact_tiled(const uint16_t *__restrict__ x, const double *__restrict__ W,
                        const uint32_t *__restrict__ flag_list, uint32_t nflag, double *__restrict__ out, uint32_t ne,
                        uint32_t hidden, XtSmem &S) {
    constexpr int EXP = 32 * NE2, RPT = EXP / 8;  // experts per item; router rows each thread copies from
    const int tid = threadIdx.x, lane = tid & 31, q = tid >> 5;
    const uint32_t ntg = (nflag + XT_TOK - 1) / XT_TOK, neg = (ne + EXP - 1) / EXP;
    const int ntile = (int)(hidden / XL_J);
    for (uint32_t item = blockIdx.x; item < ntg * neg; item += gridDim.x) {
        const uint32_t f0 = (item / neg) * XT_TOK, e0 = (item % neg) * EXP;
        // this thread's 16-byte pieces of a tile: RPT of router rows (16 per row; rows past ne
        // repeat the last row: read, never written) and, for threads 0-63, a quarter of a token row
        const double *wsrc[RPT];
#pragma unroll
        for (int k = 0; k < RPT; ++k) {
            const uint32_t e = min(e0 + (uint32_t)(tid / 16 + 8 * k), ne - 1);
            wsrc[k] = W + (size_t)e * hidden + 2 * (tid % 16);
        }
        const uint32_t fx = min(f0 + (uint32_t)(tid / 4 % XT_TOK), nflag - 1);
        const uint16_t *xsrc = x + (size_t)flag_list[fx] * hidden + 8 * (tid % 4);
        auto issue = [&](int tile) {  // tile t covers columns hidden - 32 (t + 1) .. hidden - 32 t - 1
            if (tile < ntile) {
                const int slot = tile % XT_NS, j0 = (int)hidden - XL_J * (tile + 1);
#pragma unroll
                for (int k = 0; k < RPT; ++k) cp_async16(&S.w[slot][tid / 16 + 8 * k][2 * (tid % 16)], wsrc[k] + j0);
                if (tid < 4 * XT_TOK) cp_async16(&S.x[slot][tid / 4][8 * (tid % 4)], xsrc + j0);
            }
            cp_async_commit();
        };
        auto convert = [&](int tile) {  // the tile's activations into fp64 buffer tile & 1
            if (tile < ntile) {
                const int slot = tile % XT_NS, b = tile & 1;
#pragma unroll
                for (int k = 0; k < XT_TOK * XL_J / XT_THREADS; ++k) {
                    const int i = tid + XT_THREADS * k;
                    S.xd[b][i / XL_J][i % XL_J] = (double)bf16_bits_to_float(S.x[slot][i / XL_J][i % XL_J]);
                }
            }
        };
        __syncthreads();  // the previous item's reads of the ring and buffers are done
        for (int t = 0; t < XT_NS - 1; ++t) issue(t);
        cp_async_wait<XT_NS - 2>();  // tile 0 has landed
        __syncthreads();
        convert(0);
        double a[4][NE2];
#pragma unroll
        for (int t = 0; t < 4; ++t)
#pragma unroll
            for (int c = 0; c < NE2; ++c) a[t][c] = 0.0;
        for (int tile = 0; tile < ntile; ++tile) {
            cp_async_wait<XT_NS - 3>();  // tiles up to tile + 1 have landed
            __syncthreads();             // ... for every thread; tile - 1 is folded, buffer tile & 1 converted
            issue(tile + XT_NS - 1);     // into the slot of tile - 1
            convert(tile + 1);
            const int slot = tile % XT_NS, b = tile & 1;
            // columns jj + 1, then jj: descending j; the next pair's operands load while this one folds
            double2 w[NE2], xx[4];
#pragma unroll
            for (int c = 0; c < NE2; ++c) w[c] = *reinterpret_cast<const double2 *>(&S.w[slot][lane + 32 * c][XL_J - 2]);
#pragma unroll
            for (int t = 0; t < 4; ++t) xx[t] = *reinterpret_cast<const double2 *>(&S.xd[b][4 * q + t][XL_J - 2]);
#pragma unroll
            for (int jj = XL_J - 2; jj >= 0; jj -= 2) {
                double2 w2[NE2], xx2[4];
#pragma unroll
                for (int c = 0; c < NE2; ++c) w2[c] = w[c];
#pragma unroll
                for (int t = 0; t < 4; ++t) xx2[t] = xx[t];
                if (jj >= 2) {
#pragma unroll
                    for (int c = 0; c < NE2; ++c)
                        w2[c] = *reinterpret_cast<const double2 *>(&S.w[slot][lane + 32 * c][jj - 2]);
#pragma unroll
                    for (int t = 0; t < 4; ++t) xx2[t] = *reinterpret_cast<const double2 *>(&S.xd[b][4 * q + t][jj - 2]);
                }
#pragma unroll
                for (int t = 0; t < 4; ++t) {
#pragma unroll
                    for (int c = 0; c < NE2; ++c) a[t][c] = __fma_rn(w[c].y, xx[t].y, a[t][c]);
#pragma unroll
                    for (int c = 0; c < NE2; ++c) a[t][c] = __fma_rn(w[c].x, xx[t].x, a[t][c]);
                }
#pragma unroll
                for (int c = 0; c < NE2; ++c) w[c] = w2[c];
#pragma unroll
                for (int t = 0; t < 4; ++t) xx[t] = xx2[t];
            }
        }
        cp_async_wait<0>();
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const uint32_t f = f0 + 4 * q + t;
            if (f >= nflag) continue;
#pragma unroll
            for (int c = 0; c < NE2; ++c) {
                const uint32_t e = e0 + lane + 32 * c;
                if (e < ne) out[(size_t)f * ne + e] = a[t][c];
            }
        }
    }
}

__global__ void __launch_bounds__(XT_THREADS, 1) k_exact_logits(const uint16_t *__restrict__ x, const double *__restrict__ W,
                                                             const uint32_t *__restrict__ flag_list,
                                                             const uint32_t *__restrict__ flag_count,
                                                             double *__restrict__ out, uint32_t ne, uint32_t hidden) {
    grid_dep_trigger_small();
    grid_dep_wait();
    extern __shared__ __align__(16) uint8_t xt_smem[];
    XtSmem &S = *reinterpret_cast<XtSmem *>(xt_smem);
    const uint32_t nflag = *flag_count;
    if (nflag <= XL_FEW) return;  // k_exact_logits_few takes them
    // 64-expert items while they fill more than half the CTAs, else 32-expert items (twice as many)
    const uint32_t items64 = (nflag + XT_TOK - 1) / XT_TOK * ((ne + 63) / 64);
    if (2 * items64 <= gridDim.x)
        exact_tiled<1>(x, W, flag_list, nflag, out, ne, hidden, S);
    else
        exact_tiled<2>(x, W, flag_list, nflag, out, ne, hidden, S);
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

// The reference's right-fold logits of the listed tokens: out[f * ne + e] for f < *count <= max_count;
// w64 is scratch for the router in fp64 (ne * hidden doubles).
int launch_exact_logits(const uint16_t *x, const float *w, const uint32_t *flag_list, const uint32_t *flag_count,
                        double *out, double *w64, uint32_t ne, uint32_t hidden, uint32_t max_count, cudaStream_t s) {
    if (ne == 0 || ne > 256 || hidden == 0 || hidden % XL_J != 0 || (reinterpret_cast<uintptr_t>(x) & 15) ||
        (reinterpret_cast<uintptr_t>(w) & 15) || (reinterpret_cast<uintptr_t>(w64) & 15))
        return CK_ERR_SHAPE;
    int dev = 0, nsm = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    static unsigned long long attrs = 0;
    if (attr_pending(attrs)) {
        cudaError_t e = cudaFuncSetAttribute(k_exact_logits_few, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)sizeof(XfRing));
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(k_exact_logits, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)sizeof(XtSmem));
        if (e != cudaSuccess) return (int)e;
        attr_mark(attrs);
    }
    // both forms are launched (the tiled one, with the router's fp64 copy, only where the count can
    // exceed XL_FEW); each returns at once unless the flagged count is its own.  The tiled form runs
    // one CTA per SM (shared-memory bandwidth is its bound) over its work items.
    const bool tiled = max_count > XL_FEW;
    cudaError_t e = tiled ? launch_pdl(k_router_f64, dim3(nsm), dim3(256), 0, s, reinterpret_cast<const float4 *>(w),
                                       reinterpret_cast<double2 *>(w64), (size_t)ne * hidden / 4, flag_count)
                          : cudaSuccess;
    if (e == cudaSuccess) {
        k_exact_logits_few<<<2 * nsm, XF_W * 32, sizeof(XfRing), s>>>(x, w, flag_list, flag_count, out, ne, hidden);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess && tiled)
        e = launch_pdl(k_exact_logits, dim3(nsm), dim3(XT_THREADS), sizeof(XtSmem), s, x, (const double *)w64,
                       flag_list, flag_count, out, ne, hidden);
    return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

int launch_route_exact(const uint16_t *x, const float *w, const float *bias, int32_t *ids, float *wts,
                       const uint32_t *flag_list, const uint32_t *flag_count, double *scratch, double *w64,
                       const RouteParams &p, cudaStream_t s) {
    if (p.nsel > 16 || (p.mode == 4 && p.ngroups > 32)) return CK_ERR_SHAPE;
    int rc = launch_exact_logits(x, w, flag_list, flag_count, scratch, w64, p.ne, p.hidden, p.ntok, s);
    if (rc) return rc;
    int dev = 0, nsm = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    const cudaError_t e = launch_pdl(k_exact_select, dim3(nsm * 2), dim3(256), 0, s, scratch, bias, ids, wts, flag_list,
                                     flag_count, p);
    return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

}  // namespace ck
