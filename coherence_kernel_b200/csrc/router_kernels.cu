// router_kernels.cu -- MoE gating: top-k selection, the router split for the tensor cores, and the
// single-token routers the reference's Form cells dispatch.
//
// Selection semantics are the reference's: top-k by repeated argmax where a strict '>' keeps the
// LOWER expert index on a tie (moe-msl.fk:84-98 mm-argmax-free, dsv4-forward.fk:72-81
// dsv4-argmax).  The batched layer routes in three steps:
//   1. logits            x . W_r on the tensor cores (gemm_tc.cu dense form, W_r split into three
//                        bf16 terms by k_split_bf16x3); k_router_logits is the fp32 CUDA-core form
//   2. k_route_select    one warp per token: selection, weights, and the token's decision margin
//                        (the smallest gap between a chosen and a rejected candidate, or between
//                        two chosen ones whose list order it decides)
//   3. route_exact.cu    tokens whose margin is below tau are routed again in fp64 with the
//                        reference's own fold order and numerics, so their expert ids are the
//                        reference's bit for bit.
#include "ck_common.cuh"
#include "ck_launch.h"

namespace ck {

// ------------------------------------------------------------------ warp argmax
// (value, index) maximum with the lower index winning ties.
CK_DEV void warp_argmax(float &v, int &i) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, i, o);
        if (ov > v || (ov == v && oi < i)) { v = ov; i = oi; }
    }
}
CK_DEV float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ------------------------------------------------------------------ 1. logits
// L[t, e] = sum_j x[t, j] * W[e, j]; 64 tokens x 64 experts per block, 4x4 per thread.
__global__ void __launch_bounds__(256) k_router_logits(const uint16_t *__restrict__ x, const float *__restrict__ w,
                                                       float *__restrict__ L, uint32_t T, uint32_t E, uint32_t H) {
    __shared__ float xs[32][64 + 4];
    __shared__ float ws[32][64 + 4];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const uint32_t t0 = blockIdx.x * 64, e0 = blockIdx.y * 64;
    float acc[4][4] = {};
    for (uint32_t k0 = 0; k0 < H; k0 += 32) {
        for (int i = threadIdx.x; i < 64 * 32; i += 256) {
            const int r = i >> 5, k = i & 31;
            const uint32_t t = t0 + r, e = e0 + r, kk = k0 + k;
            xs[k][r] = (t < T && kk < H) ? bf16_bits_to_float(x[(size_t)t * H + kk]) : 0.0f;
            ws[k][r] = (e < E && kk < H) ? w[(size_t)e * H + kk] : 0.0f;
        }
        __syncthreads();
#pragma unroll 8
        for (int k = 0; k < 32; ++k) {
            const float4 xv = *reinterpret_cast<const float4 *>(&xs[k][ty * 4]);
            const float4 wv = *reinterpret_cast<const float4 *>(&ws[k][tx * 4]);
            const float xa[4] = {xv.x, xv.y, xv.z, xv.w}, wa[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int b = 0; b < 4; ++b) acc[a][b] = fmaf(xa[a], wa[b], acc[a][b]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const uint32_t t = t0 + ty * 4 + a, e = e0 + tx * 4 + b;
            if (t < T && e < E) L[(size_t)t * E + e] = acc[a][b];
        }
}

// Few tokens (a decode-sized batch, ntok <= RS_TMAX): the tensor-core form would put the whole
// router on one or two CTAs, so here every expert's row is a CTA of its own and every dot is
// carried as a float pair (s, c): each fp32 x bf16 product is split exactly (p = w*x,
// e = fma(w, x, -p)) and added with Knuth's two-sum, so the pair tracks the sum to about 2^-44 of
// its terms' magnitude -- fp64-like accuracy at fp32 throughput (this GPU's fp64 FMA is a slow
// pipe).  Warp w takes the w-th eighth of the row; its lanes hold their slice of the router row in
// registers for every token, and each token's activations are loaded two tokens ahead of their use
// (the loop is bound by load latency).  The lanes' pairs are merged by two-sums in a fixed shuffle
// tree and the eighths in order; the logit is written in fp64 (for the fp64 selection) and fp32,
// with sum |w x| beside it (the scale of every rounding error in the dot).
constexpr uint32_t RS_TMAX = 128;  // tokens
constexpr uint32_t RS_IT = 8;     // float4 per lane of a warp's eighth of the row: hidden <= 8192
// (explicit round-to-nearest intrinsics: a contracted multiply-add would break the two-sum)
CK_DEV void two_sum_into(float &s, float &c, float p) {
    const float t = __fadd_rn(s, p), z = __fsub_rn(t, s);
    c = __fadd_rn(c, __fadd_rn(__fsub_rn(s, __fsub_rn(t, z)), __fsub_rn(p, z)));
    s = t;
}
CK_DEV void dot_pair(float &s, float &c, float w, float x) {
    const float p = __fmul_rn(w, x);
    c = __fadd_rn(c, __fmaf_rn(w, x, -p));
    two_sum_into(s, c, p);
}
__global__ void __launch_bounds__(256, 2) k_router_logits_few(const uint16_t *__restrict__ x,
                                                              const float *__restrict__ w, float *__restrict__ L,
                                                              double *__restrict__ Ld, float *__restrict__ sabs,
                                                              uint32_t *__restrict__ flag_count, uint32_t T, uint32_t E,
                                                              uint32_t H) {
    grid_dep_trigger_small();
    grid_dep_wait();
    // the selection's flagged-token counter starts at zero (cleared here: a memset would end the
    // chain of dependent launches)
    if (flag_count && blockIdx.x == 0 && threadIdx.x == 0) *flag_count = 0;
    __shared__ double part[8][RS_TMAX];
    __shared__ float apart[8][RS_TMAX];
    const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
    const uint32_t e = blockIdx.x, seg = H / 32, j0 = wp * seg;  // float4 per eighth, this warp's first
    float4 wv[RS_IT];
    const float4 *wr = reinterpret_cast<const float4 *>(w + (size_t)e * H) + j0;
#pragma unroll
    for (uint32_t i = 0; i < RS_IT; ++i) {
        const uint32_t j = lane + 32 * i;
        wv[i] = j < seg ? __ldg(wr + j) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    auto load_x = [&](uint32_t t, uint2 (&xv)[RS_IT]) {
        const uint2 *xr = reinterpret_cast<const uint2 *>(x + (size_t)(t < T ? t : 0) * H) + j0;
#pragma unroll
        for (uint32_t i = 0; i < RS_IT; ++i) {
            const uint32_t j = lane + 32 * i;
            xv[i] = (t < T && j < seg) ? __ldg(xr + j) : make_uint2(0u, 0u);
        }
    };
    uint2 xa[RS_IT], xb[RS_IT], xc[RS_IT];
    load_x(0, xa);
    load_x(1, xb);
    for (uint32_t t = 0; t < T; ++t) {
        load_x(t + 2, xc);
        float s = 0.0f, c = 0.0f, av = 0.0f;  // av: sum |w x|, the scale of every rounding error
#pragma unroll
        for (uint32_t i = 0; i < RS_IT; ++i) {
            const float x0 = __uint_as_float(xa[i].x << 16), x1 = __uint_as_float(xa[i].x & 0xFFFF0000u);
            const float x2 = __uint_as_float(xa[i].y << 16), x3 = __uint_as_float(xa[i].y & 0xFFFF0000u);
            dot_pair(s, c, wv[i].x, x0);
            dot_pair(s, c, wv[i].y, x1);
            dot_pair(s, c, wv[i].z, x2);
            dot_pair(s, c, wv[i].w, x3);
            av += fabsf(wv[i].x * x0) + fabsf(wv[i].y * x1) + fabsf(wv[i].z * x2) + fabsf(wv[i].w * x3);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float os = __shfl_xor_sync(0xffffffffu, s, o), oc = __shfl_xor_sync(0xffffffffu, c, o);
            c = __fadd_rn(c, oc);
            two_sum_into(s, c, os);
            av += __shfl_xor_sync(0xffffffffu, av, o);
        }
        if (lane == 0) {
            part[wp][t] = (double)s + (double)c;
            apart[wp][t] = av;
        }
#pragma unroll
        for (uint32_t i = 0; i < RS_IT; ++i) {
            xa[i] = xb[i];
            xb[i] = xc[i];
        }
    }
    __syncthreads();
    for (uint32_t t = threadIdx.x; t < T; t += blockDim.x) {
        double v = part[0][t];
        float av = apart[0][t];
        for (int q = 1; q < 8; ++q) {  // the eighths in order
            v += part[q][t];
            av += apart[q][t];
        }
        L[(size_t)t * E + e] = (float)v;
        Ld[(size_t)t * E + e] = v;
        sabs[(size_t)t * E + e] = av;
    }
}
int launch_router_logits_few(const uint16_t *x, const float *w, float *L, double *Ld, float *sabs,
                             uint32_t *flag_count, uint32_t T, uint32_t E, uint32_t H, cudaStream_t s) {
    if (T > RS_TMAX || H % 32 || H > 32 * 32 * RS_IT || (reinterpret_cast<uintptr_t>(x) & 7) ||
        (reinterpret_cast<uintptr_t>(w) & 15))
        return CK_ERR_SHAPE;
    if (!T || !E) return 0;
    const cudaError_t e = launch_pdl(k_router_logits_few, dim3(E), dim3(256), 0, s, x, w, L, Ld, sabs, flag_count, T, E, H);
    return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

// ------------------------------------------------------------------ 2. fast selection
// One warp per token; lane l holds experts e = 32*i + l.  At most 256 experts, 16 selections.
constexpr int RMAX = 8;
CK_DEV float sel_exp(float v) { return expf(v); }
CK_DEV double sel_exp(double v) { return exp(v); }
template <typename T>
CK_DEV T sel_max(T a, T b) { return a > b ? a : b; }
template <typename T>
CK_DEV T sel_min(T a, T b) { return a < b ? a : b; }
template <typename T>
CK_DEV void warp_argmax_t(T &v, int &i) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const T ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, i, o);
        if (ov > v || (ov == v && oi < i)) { v = ov; i = oi; }
    }
}
template <typename T>
CK_DEV T warp_sum_t(T v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// T = float: logits from the tensor cores, flagged below tau or 16 fp32 roundings of the largest
// logit.  T = double: logits from the decode-batch matvec, accurate to about 2^-44 of sum|w x|
// (`sabs` holds that sum per logit); the reference's own fold differs from the exact sum by at most
// 7168 x 2^-53 of it, so a token is flagged only when its margin is below 16 x 2^-40 of its largest
// sum|w x| -- in practice only exact ties take the fp64 re-route.
// `planes` (float form): the logits arrive as L plus nplanes more partial planes of [ntok, ne]
// (the tensor-core GEMM's K chunks 1 .. nplanes, chunk 0 in L); they are added to L in chunk order
// -- the additions the GEMM's own epilogue makes when it keeps the chunks together -- and the sum is
// written back to L.
template <typename T>
__global__ void k_route_select(const T *__restrict__ L, const float *__restrict__ sabs,
                               const float *__restrict__ bias, int32_t *__restrict__ ids, float *__restrict__ wts,
                               uint32_t *__restrict__ flag_list, uint32_t *__restrict__ flag_count, RouteParams p,
                               const float *__restrict__ planes, int nplanes) {
    grid_dep_trigger_small();
    grid_dep_wait();
    constexpr bool CTA = sizeof(T) == 8;  // the fp64 form: a CTA of 256 threads per token
    const int lane = threadIdx.x & 31;
    const uint32_t t = CTA ? blockIdx.x : (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (t >= p.ntok) return;
    const T NEG = (T)-3.0e38f;
    T sc[RMAX], pr[RMAX];
    const int nreg = (int)((p.ne + 31) / 32);
    float lmax = 0.0f;  // max |logit| (float form) or max sum|w x| (double form) of the token
    T pre_gsc = NEG;       // lane g: group g's score, when the CTA form computed it (one warp per group)
    bool have_gsc = false;
    if constexpr (CTA) {
        // one expert per thread: the 256 fp64 sigmoids (an exp and a division each, long dependent
        // chains on this GPU's fp64 pipe) in parallel instead of eight in a row per lane; warp 0
        // then selects from shared memory
        __shared__ T s_sc[256], s_pr[256];
        __shared__ float s_lmax[8];
        const int e = threadIdx.x;
        const bool v = e < (int)p.ne;
        const T l = v ? L[(size_t)t * p.ne + e] : NEG;
        float lm = v ? sabs[(size_t)t * p.ne + e] : 0.0f;
        T prv = (T)0, scv = NEG;
        if (v) {
            prv = p.mode == 4 ? (T)1 / ((T)1 + sel_exp(-l)) : l;
            scv = p.mode == 4 ? prv + (T)bias[e] : l;
        }
        s_sc[e] = scv;
        s_pr[e] = prv;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) lm = fmaxf(lm, __shfl_xor_sync(0xffffffffu, lm, o));
        if (lane == 0) s_lmax[threadIdx.x >> 5] = lm;
        __syncthreads();
        // groups of 32 experts (at most 8): warp g takes group g's two best scores, with the ties
        // and the sum of the warp form below
        __shared__ T s_gsc[8];
        have_gsc = p.mode == 4 && p.ngroups > 1 && p.ngroups <= 8 && p.ne == 32 * p.ngroups;
        if (have_gsc) {
            const int g = threadIdx.x >> 5;
            if (g < (int)p.ngroups) {
                T v = s_sc[threadIdx.x];
                int vi = (int)threadIdx.x;
                warp_argmax_t(v, vi);
                T b2 = (int)threadIdx.x != vi ? s_sc[threadIdx.x] : NEG;
                int dummy = 0;
                warp_argmax_t(b2, dummy);
                if (lane == 0) s_gsc[g] = b2 + v;  // tn-sum over (second, best): (0 + second) + best
            }
            __syncthreads();
            if (threadIdx.x < 32 && lane < (int)p.ngroups) pre_gsc = s_gsc[lane];
        }
        if (threadIdx.x >= 32) return;
#pragma unroll
        for (int i = 0; i < RMAX; ++i) {
            sc[i] = s_sc[32 * i + lane];
            pr[i] = s_pr[32 * i + lane];
            lmax = fmaxf(lmax, s_lmax[i]);
        }
    } else {
#pragma unroll
        for (int i = 0; i < RMAX; ++i) {
            const int e = 32 * i + lane;
            const bool v = i < nreg && e < (int)p.ne;
            T l = v ? L[(size_t)t * p.ne + e] : NEG;
            if (v && nplanes > 0) {
                const size_t at = (size_t)t * p.ne + e, plane = (size_t)p.ntok * p.ne;
                for (int a = 0; a < nplanes; ++a) l = l + (T)planes[a * plane + at];
                const_cast<T *>(L)[at] = l;
            }
            if (v) lmax = fmaxf(lmax, sabs ? sabs[(size_t)t * p.ne + e] : fabsf((float)l));
            if (p.mode == 4) {
                pr[i] = v ? (T)1 / ((T)1 + sel_exp(-l)) : (T)0;
                sc[i] = v ? pr[i] + (T)bias[e] : NEG;
            } else {
                pr[i] = l;
                sc[i] = l;
            }
        }
    }
    T margin = (T)3.0e38f;
    bool allowed[RMAX];
#pragma unroll
    for (int i = 0; i < RMAX; ++i) allowed[i] = true;
    // Per-group, per-pick and per-weight values live one per lane (group g or pick r in lane g or
    // r), not in arrays indexed at run time, which would sit in local memory on the selection's
    // chain of dependent steps.
    if (p.mode == 4 && p.ngroups > 1) {
        // group score = sum of the group's two best scores (ties: lower index first, like dsv4-topk)
        const int gs = (int)(p.ne / p.ngroups);
        T my_gsc = pre_gsc;  // lane g: group g's score
        for (int g = 0; g < (have_gsc ? 0 : (int)p.ngroups); ++g) {
            T b1 = NEG, b2 = NEG;
            int i1 = 1 << 30;
#pragma unroll
            for (int i = 0; i < RMAX; ++i) {
                const int e = 32 * i + lane;
                if (e / gs == g && sc[i] > b1) { b1 = sc[i]; i1 = e; }
            }
            T v = b1;
            int vi = i1;
            warp_argmax_t(v, vi);
            const T best = v;
#pragma unroll
            for (int i = 0; i < RMAX; ++i) {
                const int e = 32 * i + lane;
                if (e / gs == g && e != vi && sc[i] > b2) b2 = sc[i];
            }
            int dummy = 0;
            warp_argmax_t(b2, dummy);
            if (lane == g) my_gsc = b2 + best;  // tn-sum over (second, best): (0 + second) + best
        }
        // top groups by repeated argmax (ties: the lower group); the margin is min(chosen) -
        // max(rejected)
        unsigned gmask = 0;
        T gmin = (T)3.0e38f;
        for (int r = 0; r < (int)p.topk_groups; ++r) {
            T bv = lane < (int)p.ngroups && !(gmask >> lane & 1) ? my_gsc : NEG;
            int bi = lane;
            warp_argmax_t(bv, bi);
            gmask |= 1u << bi;
            gmin = sel_min(gmin, bv);
        }
        T gmax = lane < (int)p.ngroups && !(gmask >> lane & 1) ? my_gsc : NEG;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) gmax = sel_max(gmax, __shfl_xor_sync(0xffffffffu, gmax, o));
        if ((int)p.topk_groups < (int)p.ngroups) margin = sel_min(margin, gmin - gmax);
#pragma unroll
        for (int i = 0; i < RMAX; ++i) {
            const int e = 32 * i + lane;
            allowed[i] = e < (int)p.ne && (gmask >> (e / gs) & 1);
        }
    }
    // expert selection, best first: lane r keeps the r-th pick
    const int k = (int)p.nsel;
    int my_sel = 0;
    T my_selv = NEG, last = NEG;
    for (int r = 0; r < k; ++r) {
        T bv = NEG;
        int bi = 1 << 30;
#pragma unroll
        for (int i = 0; i < RMAX; ++i)
            if (allowed[i] && sc[i] > bv) { bv = sc[i]; bi = 32 * i + lane; }
        warp_argmax_t(bv, bi);
        if (lane == r) {
            my_sel = bi;
            my_selv = bv;
        }
        last = bv;
#pragma unroll
        for (int i = 0; i < RMAX; ++i)
            if (32 * i + lane == bi) allowed[i] = false;
    }
    {
        T bv = NEG;
        int bi = 1 << 30;
#pragma unroll
        for (int i = 0; i < RMAX; ++i)
            if (allowed[i] && sc[i] > bv) { bv = sc[i]; bi = 32 * i + lane; }
        warp_argmax_t(bv, bi);
        if (bv > NEG) margin = sel_min(margin, last - bv);
        // the list order of the chosen experts is part of the answer: two chosen experts closer
        // than the margin could be listed in the other order by an exact fold
        const T prev = __shfl_up_sync(0xffffffffu, my_selv, 1);
        T dm = lane >= 1 && lane < k ? prev - my_selv : (T)3.0e38f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) dm = sel_min(dm, __shfl_xor_sync(0xffffffffu, dm, o));
        margin = sel_min(margin, dm);
    }
    // weights
    if (p.mode == 4) {
        // dsv4-topk lists the picks last-first; weights from the unbiased probs, sum floored at
        // 2^-14, times wscale / sum (dsv4-forward.fk:105-111); lane r holds list position r
        T s0 = (T)0, my_w = (T)0;
        for (int r = 0; r < k; ++r) {
            const int e = __shfl_sync(0xffffffffu, my_sel, k - 1 - r);
            T pe = (T)0;
#pragma unroll
            for (int i = 0; i < RMAX; ++i)
                if (32 * i + lane == e) pe = pr[i];
            pe = __shfl_sync(0xffffffffu, pe, e & 31);
            if (lane == r) my_w = pe;
            s0 += pe;
        }
        const T s = s0 < (T)6.103515625e-05f ? (T)6.103515625e-05f : s0;
        const T scl = (T)p.wscale / s;
        my_w *= scl;
        const int my_id = __shfl_sync(0xffffffffu, my_sel, (k - 1 - lane) & 31);
        if (lane < k) {
            ids[(size_t)t * k + lane] = my_id;
            wts[(size_t)t * k + lane] = (float)my_w;
        }
    } else {
        // softmax over all experts (max-subtracted), the chosen probabilities, best first
        T mx = NEG;
#pragma unroll
        for (int i = 0; i < RMAX; ++i) mx = sel_max(mx, sc[i]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = sel_max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        T s = (T)0;
#pragma unroll
        for (int i = 0; i < RMAX; ++i)
            if (32 * i + lane < (int)p.ne) s += sel_exp(sc[i] - mx);
        s = warp_sum_t(s);
        if (lane < k) {
            ids[(size_t)t * k + lane] = my_sel;
            wts[(size_t)t * k + lane] = (float)(sel_exp(my_selv - mx) / s);
        }
    }
    // the threshold: tau, or 16 roundings of the largest logit (float form) / 16 x 2^-40 of the
    // largest sum|w x| (double form) when that is larger
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) lmax = fmaxf(lmax, __shfl_xor_sync(0xffffffffu, lmax, o));
    const T tau = sel_max((T)p.tau, (T)(sabs ? 16.0 * 9.094947017729282e-13 * lmax : 16.0 * 5.9604645e-8 * lmax));
    if (lane == 0 && !(margin > tau)) {  // an exact tie (margin 0) always goes to the exact path
        const uint32_t slot = atomicAdd(flag_count, 1u);
        flag_list[slot] = t;
    }
}

// ------------------------------------------------------------------ single-token Form routers
// form_moe_route_f32 / form_moe_route_wide_f32 (moe-msl.fk:114-117, moe-route-wide-msl.fk):
// softmax over ne logits, top-nsel best first, renormalized over the chosen.
__global__ void k_route_softmax_tokens(const float *__restrict__ L, uint32_t *__restrict__ ids, float *__restrict__ wts,
                                       uint32_t ne, uint32_t nsel, uint32_t ntok, int renorm) {
    const int lane = threadIdx.x & 31;
    const uint32_t t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (t >= ntok) return;
    float v[RMAX];
    float mx = -3.0e38f;
#pragma unroll
    for (int i = 0; i < RMAX; ++i) {
        const int e = 32 * i + lane;
        v[i] = e < (int)ne ? L[(size_t)t * ne + e] : -3.0e38f;
        mx = fmaxf(mx, v[i]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < RMAX; ++i) {
        v[i] = (32 * i + lane < (int)ne) ? expf(v[i] - mx) : -1.0f;
        if (v[i] > 0.0f) s += v[i];
    }
    s = warp_sum(s);
    const float inv = 1.0f / s;
#pragma unroll
    for (int i = 0; i < RMAX; ++i)
        if (v[i] >= 0.0f) v[i] *= inv;
    float pick[8];
    int pid[8];
    float wsum = 0.0f;
    for (uint32_t r = 0; r < nsel; ++r) {
        float bv = -2.0f;
        int bi = 1 << 30;
#pragma unroll
        for (int i = 0; i < RMAX; ++i)
            if (v[i] > bv) { bv = v[i]; bi = 32 * i + lane; }
        warp_argmax(bv, bi);
        pick[r] = bv;
        pid[r] = bi;
        wsum += bv;
#pragma unroll
        for (int i = 0; i < RMAX; ++i)
            if (32 * i + lane == bi) v[i] = -2.0f;
    }
    if (lane == 0) {
        const float winv = 1.0f / wsum;
        for (uint32_t r = 0; r < nsel; ++r) {
            ids[(size_t)t * nsel + r] = (uint32_t)pid[r];
            wts[(size_t)t * nsel + r] = renorm ? pick[r] * winv : pick[r];
        }
    }
}

// form_dsv4_router_f32 (dsv4-router-msl.fk:103-106): probs = sqrt(log(1 + exp(l))), selection on
// probs + bias, weights from the probs, sum floored at 2^-14, times wscale/sum, ids last-first.
__global__ void k_route_dsv4_tokens(const float *__restrict__ L, const float *__restrict__ bias,
                                    uint32_t *__restrict__ ids, float *__restrict__ wts, uint32_t ne, uint32_t nused,
                                    float wscale, uint32_t ntok) {
    const int lane = threadIdx.x & 31;
    const uint32_t t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (t >= ntok) return;
    float pr[RMAX], sc[RMAX];
#pragma unroll
    for (int i = 0; i < RMAX; ++i) {
        const int e = 32 * i + lane;
        if (e < (int)ne) {
            pr[i] = sqrtf(log1pf(expf(L[(size_t)t * ne + e])));
            sc[i] = pr[i] + bias[e];
        } else {
            pr[i] = 0.0f;
            sc[i] = -3.0e38f;
        }
    }
    int pick[8];
    for (uint32_t r = 0; r < nused; ++r) {
        float bv = -3.0e38f;
        int bi = 1 << 30;
#pragma unroll
        for (int i = 0; i < RMAX; ++i)
            if (sc[i] > bv) { bv = sc[i]; bi = 32 * i + lane; }
        warp_argmax(bv, bi);
        pick[r] = bi;
#pragma unroll
        for (int i = 0; i < RMAX; ++i)
            if (32 * i + lane == bi) sc[i] = -3.0e38f;
    }
    float pp[8];
    float s0 = 0.0f;
    for (uint32_t r = 0; r < nused; ++r) {
        float pe = 0.0f;
#pragma unroll
        for (int i = 0; i < RMAX; ++i)
            if (32 * i + lane == pick[r]) pe = pr[i];
        pp[r] = __shfl_sync(0xffffffffu, pe, pick[r] & 31);
        s0 += pp[r];
    }
    if (lane == 0) {
        const float s = s0 < 6.103515625e-05f ? 6.103515625e-05f : s0;
        const float scl = wscale / s;
        for (uint32_t j = 0; j < nused; ++j) {
            const uint32_t src = nused - 1 - j;
            ids[(size_t)t * nused + j] = (uint32_t)pick[src];
            wts[(size_t)t * nused + j] = pp[src] * scl;
        }
    }
}

// ------------------------------------------------------------------ router split for the tensor cores
// out[r, i*k + j] = term i of w[r, j]: t1 = bf16(w), t2 = bf16(w - t1), t3 = bf16(w - t1 - t2).
// Each difference is exact in fp32, so t1 + t2 + t3 carries about 24 significand bits of w and
// x . (t1 + t2 + t3) on bf16 tensor cores (exact bf16 products, fp32 accumulation) stands in for
// the fp32 router product.
__global__ void k_split_bf16x3(const float *__restrict__ w, __nv_bfloat16 *__restrict__ out, uint32_t rows, uint32_t k) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (uint64_t)rows * k) return;
    const uint64_t r = i / k, j = i - r * k;
    const float v = w[i];
    const __nv_bfloat16 a = __float2bfloat16_rn(v);
    const float r1 = v - __bfloat162float(a);
    const __nv_bfloat16 b = __float2bfloat16_rn(r1);
    const float r2 = r1 - __bfloat162float(b);
    const __nv_bfloat16 c = __float2bfloat16_rn(r2);
    __nv_bfloat16 *o = out + r * 3 * k;
    o[j] = a;
    o[k + j] = b;
    o[2 * k + j] = c;
}
int launch_split_bf16x3(const float *w, uint16_t *out, uint32_t rows, uint32_t k, cudaStream_t s) {
    const uint64_t n = (uint64_t)rows * k;
    if (n) k_split_bf16x3<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(w, (__nv_bfloat16 *)out, rows, k);
    return (int)cudaGetLastError();
}

// ------------------------------------------------------------------ launchers
int launch_router_logits(const uint16_t *x, const float *w, float *L, uint32_t T, uint32_t E, uint32_t H,
                         cudaStream_t s) {
    if (!T || !E) return 0;
    k_router_logits<<<dim3((T + 63) / 64, (E + 63) / 64), 256, 0, s>>>(x, w, L, T, E, H);
    return (int)cudaGetLastError();
}
int launch_route_select(float *L, const float *planes, int nplanes, const float *bias, int32_t *ids, float *wts,
                        uint32_t *flag_list, uint32_t *flag_count, const RouteParams &p, cudaStream_t s) {
    if (nplanes < 0 || nplanes > 7 || (nplanes && !planes)) return CK_ERR_ARG;
    if (p.ne == 0 || p.ne > 32 * RMAX || p.nsel == 0 || p.nsel > 16 || p.nsel > p.ne) return CK_ERR_SHAPE;
    if (p.mode == 4 && (p.ngroups == 0 || p.ngroups > 32 || p.ne % p.ngroups || p.topk_groups == 0 ||
                        p.topk_groups > p.ngroups || p.nsel > p.topk_groups * (p.ne / p.ngroups)))
        return CK_ERR_SHAPE;
    if (p.mode == 4 && !bias) return CK_ERR_ARG;
    cudaMemsetAsync(flag_count, 0, sizeof(uint32_t), s);
    if (p.ntok)
        k_route_select<float><<<(p.ntok * 32 + 255) / 256, 256, 0, s>>>(L, nullptr, bias, ids, wts, flag_list,
                                                                          flag_count, p, planes, nplanes);
    return (int)cudaGetLastError();
}
int launch_route_select_d(const double *L, const float *sabs, const float *bias, int32_t *ids, float *wts,
                          uint32_t *flag_list, uint32_t *flag_count, const RouteParams &p, cudaStream_t s) {
    if (p.ne == 0 || p.ne > 32 * RMAX || p.nsel == 0 || p.nsel > 16 || p.nsel > p.ne) return CK_ERR_SHAPE;
    if (p.mode == 4 && (p.ngroups == 0 || p.ngroups > 32 || p.ne % p.ngroups || p.topk_groups == 0 ||
                        p.topk_groups > p.ngroups || p.nsel > p.topk_groups * (p.ne / p.ngroups)))
        return CK_ERR_SHAPE;
    if (p.mode == 4 && !bias) return CK_ERR_ARG;
    if (!sabs) return CK_ERR_ARG;
    // flag_count was cleared by launch_router_logits_few, the kernel before this one
    if (p.ntok) {
        const cudaError_t e = launch_pdl(k_route_select<double>, dim3(p.ntok), dim3(256), 0, s, L, sabs, bias, ids, wts,
                                         flag_list, flag_count, p, (const float *)nullptr, 0);
        if (e != cudaSuccess) return (int)e;
    }
    return (int)cudaGetLastError();
}
int launch_route_softmax_tokens(const float *L, uint32_t *ids, float *wts, uint32_t ne, uint32_t nsel, uint32_t ntok,
                                int renorm, cudaStream_t s) {
    if (ne == 0 || ne > 32 * RMAX || nsel == 0 || nsel > 8 || nsel > ne) return CK_ERR_SHAPE;
    if (ntok) k_route_softmax_tokens<<<(ntok * 32 + 127) / 128, 128, 0, s>>>(L, ids, wts, ne, nsel, ntok, renorm);
    return (int)cudaGetLastError();
}
int launch_route_dsv4_tokens(const float *L, const float *bias, uint32_t *ids, float *wts, uint32_t ne, uint32_t nused,
                             float wscale, uint32_t ntok, cudaStream_t s) {
    if (ne == 0 || ne > 32 * RMAX || nused == 0 || nused > 8 || nused > ne) return CK_ERR_SHAPE;
    if (ntok) k_route_dsv4_tokens<<<(ntok * 32 + 127) / 128, 128, 0, s>>>(L, bias, ids, wts, ne, nused, wscale, ntok);
    return (int)cudaGetLastError();
}

}  // namespace ck
