// api.cu -- the extern "C" entry points declared in include/ck_b200.h.
#include "../../include/ck_b200.h"
#include "ck_common.cuh"
#include "ck_launch.h"

#include <mutex>
#include <stdio.h>
#include <string.h>

namespace {
thread_local char g_err[512] = "none";

int fail(int rc, const char *what) {
    if (rc == 0) return 0;
    const char *why = rc > 0 ? cudaGetErrorString((cudaError_t)rc)
                             : rc == CK_ESHAPE ? "unsupported shape"
                             : rc == CK_EARG ? "bad argument"
                             : rc == CK_ETIMEOUT ? "device wait timed out"
                             : rc == CK_ENODEV ? "no device / driver entry point"
                                                : "error";
    snprintf(g_err, sizeof(g_err), "%s: %s (%d)", what, why, rc);
    return rc;
}
inline cudaStream_t S(void *s) { return reinterpret_cast<cudaStream_t>(s); }
// The router logits GEMM gives each K-chunk accumulator a work unit of its own when its unsplit
// units (64-token tiles x 128-expert blocks) would fill at most half the GPU's 148 SMs; beyond that
// the short units' pipeline fills and the partial planes' traffic cost more than they save.
inline uint32_t route_ksplit_max(const ck_moe_config *c) {  // the largest batch that splits
    return 64u * (74u / ((c->n_experts + 127) / 128));
}
inline bool route_ksplit(const ck_moe_config *c, uint32_t ntok) {
    return ntok > CK_MOE_DECODE_TOKENS && ntok <= route_ksplit_max(c);
}
inline size_t al(size_t b) { return (b + 255) & ~(size_t)255; }

// The router's scratch: the three-term bf16 split of the router, its token tiles, the flagged-
// token list (count first), and a device error word.
struct RouteWs {
    uint16_t *wsplit;
    int4 *tiles;
    int32_t *ntiles;
    int *err;
    uint32_t *flags;
    double *exact;  // fp64 logits of the flagged tokens (and of every token on the decode-batch path)
    float *sabs;    // sum |w x| per logit on the decode-batch path
    double *w64;    // the router in fp64, for the exact re-route
    float *planes;  // the logits GEMM's K-chunk partial sums 1 .. 7 (chunk 0 in the logits)
    size_t total;
};
RouteWs route_ws(const ck_moe_config *c, uint32_t ntok, void *base) {
    RouteWs w;
    uint8_t *b = (uint8_t *)base;
    size_t o = 0;
    auto take = [&](size_t bytes) { uint8_t *p = b ? b + o : nullptr; o += al(bytes); return p; };
    w.wsplit = (uint16_t *)take((size_t)c->n_experts * 3 * c->hidden * 2);
    w.tiles = (int4 *)take(((size_t)ntok / 16 + 2) * 16);
    w.ntiles = (int32_t *)take(4);
    w.err = (int *)take(4);
    w.flags = (uint32_t *)take(((size_t)ntok + 1) * 4);
    w.exact = (double *)take((size_t)ntok * c->n_experts * 8);
    w.sabs = (float *)take((size_t)ntok * c->n_experts * 4);
    w.w64 = (double *)take((size_t)c->n_experts * c->hidden * 8);
    // sized for min(ntok, the largest split batch) above the decode sizes, so that the workspace
    // grows with ntok: one sized for a batch holds every smaller one
    const uint32_t np = ntok > CK_MOE_DECODE_TOKENS ? (ntok < route_ksplit_max(c) ? ntok : route_ksplit_max(c)) : 0;
    w.planes = np ? (float *)take((size_t)7 * np * c->n_experts * 4) : nullptr;
    w.total = o;
    return w;
}

struct MoeWs {
    float *logits;
    void *route;
    void *perm_ws;
    uint16_t *xp;
    float *row_w;
    int32_t *pair_pos;
    int4 *tiles;
    int32_t *ntiles;
    uint16_t *h;
    uint16_t *y;
    int *err;
    size_t total;
};

// Token tiles of the permute's table: decode-sized batches (at most CK_MOE_DECODE_TOKENS tokens) cut
// them to CK_MOE_FEW_TOKENS tokens, so that every tile fits the few-token grouped matvec; larger
// batches use the grouped GEMM's tiles of up to GEMM_TILE_TOKENS.  Five tokens (15 accumulator
// columns per K step, 16 with the padding) is the most whose accumulators fit twice in the
// matvec's tensor memory beside its weight stages.
uint32_t moe_tile_tokens(uint32_t ntok) {
    return ntok <= CK_MOE_DECODE_TOKENS ? (uint32_t)CK_MOE_FEW_TOKENS : ck::GEMM_TILE_TOKENS;
}

ck::PermuteParams perm_params(const ck_moe_config *c, uint32_t ntok) {
    ck::PermuteParams p;
    p.ntok = ntok;
    p.nsel = c->nsel;
    p.n_experts = c->n_experts;
    p.n_shared = c->n_shared;
    p.hidden = c->hidden;
    p.bn = moe_tile_tokens(ntok);
    p.weight_in_mid = c->mode == 4 ? 1 : 0;
    return p;
}

MoeWs moe_ws(const ck_moe_config *c, uint32_t ntok, void *base) {
    MoeWs w;
    const size_t A = (size_t)ntok * c->nsel, XR = A + ntok, R = A + (size_t)c->n_shared * ntok;
    const uint32_t mt = ck_moe_max_tiles(ntok, c->nsel, c->n_experts, c->n_shared);
    uint8_t *b = (uint8_t *)base;
    size_t o = 0;
    auto take = [&](size_t bytes) { uint8_t *p = b ? b + o : nullptr; o += al(bytes); return p; };
    w.logits = (float *)take((size_t)ntok * c->n_experts * 4);
    w.route = take(route_ws(c, ntok, nullptr).total);
    w.perm_ws = take(ck::permute_workspace_bytes(perm_params(c, ntok)));
    w.xp = (uint16_t *)take(XR * c->hidden * 2);
    w.row_w = (float *)take(R * 4);
    w.pair_pos = (int32_t *)take(A * 4);
    w.tiles = (int4 *)take((size_t)mt * 16);
    w.ntiles = (int32_t *)take(4);
    w.h = (uint16_t *)take(R * c->inter * 2);
    w.y = (uint16_t *)take(R * c->hidden * 2);
    w.err = (int *)take(4);
    w.total = o;
    return w;
}

int check_cfg(const ck_moe_config *c) {
    if (!c) return CK_EARG;
    if (c->n_experts == 0 || c->n_experts > 256 || c->nsel == 0 || c->nsel > 16 || c->nsel > c->n_experts)
        return CK_ESHAPE;
    if (c->hidden % 64 || c->inter % 64 || c->hidden == 0 || c->inter == 0) return CK_ESHAPE;
    if (c->mode != 3 && c->mode != 4) return CK_EARG;
    if (c->mode == 4 && (c->ngroups == 0 || c->ngroups > 32 || c->n_experts % c->ngroups || c->topk_groups == 0 ||
                         c->topk_groups > c->ngroups))
        return CK_ESHAPE;
    return 0;
}
}  // namespace

extern "C" {

const char *ck_last_error(void) { return g_err; }

int ck_device_ok(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) return 0;
    cudaDeviceProp prop;
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return 0;
    return prop.major == 10 ? 1 : 0;
}

int ck_q8_0_dequant_f32(const void *qb, float *w, uint64_t off, uint64_t n, void *s) {
    if (!qb || !w) return fail(CK_EARG, "ck_q8_0_dequant_f32");
    return fail(ck::launch_q80_dequant((const uint8_t *)qb, w, off, n, S(s)), "ck_q8_0_dequant_f32");
}
int ck_q4k_dequant_f32(const void *qb, float *w, uint64_t off, uint64_t n, void *s) {
    if (!qb || !w) return fail(CK_EARG, "ck_q4k_dequant_f32");
    return fail(ck::launch_q4k_dequant((const uint8_t *)qb, w, off, n, S(s)), "ck_q4k_dequant_f32");
}
int ck_q4k_dequant_bf16(const void *qb, void *w, uint64_t off, uint64_t n, void *s) {
    if (!qb || !w) return fail(CK_EARG, "ck_q4k_dequant_bf16");
    return fail(ck::launch_q4k_dequant_bf16((const uint8_t *)qb, w, off, n, S(s)), "ck_q4k_dequant_bf16");
}
int ck_q8_0_matvec_f32(const void *qb, const float *x, float *y, uint32_t rows, uint32_t cols, void *s) {
    if (!qb || !x || !y || (reinterpret_cast<uintptr_t>(qb) & 15) || (reinterpret_cast<uintptr_t>(x) & 15))
        return fail(CK_EARG, "ck_q8_0_matvec_f32");
    return fail(ck::launch_q80_matvec((const uint8_t *)qb, x, y, rows, cols, S(s)), "ck_q8_0_matvec_f32");
}
int ck_q4k_matvec_f32(const void *qb, const float *x, float *y, uint32_t rows, uint32_t cols, void *s) {
    if (!qb || !x || !y || (reinterpret_cast<uintptr_t>(qb) & 15) || (reinterpret_cast<uintptr_t>(x) & 15))
        return fail(CK_EARG, "ck_q4k_matvec_f32");
    return fail(ck::launch_q4k_matvec((const uint8_t *)qb, x, y, rows, cols, 1, S(s)), "ck_q4k_matvec_f32");
}
int ck_q4k_matvec_f32_group(uint32_t n, const void *const *qb, const float *x, float *const *y, uint32_t rows,
                            uint32_t cols, void *s) {
    if (!qb || !x || !y || n == 0 || n > 4 || (reinterpret_cast<uintptr_t>(x) & 15))
        return fail(CK_EARG, "ck_q4k_matvec_f32_group");
    for (uint32_t g = 0; g < n; ++g)
        if (!qb[g] || !y[g] || (reinterpret_cast<uintptr_t>(qb[g]) & 15)) return fail(CK_EARG, "ck_q4k_matvec_f32_group");
    return fail(ck::launch_q4k_matvec_group(n, reinterpret_cast<const uint8_t *const *>(qb), x, y, rows, cols, 1, S(s)),
                "ck_q4k_matvec_f32_group");
}
int ck_q4k_matmul_batch_f32(const void *qb, const float *x, float *y, uint32_t rows, uint32_t cols, uint32_t ntok,
                            void *s) {
    if (!qb || !x || !y || ntok == 0 || (reinterpret_cast<uintptr_t>(qb) & 15) ||
        (reinterpret_cast<uintptr_t>(x) & 15))
        return fail(CK_EARG, "ck_q4k_matmul_batch_f32");
    return fail(ck::launch_q4k_matvec((const uint8_t *)qb, x, y, rows, cols, ntok, S(s)), "ck_q4k_matmul_batch_f32");
}
int ck_matvec_ordered_f32(int t, const void *qb, const float *x, float *y, uint32_t rows, uint32_t cols, void *s) {
    if (!qb || !x || !y || (t != 8 && t != 12 && t != 14)) return fail(CK_EARG, "ck_matvec_ordered_f32");
    if ((t == 8 && cols % 32) || (t != 8 && ((uint64_t)rows * cols) % 256)) return fail(CK_ESHAPE, "ck_matvec_ordered_f32");
    if (t == 14)
        return fail(ck::launch_q6k_ordered((const uint8_t *)qb, x, y, rows, cols, S(s)), "ck_matvec_ordered_f32");
    return fail(ck::launch_matvec_ordered(t, (const uint8_t *)qb, x, y, rows, cols, S(s)), "ck_matvec_ordered_f32");
}
int ck_q6k_dequant_f32(const void *qb, float *w, uint64_t off, uint64_t n, void *s) {
    if (!qb || !w) return fail(CK_EARG, "ck_q6k_dequant_f32");
    return fail(ck::launch_q6k_dequant((const uint8_t *)qb, w, off, n, S(s)), "ck_q6k_dequant_f32");
}
int ck_q6k_matvec_f32(const void *qb, const float *x, float *y, uint32_t rows, uint32_t cols, void *s) {
    if (!qb || !x || !y) return fail(CK_EARG, "ck_q6k_matvec_f32");
    if (((uint64_t)rows * cols) % 256) return fail(CK_ESHAPE, "ck_q6k_matvec_f32");
    return fail(ck::launch_q6k_matvec((const uint8_t *)qb, x, y, rows, cols, 1, S(s)), "ck_q6k_matvec_f32");
}
int ck_q6k_matmul_batch_f32(const void *qb, const float *x, float *y, uint32_t rows, uint32_t cols, uint32_t ntok,
                            void *s) {
    if (!qb || !x || !y || ntok == 0) return fail(CK_EARG, "ck_q6k_matmul_batch_f32");
    if (((uint64_t)rows * cols) % 256) return fail(CK_ESHAPE, "ck_q6k_matmul_batch_f32");
    return fail(ck::launch_q6k_matvec((const uint8_t *)qb, x, y, rows, cols, ntok, S(s)), "ck_q6k_matmul_batch_f32");
}
int ck_q6k_matvec_part_f32(const void *qb, const float *x, float *part, uint32_t rows, uint32_t cols, uint32_t parts,
                           void *s) {
    if (!qb || !x || !part || parts == 0) return fail(CK_EARG, "ck_q6k_matvec_part_f32");
    if (((uint64_t)rows * cols) % 256) return fail(CK_ESHAPE, "ck_q6k_matvec_part_f32");
    return fail(ck::launch_q6k_part((const uint8_t *)qb, x, part, rows, cols, parts, S(s)), "ck_q6k_matvec_part_f32");
}

size_t ck_q4k_gemm_workspace_bytes(uint32_t ntok) { return al(((size_t)ntok / 16 + 2) * 16) + 256 + 256; }

int ck_q4k_gemm_bf16(const void *qb, const void *x, void *y, uint32_t rows, uint32_t cols, uint32_t ntok, void *ws,
                     size_t wsb, void *s) {
    if (!qb || !x || !y || !ws) return fail(CK_EARG, "ck_q4k_gemm_bf16");
    if (wsb < ck_q4k_gemm_workspace_bytes(ntok)) return fail(CK_EARG, "ck_q4k_gemm_bf16 workspace");
    if (ntok == 0) return 0;
    uint8_t *b = (uint8_t *)ws;
    const size_t tb = al(((size_t)ntok / 16 + 2) * 16);
    int4 *tiles = (int4 *)b;
    int32_t *ntiles = (int32_t *)(b + tb);
    int *err = (int *)(b + tb + 256);
    cudaMemsetAsync(err, 0, 4, S(s));
    int rc = ck::launch_single_tiles(tiles, ntiles, ntok, ck::GEMM_TILE_TOKENS, S(s));
    if (rc) return fail(rc, "ck_q4k_gemm_bf16 tiles");
    ck::GemmParams p = {};
    p.w0 = (const uint8_t *)qb;
    p.w_stride = 0;
    p.x = x;
    p.x_rows = ntok;
    p.out = y;
    p.out_rows = ntok;
    p.tiles = tiles;
    p.ntiles = ntiles;
    p.max_tiles = (uint32_t)(ntok / 16 + 2);
    p.n_routed = 1;
    // up to 4 tokens the table is one tile of ntok: the weights stream through the few-token
    // tensor-core matvec instead of the dequantizing GEMM (11008 x 4096: 19 / 21 / 28 us at 1 / 2 /
    // 4 tokens against the GEMM's 35-39; at 8 tokens the GEMM is ahead)
    p.max_tile_tok = ntok <= 4 ? ntok : 0;
    p.N = rows;
    p.K = cols;
    p.dual = 0;
    p.err = err;
    return fail(ck::launch_gemm_q4k(p, S(s)), "ck_q4k_gemm_bf16");
}

// Reads the error word ck_q4k_gemm_bf16 left in its workspace (synchronizes the stream).
int ck_q4k_gemm_status(uint32_t ntok, const void *ws, void *s) {
    if (!ws) return fail(CK_EARG, "ck_q4k_gemm_status");
    const size_t tb = al(((size_t)ntok / 16 + 2) * 16);
    int e = 0;
    cudaError_t r = cudaMemcpyAsync(&e, (const uint8_t *)ws + tb + 256, 4, cudaMemcpyDeviceToHost, S(s));
    if (r == cudaSuccess) r = cudaStreamSynchronize(S(s));
    if (r != cudaSuccess) return fail((int)r, "ck_q4k_gemm_status");
    if (e) {
        snprintf(g_err, sizeof(g_err), "ck_q4k_gemm_bf16: device wait timed out (role code %d)", e);
        return CK_ETIMEOUT;
    }
    return 0;
}

int ck_f16_matvec_f32(const void *w, const float *x, float *y, uint32_t rows, uint32_t cols, void *s) {
    if (!w || !x || !y) return fail(CK_EARG, "ck_f16_matvec_f32");
    return fail(ck::launch_f16_matvec((const uint16_t *)w, x, y, rows, cols, S(s)), "ck_f16_matvec_f32");
}
int ck_route_softmax_f32(const float *L, uint32_t *ids, float *wts, uint32_t ne, uint32_t nsel, uint32_t ntok,
                         int renorm, void *s) {
    if (!L || !ids || !wts) return fail(CK_EARG, "ck_route_softmax_f32");
    return fail(ck::launch_route_softmax_tokens(L, ids, wts, ne, nsel, ntok, renorm, S(s)), "ck_route_softmax_f32");
}
int ck_route_dsv4_f32(const float *L, const float *bias, uint32_t *ids, float *wts, uint32_t ne, uint32_t nused,
                      float wscale, uint32_t ntok, void *s) {
    if (!L || !bias || !ids || !wts) return fail(CK_EARG, "ck_route_dsv4_f32");
    return fail(ck::launch_route_dsv4_tokens(L, bias, ids, wts, ne, nused, wscale, ntok, S(s)), "ck_route_dsv4_f32");
}
int ck_scale_f32(const float *x, float *y, float a, uint32_t n, void *s) {
    if (!x || !y) return fail(CK_EARG, "ck_scale_f32");
    return fail(ck::launch_scale(x, y, a, n, S(s)), "ck_scale_f32");
}
int ck_axpy_f32(const float *x, float *y, float a, uint32_t n, void *s) {
    if (!x || !y) return fail(CK_EARG, "ck_axpy_f32");
    return fail(ck::launch_axpy(x, y, a, n, S(s)), "ck_axpy_f32");
}
int ck_swiglu_f32(const float *g, const float *u, float *o, uint32_t n, float w, float lim, void *s) {
    if (!g || !u || !o) return fail(CK_EARG, "ck_swiglu_f32");
    return fail(ck::launch_swiglu(g, u, o, n, w, lim, S(s)), "ck_swiglu_f32");
}

// ------------------------------------------------------------------------------ MoE layer
uint32_t ck_moe_max_tiles(uint32_t ntok, uint32_t nsel, uint32_t n_experts, uint32_t n_shared) {
    // A segment of c rows makes ceil(c / bn) tiles (permute's seg_tiles), at most c / bn + 1.  The
    // bound is monotone in ntok, so a table sized for ntok also holds the tiles of any smaller batch,
    // whose tiles may be the shorter decode-sized ones (a caller sizes once for its largest batch).
    const auto bound = [&](uint64_t t, uint64_t bn) {
        return n_experts + t * nsel / bn + 1 + (uint64_t)n_shared * (t / bn + 2);
    };
    const uint64_t few = bound(ntok < CK_MOE_DECODE_TOKENS ? ntok : CK_MOE_DECODE_TOKENS, CK_MOE_FEW_TOKENS);
    const uint64_t big = ntok > CK_MOE_DECODE_TOKENS ? bound(ntok, 128) : 0;
    return (uint32_t)(few > big ? few : big);
}
size_t ck_moe_permute_workspace_bytes(uint32_t ntok, uint32_t nsel, uint32_t n_experts) {
    ck::PermuteParams p = {};
    p.ntok = ntok;
    p.nsel = nsel;
    p.n_experts = n_experts;
    return ck::permute_workspace_bytes(p);
}
size_t ck_moe_workspace_bytes(const ck_moe_config *c, uint32_t ntok) {
    if (check_cfg(c)) return 0;
    return moe_ws(c, ntok, nullptr).total;
}

size_t ck_moe_route_workspace_bytes(const ck_moe_config *c, uint32_t ntok) {
    if (check_cfg(c)) return 0;
    return route_ws(c, ntok, nullptr).total;
}

int ck_moe_route(const ck_moe_config *c, const void *x, uint32_t ntok, const float *rw, const float *bias,
                 float *logits, int32_t *ids, float *wts, void *ws, size_t wsb, void *s) {
    int rc = check_cfg(c);
    if (rc) return fail(rc, "ck_moe_route config");
    if (!x || !rw || !logits || !ids || !wts || !ws || (c->mode == 4 && !bias)) return fail(CK_EARG, "ck_moe_route");
    if (wsb < ck_moe_route_workspace_bytes(c, ntok)) return fail(CK_EARG, "ck_moe_route workspace");
    if (ntok == 0) return 0;
    RouteWs w = route_ws(c, ntok, ws);
    ck::RouteParams p = {ntok, c->n_experts, c->nsel, c->hidden, c->mode, c->ngroups, c->topk_groups, c->wscale, c->tau};
    // A decode-sized batch (at most CK_MOE_DECODE_TOKENS tokens): the router as a matvec over all SMs with compensated
    // sums, selected in fp64 with a margin sized by the dot's own rounding (about 1e-9 here), so in
    // practice only exact ties take the fp64 re-route.  Otherwise the logits run on the tensor cores,
    // x . [W1 | W2 | W3]^T with the fp32 router split into bf16 terms, and are selected in fp32
    // with the margin tau.
    rc = ntok <= CK_MOE_DECODE_TOKENS ? ck::launch_router_logits_few((const uint16_t *)x, rw, logits, w.exact, w.sabs, w.flags, ntok,
                                                   c->n_experts, c->hidden, S(s))
                    : CK_ERR_SHAPE;
    if (rc == 0) {
        p.tau = 0.0f;
        rc = ck::launch_route_select_d(w.exact, w.sabs, bias, ids, wts, w.flags + 1, w.flags, p, S(s));
        if (rc) return fail(rc, "ck_moe_route select");
    } else if (rc == CK_ERR_SHAPE) {
        rc = ck::launch_split_bf16x3(rw, w.wsplit, c->n_experts, c->hidden, S(s));
        if (!rc) rc = ck::launch_single_tiles(w.tiles, w.ntiles, ntok, 64, S(s));
        if (rc) return fail(rc, "ck_moe_route split");
        cudaMemsetAsync(w.err, 0, 4, S(s));
        ck::GemmParams g = {};
        g.a_dense = w.wsplit;
        g.kx = c->hidden;
        g.K = 3 * c->hidden;
        g.N = c->n_experts;
        g.x = x;
        g.x_rows = ntok;
        g.out_f32 = logits;
        g.out_rows = ntok;
        g.tiles = w.tiles;
        g.ntiles = w.ntiles;
        g.max_tiles = ntok / 16 + 2;
        g.err = w.err;
        // a small batch: each of the GEMM's eight K-chunk accumulators is a unit of its own (eight
        // times the CTAs: 1024 tokens otherwise ran on 32 of them), and the selection adds the
        // chunks in order -- the same sums as the unsplit epilogue's, so the same logits
        const bool split = route_ksplit(c, ntok);
        g.ksplit = split ? 8 : 1;
        g.out_planes = w.planes;
        rc = ck::launch_gemm_dense(g, S(s));
        if (rc) return fail(rc, "ck_moe_route logits");
        const int nk = (int)(3 * c->hidden / 64), kchunk = (nk + 7) / 8;
        rc = ck::launch_route_select(logits, w.planes, split ? (nk + kchunk - 1) / kchunk - 1 : 0, bias, ids, wts,
                                     w.flags + 1, w.flags, p, S(s));
        if (rc) return fail(rc, "ck_moe_route select");
    } else {
        return fail(rc, "ck_moe_route logits");
    }
    rc = ck::launch_route_exact((const uint16_t *)x, rw, bias, ids, wts, w.flags + 1, w.flags, w.exact, w.w64, p,
                                S(s));
    return fail(rc, "ck_moe_route exact");
}

// How many tokens the last ck_moe_route sent to the exact fp64 re-route (synchronizes the stream).
int ck_moe_route_flagged(const ck_moe_config *c, uint32_t ntok, const void *ws, void *s) {
    if (check_cfg(c) || !ws) return fail(CK_EARG, "ck_moe_route_flagged");
    RouteWs w = route_ws(c, ntok, const_cast<void *>(ws));
    uint32_t n = 0;
    cudaError_t r = cudaMemcpyAsync(&n, w.flags, 4, cudaMemcpyDeviceToHost, S(s));
    if (r == cudaSuccess) r = cudaStreamSynchronize(S(s));
    if (r != cudaSuccess) return fail((int)r, "ck_moe_route_flagged");
    return (int)n;
}

// The reference's router logits (tb-dot's right fold in fp64) of the listed tokens.
int ck_router_exact_logits(const void *x, const float *rw, const uint32_t *tokens, const uint32_t *count,
                           uint32_t n_experts, uint32_t hidden, double *out, double *router_f64, void *s) {
    if (!x || !rw || !tokens || !count || !out || !router_f64) return fail(CK_EARG, "ck_router_exact_logits");
    return fail(ck::launch_exact_logits((const uint16_t *)x, rw, tokens, count, out, router_f64, n_experts, hidden,
                                        0xffffffffu, S(s)),
                "ck_router_exact_logits");
}

int ck_moe_permute(const int32_t *ids, const float *wts, const void *x, uint32_t ntok, uint32_t nsel,
                   uint32_t n_experts, uint32_t n_shared, uint32_t hidden, int weight_in_mid, void *xp, float *row_w,
                   int32_t *pair_pos, int32_t *counts, void *tiles, int32_t *ntiles, void *ws, void *s) {
    ck::PermuteParams p = {ntok, nsel, n_experts, n_shared, hidden, moe_tile_tokens(ntok),
                           (uint32_t)(weight_in_mid ? 1 : 0)};
    return fail(ck::launch_permute(ids, wts, (const uint16_t *)x, (uint16_t *)xp, row_w, pair_pos, counts,
                                   (int4 *)tiles, ntiles, ws, p, S(s)),
                "ck_moe_permute");
}

int ck_moe_expert_gemm(int dual, const void *w0, const void *w1, const void *s0, const void *s1, uint64_t w_stride,
                       uint32_t n_routed, uint32_t n_shared, const void *x, uint32_t x_rows, void *out,
                       uint32_t out_rows, const float *row_w, const void *tiles, const int32_t *ntiles,
                       uint32_t max_tiles, uint32_t n, uint32_t k, int xrow_is_orow, int *err, void *s) {
    return ck_moe_expert_gemm_bounded(dual, w0, w1, s0, s1, w_stride, n_routed, n_shared, x, x_rows, out, out_rows,
                                      row_w, tiles, ntiles, max_tiles, n, k, xrow_is_orow, 0, err, s);
}

int ck_moe_expert_gemm_bounded(int dual, const void *w0, const void *w1, const void *s0, const void *s1,
                               uint64_t w_stride, uint32_t n_routed, uint32_t n_shared, const void *x, uint32_t x_rows,
                               void *out, uint32_t out_rows, const float *row_w, const void *tiles,
                               const int32_t *ntiles, uint32_t max_tiles, uint32_t n, uint32_t k, int xrow_is_orow,
                               uint32_t max_tile_tokens, int *err, void *s) {
    ck::GemmParams p = {};
    p.max_tile_tok = max_tile_tokens;
    p.w0 = (const uint8_t *)w0;
    p.w1 = (const uint8_t *)w1;
    p.s0 = (const uint8_t *)s0;
    p.s1 = (const uint8_t *)s1;
    p.n_shared = s0 ? n_shared : 0;
    p.w_stride = w_stride;
    p.x = x;
    p.x_rows = x_rows;
    p.out = out;
    p.out_rows = out_rows;
    p.row_w = row_w;
    p.tiles = (const int4 *)tiles;
    p.ntiles = ntiles;
    p.max_tiles = max_tiles;
    p.n_routed = n_routed;
    p.N = n;
    p.K = k;
    p.dual = dual;
    p.xrow_is_orow = xrow_is_orow;
    p.err = err;
    return fail(ck::launch_gemm_q4k(p, S(s)), "ck_moe_expert_gemm");
}

int ck_moe_expert_gemm_rows(const void *w0, uint64_t w_stride, uint32_t n_routed, const void *x, uint32_t x_rows,
                            const unsigned long long *row_dst, uint32_t out_rows, const void *tiles,
                            const int32_t *ntiles, uint32_t max_tiles, uint32_t n, uint32_t k, int xrow_is_orow,
                            int *err, void *s) {
    if (!row_dst) return fail(CK_ERR_ARG, "ck_moe_expert_gemm_rows: row_dst is null");
    ck::GemmParams p = {};
    p.w0 = (const uint8_t *)w0;
    p.w_stride = w_stride;
    p.x = x;
    p.x_rows = x_rows;
    p.row_dst = row_dst;
    p.out_rows = out_rows;
    p.tiles = (const int4 *)tiles;
    p.ntiles = ntiles;
    p.max_tiles = max_tiles;
    p.n_routed = n_routed;
    p.N = n;
    p.K = k;
    p.xrow_is_orow = xrow_is_orow;
    p.err = err;
    return fail(ck::launch_gemm_q4k(p, S(s)), "ck_moe_expert_gemm_rows");
}

int ck_moe_combine(const void *y, const int32_t *ids, const float *wts, const int32_t *pair_pos, uint32_t ntok,
                   uint32_t nsel, uint32_t n_shared, uint32_t hidden, int order_by_expert, void *out, float *out_f32,
                   void *s) {
    ck::PermuteParams p = {ntok, nsel, 0, n_shared, hidden, ck::GEMM_TILE_TOKENS, 0};
    return fail(ck::launch_combine((const uint16_t *)y, ids, wts, pair_pos, (uint16_t *)out, out_f32, p,
                                   order_by_expert, S(s)),
                "ck_moe_combine");
}

int ck_token_tiles(void *tiles, int32_t *ntiles, uint32_t ntok, void *s) {
    return fail(ck::launch_single_tiles((int4 *)tiles, ntiles, ntok, ck::GEMM_TILE_TOKENS, S(s)), "ck_token_tiles");
}
int ck_token_tiles_n(void *tiles, int32_t *ntiles, uint32_t ntok, uint32_t tile_tokens, void *s) {
    return fail(ck::launch_single_tiles((int4 *)tiles, ntiles, ntok, tile_tokens, S(s)), "ck_token_tiles_n");
}

int ck_ep_dispatch_plan(const int32_t *ids, const float *wts, uint32_t ntok, uint32_t nsel, uint32_t n_experts,
                        uint32_t world, int32_t *counts, int64_t *sizes, int32_t *send_tok, int32_t *meta,
                        int32_t *ret_pos, void *s) {
    return fail(ck::launch_ep_plan(ids, wts, ntok, nsel, n_experts, world, counts, (long long *)sizes, send_tok,
                                   meta, ret_pos, S(s)),
                "ck_ep_dispatch_plan");
}

int ck_gather_rows(const void *src, const int32_t *idx, void *dst, uint32_t nrows, uint32_t row_bytes, void *s) {
    return fail(ck::launch_gather_rows(src, idx, dst, nrows, row_bytes, S(s)), "ck_gather_rows");
}

int ck_moe_layer_bf16(const ck_moe_config *c, const void *x, uint32_t ntok, const void *wg, const void *wu,
                      const void *wd, const void *sg, const void *su, const void *sd, const float *rw,
                      const float *bias, int32_t *ids, float *wts, int32_t *counts, void *out, void *ws, size_t wsb,
                      void *s) {
    int rc = check_cfg(c);
    if (rc) return fail(rc, "ck_moe_layer_bf16 config");
    if (!x || !wg || !wu || !wd || !rw || !ids || !wts || !counts || !out || !ws) return fail(CK_EARG, "ck_moe_layer_bf16");
    if (c->n_shared && (!sg || !su || !sd)) return fail(CK_EARG, "ck_moe_layer_bf16 shared weights");
    if (wsb < ck_moe_workspace_bytes(c, ntok)) return fail(CK_EARG, "ck_moe_layer_bf16 workspace");
    if (ntok == 0) return 0;
    MoeWs w = moe_ws(c, ntok, ws);
    cudaStream_t st = S(s);
    cudaMemsetAsync(w.err, 0, 4, st);
    rc = ck_moe_route(c, x, ntok, rw, bias, w.logits, ids, wts, w.route, route_ws(c, ntok, nullptr).total, s);
    if (rc) return rc;
    const uint32_t A = ntok * c->nsel, R = A + c->n_shared * ntok;
    rc = ck_moe_permute(ids, wts, x, ntok, c->nsel, c->n_experts, c->n_shared, c->hidden, c->mode == 4, w.xp, w.row_w,
                        w.pair_pos, counts, w.tiles, w.ntiles, w.perm_ws, s);
    if (rc) return rc;
    const uint32_t mt = ck_moe_max_tiles(ntok, c->nsel, c->n_experts, c->n_shared);
    const uint64_t stride = (uint64_t)c->inter * c->hidden / 256 * 144;
    // every tile holds at most ntok tokens (a token picks an expert once; the shared tiles take the
    // ntok tokens), and at most CK_MOE_FEW_TOKENS in a decode-sized batch: there the expert weights
    // stream through the grouped matvec
    const uint32_t bound = ntok <= CK_MOE_DECODE_TOKENS ? (ntok < CK_MOE_FEW_TOKENS ? ntok : CK_MOE_FEW_TOKENS) : 0;
    rc = ck_moe_expert_gemm_bounded(1, wg, wu, sg, su, stride, c->n_experts, c->n_shared, w.xp, A + ntok, w.h, R,
                                    w.row_w, w.tiles, w.ntiles, mt, c->inter, c->hidden, 0, bound, w.err, s);
    if (rc) return rc;
    rc = ck_moe_expert_gemm_bounded(0, wd, nullptr, sd, nullptr, stride, c->n_experts, c->n_shared, w.h, R, w.y, R,
                                    nullptr, w.tiles, w.ntiles, mt, c->hidden, c->inter, 1, bound, w.err, s);
    if (rc) return rc;
    return ck_moe_combine(w.y, ids, wts, w.pair_pos, ntok, c->nsel, c->n_shared, c->hidden, c->mode == 3, out, nullptr,
                          s);
}

// Reads the device error word of a layer's workspace (synchronizes the stream).
int ck_moe_layer_status(const ck_moe_config *c, uint32_t ntok, const void *ws, void *s) {
    if (check_cfg(c) || !ws) return fail(CK_EARG, "ck_moe_layer_status");
    MoeWs w = moe_ws(c, ntok, const_cast<void *>(ws));
    int e = 0;
    cudaError_t r = cudaMemcpyAsync(&e, w.err, 4, cudaMemcpyDeviceToHost, S(s));
    if (r == cudaSuccess) r = cudaStreamSynchronize(S(s));
    if (r != cudaSuccess) return fail((int)r, "ck_moe_layer_status");
    if (e) {
        snprintf(g_err, sizeof(g_err), "ck_moe_layer_bf16: device wait timed out (role code %d)", e);
        return CK_ETIMEOUT;
    }
    return 0;
}

}  // extern "C"

// ----------------------------------------------------------------------------- no-allocation GEMM
// ck_q4k_gemm_bf16 takes its scratch (the token-tile table, the table's length and the device
// error word) from a caller workspace.  Some callers cannot provide one: a host runtime that keeps
// its own arenas and has no CUDA-aware allocator (the reference's C runtime is one), a serving
// loop that must not allocate between requests, or code that runs while holding a lock the
// allocator may also take.  ck_q4k_gemm_bf16_noalloc keeps that scratch in one fixed array in
// device memory instead, sized for CK_Q4K_GEMM_NOALLOC_MAX_TOKENS tokens (about 65 KB), so no call
// allocates: no cudaMalloc, no cudaFree, no allocating library call.
//
// The array is shared by every call on a device and keeps whatever the last call left in it; each
// call rewrites the tile table and its length and clears the error word before its kernels run.
// Two calls in flight at the same time on one device (different streams, or host threads) race on
// it and must be serialized by the caller.
namespace {
constexpr size_t kNoallocTileBytes = ((size_t)CK_Q4K_GEMM_NOALLOC_MAX_TOKENS / 16 + 2) * 16;
constexpr size_t kNoallocTileRegion = (kNoallocTileBytes + 255) & ~(size_t)255;
constexpr size_t kNoallocBytes = kNoallocTileRegion + 256 + 256;  // + table length + error word
constexpr int kNoallocMaxDevices = 64;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoallocBytes];

std::mutex g_noalloc_mu;
void *g_noalloc_ptr[kNoallocMaxDevices];

// The array's device address on the current device, looked up once per device (the first call on
// a device does this; it may load the module, so make that first call before any stream capture).
int noalloc_scratch(void **out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    if (dev < 0 || dev >= kNoallocMaxDevices) return CK_ENODEV;
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return (int)e;
        g_noalloc_ptr[dev] = p;
    }
    *out = g_noalloc_ptr[dev];
    return 0;
}
}  // namespace

extern "C" int ck_q4k_gemm_bf16_noalloc(const void *qb, const void *x, void *y, uint32_t rows, uint32_t cols,
                                        uint32_t ntok, void *s) {
    if (ntok > CK_Q4K_GEMM_NOALLOC_MAX_TOKENS) {
        static thread_local char what[160];
        snprintf(what, sizeof(what), "ck_q4k_gemm_bf16_noalloc: %u tokens, the fixed scratch holds at most %u",
                 ntok, (unsigned)CK_Q4K_GEMM_NOALLOC_MAX_TOKENS);
        return fail(CK_ESHAPE, what);
    }
    // the set-up comes before the pointer check, so that a warm-up call with ntok == 0 (null
    // pointers allowed) looks the array up outside any stream capture
    void *base = nullptr;
    int rc = noalloc_scratch(&base);
    if (rc) return fail(rc, "ck_q4k_gemm_bf16_noalloc scratch address");
    if (ntok == 0) return 0;
    if (!qb || !x || !y) return fail(CK_EARG, "ck_q4k_gemm_bf16_noalloc");
    uint8_t *b = (uint8_t *)base;
    int4 *tiles = (int4 *)b;
    int32_t *ntiles = (int32_t *)(b + kNoallocTileRegion);
    int *err = (int *)(b + kNoallocTileRegion + 256);
    cudaError_t e = cudaMemsetAsync(err, 0, 4, S(s));  // the one field that must start at zero
    if (e != cudaSuccess) return fail((int)e, "ck_q4k_gemm_bf16_noalloc");
    rc = ck::launch_single_tiles(tiles, ntiles, ntok, ck::GEMM_TILE_TOKENS, S(s));
    if (rc) return fail(rc, "ck_q4k_gemm_bf16_noalloc tiles");
    ck::GemmParams p = {};
    p.w0 = (const uint8_t *)qb;
    p.x = x;
    p.x_rows = ntok;
    p.out = y;
    p.out_rows = ntok;
    p.tiles = tiles;
    p.ntiles = ntiles;
    p.max_tiles = (uint32_t)(ntok / 16 + 2);
    p.n_routed = 1;
    // up to 4 tokens the table is one tile of ntok: the weights stream through the few-token
    // tensor-core matvec instead of the dequantizing GEMM (11008 x 4096: 19 / 21 / 28 us at 1 / 2 /
    // 4 tokens against the GEMM's 35-39; at 8 tokens the GEMM is ahead)
    p.max_tile_tok = ntok <= 4 ? ntok : 0;
    p.N = rows;
    p.K = cols;
    p.err = err;
    return fail(ck::launch_gemm_q4k(p, S(s)), "ck_q4k_gemm_bf16_noalloc");
}

// Reads the error word the last ck_q4k_gemm_bf16_noalloc call on the current device left in the
// fixed scratch (synchronizes `stream`).  It shares the scratch's rule: a call still in flight on
// another stream may rewrite the word.
extern "C" int ck_q4k_gemm_bf16_noalloc_status(void *s) {
    void *base = nullptr;
    int rc = noalloc_scratch(&base);
    if (rc) return fail(rc, "ck_q4k_gemm_bf16_noalloc_status scratch address");
    int e = 0;
    cudaError_t r = cudaMemcpyAsync(&e, (uint8_t *)base + kNoallocTileRegion + 256, 4, cudaMemcpyDeviceToHost, S(s));
    if (r == cudaSuccess) r = cudaStreamSynchronize(S(s));
    if (r != cudaSuccess) return fail((int)r, "ck_q4k_gemm_bf16_noalloc_status");
    if (e) {
        snprintf(g_err, sizeof(g_err), "ck_q4k_gemm_bf16_noalloc: device wait timed out (role code %d)", e);
        return CK_ETIMEOUT;
    }
    return 0;
}
