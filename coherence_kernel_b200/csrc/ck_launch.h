// ck_launch.h -- internal launcher declarations shared by the kernel files and the C-ABI layer.
// Launchers return 0 on success, a positive cudaError_t, or one of the negative CK_ERR_* codes.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#define CK_ERR_SHAPE (-2)    // a size the kernel does not support (stated in the entry point's doc)
#define CK_ERR_ARG (-3)      // a null pointer or an out-of-range argument
#define CK_ERR_TIMEOUT (-4)  // a device-side bounded wait gave up (the kernel returned early)
#define CK_ERR_NODEV (-5)    // no CUDA device, or the driver entry point is unavailable

namespace ck {

int launch_q80_dequant(const uint8_t *qb, float *w, uint64_t off, uint64_t n, cudaStream_t s);
int launch_q4k_dequant(const uint8_t *qb, float *w, uint64_t off, uint64_t n, cudaStream_t s);
int launch_q4k_dequant_bf16(const uint8_t *qb, void *w, uint64_t off, uint64_t n, cudaStream_t s);
int launch_matvec_ordered(int kind, const uint8_t *qb, const float *x, float *y, uint32_t rows, uint32_t cols,
                          cudaStream_t s);
int launch_q4k_matvec_group(uint32_t ng, const uint8_t *const *qb, const float *x, float *const *y, uint32_t rows,
                            uint32_t cols, uint32_t ntok, cudaStream_t s);
int launch_q4k_matvec(const uint8_t *qb, const float *x, float *y, uint32_t rows, uint32_t cols, uint32_t ntok,
                      cudaStream_t s);
int launch_q80_matvec(const uint8_t *qb, const float *x, float *y, uint32_t rows, uint32_t cols, cudaStream_t s);
// Q6_K (q6k_kernels.cu): exact dequant, the attestant-order matvec, its column-split form, and the
// decode / batched matvec (ntok tokens, token-major x and y)
int launch_q6k_dequant(const uint8_t *qb, float *w, uint64_t off, uint64_t n, cudaStream_t s);
int launch_q6k_ordered(const uint8_t *qb, const float *x, float *y, uint32_t rows, uint32_t cols, cudaStream_t s);
int launch_q6k_part(const uint8_t *qb, const float *x, float *part, uint32_t rows, uint32_t cols, uint32_t parts,
                    cudaStream_t s);
int launch_q6k_matvec(const uint8_t *qb, const float *x, float *y, uint32_t rows, uint32_t cols, uint32_t ntok,
                      cudaStream_t s);
// HBM-streaming decode matvec (gemv_stream.cu): kind 12 = Q4_K, 8 = Q8_0; cols % 256 == 0,
// cols <= 8192, weights and x 16-byte aligned
bool gemv_stream_ok(const void *qb, const float *x, uint32_t cols);
int launch_gemv_stream(int kind, const uint8_t *qb, const float *x, float *y, uint32_t rows, uint32_t cols,
                       cudaStream_t s);
// tensor-core Q4_K decode matvec (gemv_tc.cu): cols % 256 == 0, weights and x 16-byte aligned
bool gemv_tc_ok(const void *qb, const float *x, uint32_t rows, uint32_t cols);
int launch_gemv_tc(const uint8_t *qb, const float *x, float *y, uint32_t rows, uint32_t cols, cudaStream_t s);
// up to 4 matrices of one shape against the same x in one launch (each y as its single launch)
int launch_gemv_tc_group(uint32_t ng, const uint8_t *const *qb, const float *x, float *const *y, uint32_t rows,
                         uint32_t cols, cudaStream_t s);
int launch_f16_matvec(const uint16_t *w, const float *x, float *y, uint32_t rows, uint32_t cols, cudaStream_t s);
int launch_scale(const float *x, float *y, float a, uint32_t n, cudaStream_t s);
int launch_axpy(const float *x, float *y, float a, uint32_t n, cudaStream_t s);
int launch_swiglu(const float *g, const float *u, float *out, uint32_t n, float w, float lim, cudaStream_t s);

// routers (router_kernels.cu)
int launch_route_softmax_tokens(const float *logits, uint32_t *ids, float *wts, uint32_t ne, uint32_t nsel,
                                uint32_t ntok, int renorm, cudaStream_t s);
int launch_route_dsv4_tokens(const float *logits, const float *bias, uint32_t *ids, float *wts, uint32_t ne,
                             uint32_t nused, float wscale, uint32_t ntok, cudaStream_t s);
int launch_router_logits(const uint16_t *x_bf16, const float *w, float *logits, uint32_t ntok, uint32_t ne,
                         uint32_t hidden, cudaStream_t s);
struct RouteParams {
    uint32_t ntok, ne, nsel, hidden;
    uint32_t mode;         // 3: softmax top-k (no renorm); 4: sigmoid + bias, group-limited
    uint32_t ngroups, topk_groups;
    float wscale;          // mode 4 weight scale
    float tau;             // decision margin below which a token is re-routed exactly in fp64
};
// router logits for at most 128 tokens (compensated sums over the fp32 router) in fp32 and fp64, with
// sum |w x| per logit; ntok > 128 returns CK_ERR_SHAPE
int launch_router_logits_few(const uint16_t *x, const float *w, float *L, double *Ld, float *sabs, uint32_t *flag_count, uint32_t T,
                             uint32_t E, uint32_t H, cudaStream_t s);
// the fast selection over fp64 logits (the decode-batch form); its margin scales with sabs
int launch_route_select_d(const double *L, const float *sabs, const float *bias, int32_t *ids, float *wts,
                          uint32_t *flag_list, uint32_t *flag_count, const RouteParams &p, cudaStream_t s);
// the fast selection over the tensor-core logits; `planes` holds nplanes (<= 7) more K-chunk partial
// planes of [ntok, ne] to add to `logits` in chunk order first (the sums are written to `logits`)
int launch_route_select(float *logits, const float *planes, int nplanes, const float *bias, int32_t *ids, float *wts,
                        uint32_t *flag_list, uint32_t *flag_count, const RouteParams &p, cudaStream_t s);
// scratch: fp64 [ntok, ne] (the exact logits of the flagged tokens)
// out fp64 [*flag_count, ne]: the right-fold logits of the listed tokens (at most 256 experts,
// hidden % 32 == 0); w64: scratch for the router in fp64, ne * hidden doubles; max_count: a bound
// on *flag_count known to the host (the batch's tokens)
int launch_exact_logits(const uint16_t *x_bf16, const float *w, const uint32_t *flag_list, const uint32_t *flag_count,
                        double *out, double *w64, uint32_t ne, uint32_t hidden, uint32_t max_count, cudaStream_t s);
int launch_route_exact(const uint16_t *x_bf16, const float *w, const float *bias, int32_t *ids, float *wts,
                       const uint32_t *flag_list, const uint32_t *flag_count, double *scratch, double *w64,
                       const RouteParams &p, cudaStream_t s);

// The grouped GEMM's largest token tile: its accumulators (gate and up, or two buffers) and its
// tensor-memory A stages share the 512 TMEM columns.  Every token-tile table is built with it.
constexpr uint32_t GEMM_TILE_TOKENS = 192;

// MoE permute / combine (moe_kernels.cu)
struct PermuteParams {
    uint32_t ntok, nsel, n_experts, n_shared, hidden;
    uint32_t bn;           // token tile of the grouped GEMM
    uint32_t weight_in_mid;  // 1: the route weight scales the SwiGLU product (dsv4); 0: combine
};
size_t permute_workspace_bytes(const PermuteParams &p);
int launch_permute(const int32_t *ids, const float *wts, const uint16_t *x_bf16, uint16_t *xp, float *row_w,
                   int32_t *pair_pos, int32_t *counts, int4 *tiles, int32_t *ntiles, void *workspace,
                   const PermuteParams &p, cudaStream_t s);
int launch_single_tiles(int4 *tiles, int32_t *ntiles, uint32_t ntok, uint32_t bn, cudaStream_t s);
int launch_ep_plan(const int32_t *ids, const float *wts, uint32_t ntok, uint32_t nsel, uint32_t n_experts,
                   uint32_t world, int32_t *counts, long long *sizes, int32_t *send_tok, int32_t *meta,
                   int32_t *ret_pos, cudaStream_t s);
int launch_gather_rows(const void *src, const int32_t *idx, void *dst, uint32_t nrows, uint32_t row_bytes,
                       cudaStream_t s);
int launch_combine(const uint16_t *y, const int32_t *ids, const float *wts, const int32_t *pair_pos, uint16_t *out,
                   float *out_f32, const PermuteParams &p, int order_by_expert, cudaStream_t s);

// tcgen05 grouped Q4_K GEMM (gemm_tc.cu)
struct GemmParams {
    const uint8_t *w0;       // routed weights (gate, or the only matrix), expert g at w0 + g*w_stride
    const uint8_t *w1;       // routed up weights (dual mode), same stride
    const uint8_t *s0;       // shared-expert weights, expert s at s0 + s*w_stride
    const uint8_t *s1;
    uint64_t w_stride;       // bytes per expert matrix
    const void *x;           // bf16 activations [x_rows, K], rows addressed by the tile table
    uint32_t x_rows;
    void *out;               // bf16 output [out_rows, N]
    uint32_t out_rows;
    const float *row_w;      // per output row weight (dual mode; null = 1)
    const int4 *tiles;       // (group, x_row, out_row, ntok) per token tile
    const int32_t *ntiles;   // device-side tile count
    uint32_t max_tiles;
    uint32_t n_routed;       // groups >= n_routed use the shared weights
    uint32_t n_shared;       // how many shared matrices s0/s1 hold
    uint32_t N, K;           // output features (weight rows), reduction length
    int dual;                // 1: out = silu(x.W0) * (x.W1) * row_w ; 0: out = x.W0
    int xrow_is_orow;        // 1: read X at the tile's output row (the down projection over H)
    int *err;                // device error word (bounded waits)
    // dense form (router logits): A is bf16 [N, K] read by TMA, X is walked every kx columns
    // (A = [W1 | W2 | W3], the three bf16 terms of an fp32 matrix), the output is fp32 [rows, N]
    const void *a_dense;
    uint32_t kx;
    float *out_f32;
    // ksplit > 1: every K-chunk accumulator of the dense form is a unit of its own; chunk 0 goes to
    // out_f32 and chunk c > 0 to plane c - 1 of out_planes ([DENSE_ACC - 1][out_rows, N]), for the
    // reader to add in chunk order (the sums the unsplit form's epilogue makes)
    float *out_planes;
    uint32_t ksplit;
    // a bound on the tokens of every tile (0: none known); 1..8 runs the few-token grouped matvec
    // (moe_gemv.cu) where its shape rules hold
    uint32_t max_tile_tok;
    // single form only: output row o is stored at the bf16 row whose address is row_dst[o] instead of
    // at out + o * N -- rows may sit in another GPU's memory (the expert-parallel return written by
    // the down projection's epilogue); every address 16-byte aligned, N % 8 == 0
    const unsigned long long *row_dst;
};
int launch_gemm_q4k(const GemmParams &p, cudaStream_t s);
bool gemv_moe_ok(const GemmParams &p);
int launch_gemv_moe(const GemmParams &p, cudaStream_t s);
int launch_gemm_dense(const GemmParams &p, cudaStream_t s);
// fp32 [rows, k] -> bf16 [rows, 3k]: w = w1 + w2 + w3 with each term the bf16 rounding of the
// remainder (exact to about 2^-24 relative)
int launch_split_bf16x3(const float *w, uint16_t *out, uint32_t rows, uint32_t k, cudaStream_t s);

}  // namespace ck
