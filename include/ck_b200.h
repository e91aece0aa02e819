/* ck_b200.h -- C ABI of the B200 (sm_100a) kernels for coherence-kernel's quantized path.
 *
 * Plain pointers and sizes only.  Every pointer argument named *_dev is CUDA device memory (or
 * host memory the device can address); `stream` is a cudaStream_t (NULL = the legacy default
 * stream).  Every entry point enqueues work and returns without waiting.  Return value: 0 on
 * success, a positive cudaError_t, or a negative CK_E* code; ck_last_error() names the failure.
 *
 * Layouts are the reference's: GGUF block_q8_0 (34 bytes / 32 weights) and block_q4_K (144 bytes
 * / 256 weights) read by FLAT weight index, so row r of a rows x cols tensor is the flat range
 * [r*cols, (r+1)*cols) and may straddle blocks (form/form-stdlib/q4k-msl.fk:73-86,
 * q8-0-msl.fk:53-70).  Token-major activations x[t*cols + j] and outputs y[t*rows + r]
 * (form/form-stdlib/qk-matmul-batch.fk:117-121).
 */
#ifndef CK_B200_H
#define CK_B200_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CK_OK 0
#define CK_ESHAPE (-2)   /* a size outside the entry point's stated limits */
#define CK_EARG (-3)     /* a null or misaligned pointer, or an out-of-range argument */
#define CK_ETIMEOUT (-4) /* a device-side bounded wait gave up; the kernel returned early */
#define CK_ENODEV (-5)   /* no CUDA device / driver entry point */

const char *ck_last_error(void);
/* 1 when the library was built for sm_100a and a device is present */
int ck_device_ok(void);

/* ---- dequant (replaces form_q8_0_dequant_f32, q8-0-msl.fk:92-95; form_q4k_dequant_f32,
 *      q4k-msl.fk:104-107): w[i] = weight(off + i), i < n */
int ck_q8_0_dequant_f32(const void *qb_dev, float *w_dev, uint64_t off, uint64_t n, void *stream);
int ck_q4k_dequant_f32(const void *qb_dev, float *w_dev, uint64_t off, uint64_t n, void *stream);
int ck_q4k_dequant_bf16(const void *qb_dev, void *w_bf16_dev, uint64_t off, uint64_t n, void *stream);

/* ---- decode matvec, fp32 x / y (replaces form_q8_0_matvec_f32 / _lane / wide,
 *      q8-0-msl.fk:100-123; form_q4k_matvec_f32, q4k-msl.fk:111-114, and the hoist / lane / slot
 *      variants, qk-matvec-lane.fk:218-238, qk-matvec-slot.fk:163-235).
 *      Q8_0: cols % 32 == 0 (fastest at cols % 256 == 0).  Q4_K: cols % 64 == 0. */
int ck_q8_0_matvec_f32(const void *qb_dev, const float *x_dev, float *y_dev, uint32_t rows, uint32_t cols,
                       void *stream);
int ck_q4k_matvec_f32(const void *qb_dev, const float *x_dev, float *y_dev, uint32_t rows, uint32_t cols,
                      void *stream);
/* The attestant association: one thread per row, j counting down, acc = w*x + acc with no fused
 * multiply-add (q8-0-msl.fk:100-103, q4k-msl.fk:111-114, q6k-msl.fk:118-123).  ggml_type 8 = Q8_0,
 * 12 = Q4_K, 14 = Q6_K. */
int ck_matvec_ordered_f32(int ggml_type, const void *qb_dev, const float *x_dev, float *y_dev, uint32_t rows,
                          uint32_t cols, void *stream);
/* ---- GGUF Q6_K (210 bytes / 256 weights: ql[128], qh[64], 16 signed int8 scales, f16 d), read by
 * flat weight index like the others (form/form-stdlib/q6k-msl.fk:62-81).  rows*cols % 256 == 0.
 * Dequant replaces form_q6k_dequant_f32 (q6k-msl.fk:109-113) and is bit-exact; the matvec replaces
 * form_q6k_matvec_lane_f32 / _slot_f32 (qk-matvec-lane.fk:232-238, qk-matvec-slot.fk:163-166) --
 * for the attestant association (form_q6k_matvec_f32) call ck_matvec_ordered_f32 with type 14;
 * the batched form replaces form_q6k_matmul_batch_f32 (qk-matmul-batch.fk); the split form
 * replaces form_q6k_matvec_part_f32 / _hoist_f32 (qk-matvec-split.fk:114-121): part[r*parts + p] =
 * the right fold of row r over column chunk p (chunk = ceil(cols / parts)). */
int ck_q6k_dequant_f32(const void *qb_dev, float *w_dev, uint64_t off, uint64_t n, void *stream);
int ck_q6k_matvec_f32(const void *qb_dev, const float *x_dev, float *y_dev, uint32_t rows, uint32_t cols,
                      void *stream);
int ck_q6k_matmul_batch_f32(const void *qb_dev, const float *x_dev, float *y_dev, uint32_t rows, uint32_t cols,
                            uint32_t ntok, void *stream);
int ck_q6k_matvec_part_f32(const void *qb_dev, const float *x_dev, float *part_dev, uint32_t rows, uint32_t cols,
                           uint32_t parts, void *stream);
/* Batched matvec over ntok tokens, fp32 (replaces form_q4k_matmul_batch_f32,
 * qk-matmul-batch.fk:206-217): y[t*rows + r] = sum_j W[r, j] x[t*cols + j].  cols % 64 == 0. */
/* 1 to 4 Q4_K matrices of one shape against the same x (a decode step's Q/K/V projections):
 * y_list[g] = qb_list[g] . x.  qb_list and y_list are host arrays of device pointers.  Where one such
 * matvec takes the tensor-core kernel, all of them run in one launch, each y bit-identical to its
 * own ck_q4k_matvec_f32; otherwise they run one after another. */
int ck_q4k_matvec_f32_group(uint32_t n, const void *const *qb_list, const float *x_dev, float *const *y_list,
                            uint32_t rows, uint32_t cols, void *stream);
int ck_q4k_matmul_batch_f32(const void *qb_dev, const float *x_dev, float *y_dev, uint32_t rows, uint32_t cols,
                            uint32_t ntok, void *stream);

/* ---- prefill GEMM on the tensor cores: Y[t, r] = sum_j X[t, j] W[r, j], X bf16 [ntok, cols],
 *      Y bf16 [ntok, rows], fp32 accumulation (the bf16-MMA form of form_q4k_matmul_batch_f32).
 *      cols % 64 == 0, rows*cols % 256 == 0.  workspace: ck_q4k_gemm_workspace_bytes(ntok). */
size_t ck_q4k_gemm_workspace_bytes(uint32_t ntok);
int ck_q4k_gemm_bf16(const void *qb_dev, const void *x_bf16_dev, void *y_bf16_dev, uint32_t rows, uint32_t cols,
                     uint32_t ntok, void *workspace_dev, size_t workspace_bytes, void *stream);
/* After a ck_q4k_gemm_bf16 call with this workspace and ntok: synchronizes `stream` and returns
 * CK_ETIMEOUT when a device-side wait of the GEMM gave up (y is then not valid), else 0. */
int ck_q4k_gemm_status(uint32_t ntok, const void *workspace_dev, void *stream);

/* The same GEMM for callers that cannot allocate or hand over a workspace (a host runtime with its
 * own arenas and no CUDA-aware allocator, a serving loop that must not allocate per request).  No
 * counterpart in the reference, whose matmul kernels take no scratch.  The scratch lives in one
 * fixed array in device memory (about 65 KB), so ntok <= CK_Q4K_GEMM_NOALLOC_MAX_TOKENS; larger
 * ntok fails with CK_ESHAPE.  The first call on a device looks the array up (it may load the
 * module): make it before stream capture -- a call with ntok 0 does only that, and accepts null
 * pointers.  The address is cached per device for the life of the process, so cudaDeviceReset is
 * not supported between calls.  Every call on a device shares the array and leaves its contents
 * behind; calls that overlap in time on one device race on it and must be serialized by the
 * caller. */
#define CK_Q4K_GEMM_NOALLOC_MAX_TOKENS 65536u
int ck_q4k_gemm_bf16_noalloc(const void *qb_dev, const void *x_bf16_dev, void *y_bf16_dev, uint32_t rows,
                             uint32_t cols, uint32_t ntok, void *stream);
/* Synchronizes `stream` and returns CK_ETIMEOUT when a device-side wait of the last
 * ck_q4k_gemm_bf16_noalloc call on the current device gave up (its y is then not valid), else 0.
 * The error word lives in the same shared array, so the serialization rule above applies. */
int ck_q4k_gemm_bf16_noalloc_status(void *stream);

/* ---- small kernels of the reference's MoE decode (moe-msl.fk:114-140, dsv4-moe-msl.fk:87-88,
 *      dsv4-router-msl.fk:103-106, moe-route-wide-msl.fk) -- one routing per token, ntok tokens */
int ck_f16_matvec_f32(const void *w_f16_dev, const float *x_dev, float *y_dev, uint32_t rows, uint32_t cols,
                      void *stream);
int ck_route_softmax_f32(const float *logits_dev, uint32_t *ids_dev, float *wts_dev, uint32_t ne, uint32_t nsel,
                         uint32_t ntok, int renorm, void *stream);
int ck_route_dsv4_f32(const float *logits_dev, const float *bias_dev, uint32_t *ids_dev, float *wts_dev,
                      uint32_t ne, uint32_t nused, float wscale, uint32_t ntok, void *stream);
int ck_scale_f32(const float *x_dev, float *y_dev, float a, uint32_t n, void *stream);
int ck_axpy_f32(const float *x_dev, float *y_dev, float a, uint32_t n, void *stream);
int ck_swiglu_f32(const float *gate_dev, const float *up_dev, float *out_dev, uint32_t n, float w, float lim,
                  void *stream);

/* ---- the batched MoE layer (new: the reference routes and combines one token at a time) ----
 * mode 3: softmax router, top-nsel, no renormalization, combine in ascending expert index with
 *         the weight applied at the combine (moe-gate.fk:22-37), n_shared shared experts added.
 * mode 4: sigmoid + bias, group-limited (ngroups, topk_groups), top-nsel, weights renormalized x
 *         wscale (dsv4-forward.fk:105-111), applied inside the expert (dsv4-mid), combine in
 *         selection-list order, shared expert(s) added.
 * Experts: Q4_K gate/up [inter x hidden] and down [hidden x inter], expert e at byte offset
 * e * (inter*hidden/256*144) of each array; shared experts likewise.  router_w fp32 [ne, hidden];
 * bias fp32 [ne] (mode 4).  x bf16 [ntok, hidden].  Outputs: ids int32 [ntok, nsel], wts fp32
 * [ntok, nsel] (the reference's list order), counts int32 [ne], out bf16 [ntok, hidden].
 * Limits: ne <= 256, nsel <= 16, hidden % 64 == 0, inter % 64 == 0, ngroups <= 32.
 * tau: a token whose decision margin (smallest gap between a chosen and a rejected candidate's
 * fp32 score) is below tau is routed again in fp64 in the reference's own fold order. */
typedef struct {
    uint32_t hidden, inter, n_experts, n_shared, nsel, mode, ngroups, topk_groups;
    float wscale, tau;
} ck_moe_config;

size_t ck_moe_workspace_bytes(const ck_moe_config *cfg, uint32_t ntok);
int ck_moe_layer_bf16(const ck_moe_config *cfg, const void *x_bf16_dev, uint32_t ntok, const void *w_gate_dev,
                      const void *w_up_dev, const void *w_down_dev, const void *s_gate_dev, const void *s_up_dev,
                      const void *s_down_dev, const float *router_w_dev, const float *bias_dev, int32_t *ids_dev,
                      float *wts_dev, int32_t *counts_dev, void *out_bf16_dev, void *workspace_dev,
                      size_t workspace_bytes, void *stream);

/* After a layer has run: synchronizes `stream` and returns CK_ETIMEOUT when a device-side wait in
 * the grouped GEMM gave up (the layer's output is then not valid), else 0. */
int ck_moe_layer_status(const ck_moe_config *cfg, uint32_t ntok, const void *workspace_dev, void *stream);

/* the layer's steps, for callers that place an all-to-all between them (expert parallelism).
 * ck_moe_route: router logits on the tensor cores (the fp32 router split into three bf16 terms),
 * selection, and the exact fp64 re-route of near-tie tokens; route_ws sized by
 * ck_moe_route_workspace_bytes.  ck_moe_route_flagged synchronizes and answers how many tokens
 * the last route re-routed exactly. */
size_t ck_moe_route_workspace_bytes(const ck_moe_config *cfg, uint32_t ntok);
int ck_moe_route(const ck_moe_config *cfg, const void *x_bf16_dev, uint32_t ntok, const float *router_w_dev,
                 const float *bias_dev, float *logits_dev, int32_t *ids_dev, float *wts_dev, void *route_ws_dev,
                 size_t route_ws_bytes, void *stream);
int ck_moe_route_flagged(const ck_moe_config *cfg, uint32_t ntok, const void *route_ws_dev, void *stream);
/* The reference's router logits for a list of tokens: out[f * n_experts + e] = tb-dot's right fold
 * (transformer-block.fk:25-26) of router row e with token tokens[f]'s bf16 activations, in fp64 and
 * bit-identical to the reference, for f < *count_dev (device memory, read by the kernels).  The
 * route's exact re-route runs these kernels on its near-tie tokens.  router_f64_dev is scratch
 * (n_experts * hidden doubles) that receives the router in fp64.  n_experts <= 256,
 * hidden % 32 == 0, x, the router and the scratch 16-byte aligned. */
int ck_router_exact_logits(const void *x_bf16_dev, const float *router_w_dev, const uint32_t *tokens_dev,
                           const uint32_t *count_dev, uint32_t n_experts, uint32_t hidden, double *out_dev,
                           double *router_f64_dev, void *stream);
size_t ck_moe_permute_workspace_bytes(uint32_t ntok, uint32_t nsel, uint32_t n_experts);
uint32_t ck_moe_max_tiles(uint32_t ntok, uint32_t nsel, uint32_t n_experts, uint32_t n_shared);
int ck_moe_permute(const int32_t *ids_dev, const float *wts_dev, const void *x_bf16_dev, uint32_t ntok,
                   uint32_t nsel, uint32_t n_experts, uint32_t n_shared, uint32_t hidden, int weight_in_mid,
                   void *xp_bf16_dev, float *row_w_dev, int32_t *pair_pos_dev, int32_t *counts_dev,
                   void *tiles_dev, int32_t *ntiles_dev, void *workspace_dev, void *stream);
int ck_moe_expert_gemm(int dual, const void *w0_dev, const void *w1_dev, const void *s0_dev, const void *s1_dev,
                       uint64_t w_stride, uint32_t n_routed, uint32_t n_shared, const void *x_bf16_dev, uint32_t x_rows,
                       void *out_bf16_dev, uint32_t out_rows, const float *row_w_dev, const void *tiles_dev,
                       const int32_t *ntiles_dev, uint32_t max_tiles, uint32_t n, uint32_t k, int xrow_is_orow,
                       int *err_dev, void *stream);
/* ck_moe_expert_gemm with a bound on the tokens of every tile of the table (0: none known).  A bound
 * of 1..8 streams the expert weights through the few-token grouped matvec on the integer tensor
 * cores (where n % 128 == 0, k % 256 == 0 and the pointers are 16-byte aligned); the results agree
 * with the grouped GEMM's to its bf16 output rounding.  ck_moe_layer_bf16 passes
 * min(ntok, CK_MOE_FEW_TOKENS) when ntok <= CK_MOE_DECODE_TOKENS.  Up to 5 tokens a tile's
 * accumulators fit twice in tensor memory, so the matvec of one step overlaps the epilogue of the
 * step before; 6 to 8 tokens fit once. */
#define CK_MOE_FEW_TOKENS 5
/* batches of at most this many tokens are permuted into tiles of at most CK_MOE_FEW_TOKENS tokens
 * (ck_moe_permute, ck_moe_max_tiles) and their expert projections run the few-token matvec */
#define CK_MOE_DECODE_TOKENS 128
int ck_moe_expert_gemm_bounded(int dual, const void *w0_dev, const void *w1_dev, const void *s0_dev,
                               const void *s1_dev, uint64_t w_stride, uint32_t n_routed, uint32_t n_shared,
                               const void *x_bf16_dev, uint32_t x_rows, void *out_bf16_dev, uint32_t out_rows,
                               const float *row_w_dev, const void *tiles_dev, const int32_t *ntiles_dev,
                               uint32_t max_tiles, uint32_t n, uint32_t k, int xrow_is_orow,
                               uint32_t max_tile_tokens, int *err_dev, void *stream);
/* The single-matrix grouped GEMM of ck_moe_expert_gemm_bounded (dual = 0, the grouped-GEMM form only)
 * with output row o stored at the bf16 row whose device address is row_dst_dev[o] rather than in a
 * contiguous output: the rows may lie in other GPUs' memory mapped into this process.  No counterpart
 * in the reference (its MoE runs on one device): the expert-parallel layer's down projection writes
 * each (token, slot) row straight into the source rank's return buffer (row_dst from
 * ck_ep_peer_return_rows), so the return crosses NVLink while the GEMM runs.  n % 8 == 0 and every
 * address 16-byte aligned; out_rows bounds o. */
int ck_moe_expert_gemm_rows(const void *w0_dev, uint64_t w_stride, uint32_t n_routed, const void *x_bf16_dev,
                            uint32_t x_rows, const unsigned long long *row_dst_dev, uint32_t out_rows,
                            const void *tiles_dev, const int32_t *ntiles_dev, uint32_t max_tiles, uint32_t n,
                            uint32_t k, int xrow_is_orow, int *err_dev, void *stream);
int ck_moe_combine(const void *y_bf16_dev, const int32_t *ids_dev, const float *wts_dev, const int32_t *pair_pos_dev,
                   uint32_t ntok, uint32_t nsel, uint32_t n_shared, uint32_t hidden, int order_by_expert,
                   void *out_bf16_dev, float *out_f32_dev, void *stream);
/* the token-tile table of one matrix over ntok rows (group 0, rows in order), at most
 * ntok/16 + 2 entries of 4 int32 */
int ck_token_tiles(void *tiles_dev, int32_t *ntiles_dev, uint32_t ntok, void *stream);
/* the same table with tiles of at most tile_tokens tokens (1..8, or a multiple of 16 up to 192):
 * ceil(ntok / tile_tokens) entries.  Tiles of at most CK_MOE_FEW_TOKENS feed the few-token grouped
 * matvec (ck_moe_expert_gemm_bounded with that bound). */
int ck_token_tiles_n(void *tiles_dev, int32_t *ntiles_dev, uint32_t ntok, uint32_t tile_tokens, void *stream);
int ck_gather_rows(const void *src_dev, const int32_t *idx_dev, void *dst_dev, uint32_t nrows, uint32_t row_bytes,
                   void *stream);
/* Expert-parallel dispatch plan (no counterpart in the reference, whose MoE runs on one device).
 * Rank d of `world` owns experts [d*E/world, (d+1)*E/world).  From the routed ids/wts
 * [ntok, nsel] (one CTA, stream-ordered): counts [E] pairs per expert; sizes [world][2] int64 =
 * (rows, pairs) sent to each rank; send_tok [rows] the token of every dispatch row, one row per
 * (rank, token) with at least one of the token's experts there, in (rank, token) order; meta
 * [rows][2*nsel] int32 = the slots' local experts (-1 for slots owned elsewhere) then their
 * route weights as float bits (0 there); ret_pos [ntok*nsel] the row of every (token, slot)
 * pair in the return exchange (ranks in order, (token, slot) order inside a rank).  world <= 32,
 * nsel <= 16, E <= 1024, E % world == 0; send_tok/meta hold up to ntok*min(world, nsel) rows. */
int ck_ep_dispatch_plan(const int32_t *ids_dev, const float *wts_dev, uint32_t ntok, uint32_t nsel,
                        uint32_t n_experts, uint32_t world, int32_t *counts_dev, int64_t *sizes_dev,
                        int32_t *send_tok_dev, int32_t *meta_dev, int32_t *ret_pos_dev, void *stream);

/* ---- a device-resident decode step of a transformer block with an MoE feed-forward (no single
 * counterpart in the reference, whose decode token is ~400 separate host dispatches; its measured
 * seam cost is receipts/2026-07-22-ship-the-slot-map.md:135-145).  Per token, in one stream:
 *   a = rmsnorm(h, g_attn) (ln-rmsnorm, llama-numerics.fk:40-50); q = Wq a, k = Wk a, v = Wv a;
 *   h += Wo v (attention at a single position, whose output is v); b = bf16(rmsnorm(h, g_ffn));
 *   h += ck_moe_layer_bf16(b).
 * Wq/Wk/Wv/Wo are Q4_K [hidden x hidden]; g_* fp32 [hidden]; the MoE weights as for
 * ck_moe_layer_bf16 (moe.hidden == hidden).  h fp32 [ntok, hidden] is updated in place; q, k, v
 * are fp32 [ntok, hidden] outputs.  hidden % 256 == 0, ntok <= max_tokens.  All scratch comes from
 * the caller's workspace (ck_decode_step_workspace_bytes).  ck_decode_step_run issues the step;
 * ck_decode_step_capture records one run with these buffer addresses into a CUDA graph on a
 * non-default stream (make one ck_decode_step_run first: it loads the kernels), and
 * ck_decode_step_replay launches that graph -- the whole step as one launch. */
typedef struct {
    uint32_t hidden, max_tokens;
    float eps;
    ck_moe_config moe;
} ck_decode_config;
typedef struct ck_decode_step ck_decode_step;
size_t ck_decode_step_workspace_bytes(const ck_decode_config *cfg);
/* NULL on a bad configuration, a short workspace or a missing weight */
ck_decode_step *ck_decode_step_create(const ck_decode_config *cfg, const void *wq_dev, const void *wk_dev,
                                      const void *wv_dev, const void *wo_dev, const float *g_attn_dev,
                                      const float *g_ffn_dev, const void *w_gate_dev, const void *w_up_dev,
                                      const void *w_down_dev, const void *s_gate_dev, const void *s_up_dev,
                                      const void *s_down_dev, const float *router_w_dev, const float *bias_dev,
                                      void *workspace_dev, size_t workspace_bytes);
int ck_decode_step_run(ck_decode_step *step, float *h_dev, float *q_dev, float *k_dev, float *v_dev, uint32_t ntok,
                       void *stream);
int ck_decode_step_capture(ck_decode_step *step, float *h_dev, float *q_dev, float *k_dev, float *v_dev,
                           uint32_t ntok, void *stream);
int ck_decode_step_replay(ck_decode_step *step, void *stream);
/* synchronizes; CK_ETIMEOUT when a device wait of the step's MoE layer over ntok tokens gave up */
int ck_decode_step_status(ck_decode_step *step, uint32_t ntok, void *stream);
void ck_decode_step_destroy(ck_decode_step *step);

/* ---- expert parallelism over NVLink peer memory (no counterpart in the reference, whose MoE runs on
 * one device).  Each rank owns a zeroed device arena (ck_ep_arena_alloc) that its peers map with CUDA
 * IPC (ck_ipc_get_handle / ck_ipc_open_handle).  ck_ep_peers names, for this rank, where its stores
 * go in every peer's arena and where its own flags, step counter and error word are.  One forward:
 * ck_ep_peer_begin (step += 1), ck_ep_dispatch_plan, ck_ep_peer_dispatch (every dispatch row into
 * region `rank` of its destination; the unused rows of that region get expert -1), signal / wait
 * (which = 0), the receiver's ck_moe_permute over world * cap rows and expert GEMMs,
 * ck_ep_peer_return (every computed (row, slot) pair into its source's return buffer at row
 * token * nsel + slot; or ck_ep_peer_return_rows before a down projection that stores its rows there
 * itself), signal / wait (which = 1), ck_moe_combine.  No host synchronization: the
 * step count is a device value, so a forward can be captured in a CUDA graph.  Every wait is
 * bounded; a timeout sets the error word (20 dispatch, 21 return) and the step's outputs are not
 * valid.  All ranks must run the same sequence of forwards. */
#define CK_EP_MAX_RANKS 32
typedef struct {
    uint32_t world, rank, cap, nsel, hidden, reserved;
    void *recv_x[CK_EP_MAX_RANKS];                 /* peer d's region for this rank: bf16 [cap, hidden] */
    int32_t *recv_ids[CK_EP_MAX_RANKS];            /* int32 [cap, nsel] local experts, -1 = none */
    float *recv_w[CK_EP_MAX_RANKS];                /* fp32 [cap, nsel] route weights */
    int32_t *recv_tok[CK_EP_MAX_RANKS];            /* int32 [cap] the source's token numbers */
    void *ret_y[CK_EP_MAX_RANKS];                  /* peer s's return buffer, bf16 rows t * nsel + k */
    unsigned long long *dflag[CK_EP_MAX_RANKS];    /* peer d's dispatch flag slot for this rank */
    unsigned long long *rflag[CK_EP_MAX_RANKS];    /* peer s's return flag slot for this rank */
    unsigned long long *my_dflags, *my_rflags;     /* this rank's flag arrays [world] */
    unsigned long long *ctr;                       /* this rank's step counter */
    int *err;                                      /* this rank's error word */
} ck_ep_peers;
int ck_ep_arena_alloc(size_t bytes, void **dev_ptr_out);
int ck_ep_arena_free(void *dev_ptr);
int ck_ipc_get_handle(const void *dev_ptr, void *handle_out /* 64 bytes */);
int ck_ipc_open_handle(const void *handle /* 64 bytes */, void **dev_ptr_out);
int ck_ipc_close(void *dev_ptr);
int ck_ep_peer_begin(const ck_ep_peers *peers, void *stream);
/* synchronizes; CK_ETIMEOUT when a wait (or an expert GEMM wait) of this rank gave up */
int ck_ep_peer_status(const ck_ep_peers *peers, void *stream);
int ck_ep_peer_dispatch(const ck_ep_peers *peers, const void *x_bf16_dev, const int32_t *send_tok_dev,
                        const int32_t *meta_dev, const int64_t *sizes_dev, uint32_t ntok, void *stream);
int ck_ep_peer_signal(const ck_ep_peers *peers, int which, void *stream);
int ck_ep_peer_wait(const ck_ep_peers *peers, int which, uint64_t limit_ns, void *stream);
int ck_ep_peer_return(const ck_ep_peers *peers, const void *y2_bf16_dev, const int32_t *pair_pos2_dev,
                      const int32_t *ids_own_dev, const int32_t *tok_own_dev, void *stream);
/* In place of ck_ep_peer_return when the down projection runs on the grouped GEMM: row_dst_dev
 * (world * cap * nsel entries, indexed by the permute's pair positions) receives, for every pair
 * with a local expert, the address of its row token * nsel + slot in its source's return buffer;
 * ck_moe_expert_gemm_rows over those rows then does the return from its epilogue. */
int ck_ep_peer_return_rows(const ck_ep_peers *peers, const int32_t *pair_pos2_dev, const int32_t *ids_own_dev,
                           const int32_t *tok_own_dev, unsigned long long *row_dst_dev, void *stream);

/* ---- one process, several GPUs (no counterpart in the reference): the same expert-parallel layer for
 * a host that owns the box's GPUs itself (the reference runtime with this carrier is one).  A group
 * of `world` member GPUs (devices[0] first) with peer access between them; every member holds
 * E / world experts, replicas of the router and shared expert(s), and room for `cap` tokens.
 * ck_ep_group_load copies the member shares from full weight arrays anywhere in device memory.
 * ck_ep_group_forward splits ntok <= world * cap tokens evenly over the members, runs the layer
 * over peer memory and gathers ids, weights, per-expert counts and out back; x / ids / wts /
 * counts / out live on devices[0] and `stream` is a stream of devices[0].  The host never waits;
 * ck_ep_group_status synchronizes and answers CK_ETIMEOUT when a member's device wait gave up. */
typedef struct ck_ep_group ck_ep_group;
ck_ep_group *ck_ep_group_create(const ck_moe_config *cfg, uint32_t world, const int *devices, uint32_t cap);
int ck_ep_group_load(ck_ep_group *group, const void *w_gate_dev, const void *w_up_dev, const void *w_down_dev,
                     const void *s_gate_dev, const void *s_up_dev, const void *s_down_dev, const float *router_w_dev,
                     const float *bias_dev);
int ck_ep_group_forward(ck_ep_group *group, const void *x_bf16_dev, uint32_t ntok, int32_t *ids_dev, float *wts_dev,
                        int32_t *counts_dev, void *out_bf16_dev, void *stream);
int ck_ep_group_status(ck_ep_group *group);
void ck_ep_group_destroy(ck_ep_group *group);

/* Failure-path self-test (no counterpart in the reference).  Runs the library's bounded device wait
 * on an mbarrier that nothing ever arrives on, with a time limit of limit_ns (1 ns .. 2 s): the wait
 * gives up, writes code 77 to *err_dev (which the caller zeroes first) and the time it waited to
 * *waited_ns_dev, and the kernel returns.  Every pipeline here ends a stuck wait the same way,
 * with its own code in its own error word. */
int ck_wait_selftest(uint64_t limit_ns, int *err_dev, unsigned long long *waited_ns_dev, void *stream);

#ifdef __cplusplus
}
#endif
#endif
