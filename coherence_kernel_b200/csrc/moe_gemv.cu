// moe_gemv.cu -- the grouped expert projections of a decode-sized MoE batch (at most 8 tokens per
// token tile) on the integer tensor cores; the few-token form of k_gemm_q4k (gemm_tc.cu), same
// tile table and output layout:
//   dual = 1 :  out[o + t, n] = silu(sum_k X W0_g) * (sum_k X W1_g) * row_w[o + t]
//   dual = 0 :  out[o + t, n] = sum_k X W_g
// for each tile (g, x_row, o, n) of the permute's table and t < n (moe-msl.fk's expert matvecs).
//
// At these sizes the projections only stream weights: every expert matrix is read once for its
// few tokens.  The weights reach the MMA as in the single-token matvec (gemv_tc.cu): u8 codes in
// tensor memory (low nibbles, and high nibbles in place = 16 q), one K step of 32 per Q4_K
// sub-block; the tokens' activations are s8 fixed-point digits (tc_i8.cuh).  Here the B operand of
// K step k holds only sub-block s(k)'s 32 activations of every token -- row 3t + d is digit d of
// token t -- and each K step accumulates into its own NN columns, so N is 3 x tokens rounded up to
// 8, 16 or 32 instead of a block-diagonal 32 per token.
//
// Persistent CTAs walk the work items (tile, 128-row block of the matrix) in a fixed stride; in
// dual mode an item runs the gate rows and then the same rows of the up matrix, so the epilogue
// applies silu * up * route weight itself.  An item covers the whole reduction: no cross-CTA sums.
// Roles (640 threads): warp 0 TMA-loads superblock columns of 128 weight rows (3D maps over the
// stacked expert matrices); warp 1 owns tensor memory and issues the MMAs from an elected lane;
// warps 2-3 write the B tiles of alternate steps; warps 4-11, two sets of four on alternate steps,
// build A and pass the rows' headers on; warps 12-19, again two sets on alternate steps, apply the
// scales and meet once per item to finish it.  Every wait is bounded (about one second) and a wait
// that gives up records its code in the error word.
#include "ck_common.cuh"
#include "ck_launch.h"
#include "tc_i8.cuh"

namespace ck {
namespace gmv {
using namespace tci8;

constexpr int NTHR = 640;
constexpr int ROWS = 128;
constexpr int MAXT = 8;      // tokens per tile
constexpr int WST = 6;       // weight stages (one superblock column of 128 rows each)
constexpr int NA = 4;        // A stages in tensor memory (64 columns each)
constexpr int BST = 4;       // B stages
constexpr int NSLOT = 8;     // per-step rings: headers, x sums and scales, MMA / epilogue barriers
constexpr uint32_t W_STAGE = ROWS * Q4K_BYTES;  // 18432
constexpr uint32_t B_TILE = 32 * 128;           // [32 rows (token, digit) x 128 K] s8, 128-byte swizzle
constexpr uint32_t B_STAGE = 2 * B_TILE;        // one superblock: K steps 0-3, then 4-7
constexpr uint32_t H_STAGE = ROWS * 16;
constexpr uint32_t XS_SLOT = MAXT * 16 * 4;     // per token: X_s[8], digit scale_s[8]
constexpr uint32_t W_OFF = 0;
constexpr uint32_t B_OFF = W_OFF + WST * W_STAGE;       // 110592, 1024-aligned
constexpr uint32_t H_OFF = B_OFF + BST * B_STAGE;       // 143360
constexpr uint32_t XS_OFF = H_OFF + NSLOT * H_STAGE;    // 159744
constexpr uint32_t RED_OFF = XS_OFF + NSLOT * XS_SLOT;  // 163840: [item parity][gate, up][token][row]
constexpr uint32_t RED_BYTES = 2 * 2 * MAXT * ROWS * 4;
constexpr uint32_t STG_OFF = RED_OFF + RED_BYTES;  // B builders' activation staging
constexpr uint32_t STG_BUF = MAXT * 32 * 16;        // one step: 8 tokens x 32 lanes x 16 bytes
constexpr uint32_t BAR_OFF = STG_OFF + 2 * 2 * STG_BUF;  // [B warp][buffer]
constexpr uint32_t SMEM = BAR_OFF + 512 + 1024;  // + barriers, + alignment slack
constexpr uint32_t A_COLS = 64, D_OFF = NA * A_COLS, TMEM_COLS = 512;
static_assert(SMEM <= 227 * 1024, "shared memory");

struct Params {
    const uint16_t *x;      // bf16 activations [x_rows, K]
    uint16_t *out;          // bf16 [out_rows, N]
    const float *row_w;     // dual mode: weight per output row (null = 1)
    const int4 *tiles;      // (group, x_row, out_row, ntok)
    const int32_t *ntiles;  // device-side tile count
    uint32_t n_routed, N, K, nsb, rtiles, dual, xrow_is_orow;
    int *err;               // device error word
};

// A role's position in this CTA's step sequence: items blockIdx.x + k gridDim.x, each S steps.
// Advanced incrementally; the tile entry is read only when the item changes (a read per step
// would put a global-memory round trip on the critical path of every role).
struct Step {
    int4 tl;     // the tile
    int kit;     // the item's index in this CTA's sequence
    int rt;      // 128-row block of the matrix
    int m;       // 0: W0 (gate or the only matrix), 1: W1 (up)
    int sb;      // superblock column
    int js;      // step within the item
};
CK_DEV void step_item(Step &st, const Params &p) {
    const int it = (int)blockIdx.x + st.kit * (int)gridDim.x;
    const int tile = it / (int)p.rtiles;
    st.rt = it - tile * (int)p.rtiles;
    st.tl = p.tiles[tile];
}
CK_DEV void step_fields(Step &st, const Params &p) {
    st.m = (p.dual && st.js >= (int)p.nsb) ? 1 : 0;
    st.sb = st.js - st.m * (int)p.nsb;
}
CK_DEV Step step_at(const Params &p, int j, int S) {
    Step st;
    st.kit = j / S;
    st.js = j - st.kit * S;
    step_item(st, p);
    step_fields(st, p);
    return st;
}
// Moves `by` steps on (an item may have fewer steps than that); the caller passes more = false when
// the new position is past its sequence, so the tile entry there is not read.
CK_DEV void step_advance(Step &st, const Params &p, int by, int S, bool more) {
    st.js += by;
    if (st.js >= S) {
        const int w = st.js / S;
        st.js -= w * S;
        st.kit += w;
        if (more) step_item(st, p);
    }
    step_fields(st, p);
}

// mbar_wait_bounded over a whole warp with one uniform outcome
CK_DEV bool warp_wait(uint64_t *bar, uint32_t parity, int *err, int code) {
    return __all_sync(0xffffffffu, mbar_wait_bounded(bar, parity, err, code));
}

// The epilogue of set H (warps 12-15 for H = 0, 16-19 for H = 1), which takes the steps j with
// j % 2 == H: per step, the eight K steps' accumulators of every row and token to sums of q x,
// weighted by the rows' scales.  An item's last step belongs to one set (the finisher); the other
// set hands its partial sums over after its own last step of the item (at step S - 2), and the
// finisher applies silu * up * route weight (dual) and stores.  In the dual form each set moves its
// gate sums aside at its first up step of the item.
template <int NN>
CK_DEV void epilogue(const Params &p, int S, int nj, uint8_t *smem, uint64_t *mma_done, uint64_t *d_empty,
                     uint64_t *red_full, uint64_t *red_empty, int *err, uint32_t tmem, int H, int sub, int lane) {
    constexpr int DS = 8 * NN;
    constexpr int ND = (int)(TMEM_COLS - D_OFF) / DS;
    constexpr int KB = 32 / NN;  // K steps per accumulator load (32 registers)
    // the tokens this variant's N holds (3 digit rows each): the token loops are unrolled only that
    // far, which keeps the code small (the roles share each scheduler's instruction cache)
    constexpr int MT = NN / 3 < MAXT ? NN / 3 : MAXT;
    const int r = 32 * sub + lane;
    const uint32_t trow = tmem + ((uint32_t)(32 * sub) << 16);
    float *xs = reinterpret_cast<float *>(smem + XS_OFF);
    float *red = reinterpret_cast<float *>(smem + RED_OFF);
    float acc[MT], accg[MT];
#pragma unroll
    for (int t = 0; t < MT; ++t) acc[t] = accg[t] = 0.0f;
    Step st = {};
    if (H < nj) st = step_at(p, H, S);
    int cur_kit = -1;
    bool up = false;  // this set has reached the item's up rows
    for (int j = H; j < nj; j += 2, step_advance(st, p, 2, S, j < nj)) {
        if (!warp_wait(&mma_done[j % NSLOT], (j / NSLOT) & 1, err, 9)) break;
        tc_fence_after();
        if (st.kit != cur_kit) {
            cur_kit = st.kit;
            up = false;
        }
        if (p.dual && !up && st.js >= (int)p.nsb) {  // the gate rows are done; the up rows follow
            up = true;
#pragma unroll
            for (int t = 0; t < MT; ++t) {
                accg[t] = acc[t];
                acc[t] = 0.0f;
            }
        }
        const int n = min(st.tl.w, MT);
        const uint4 hdr = reinterpret_cast<const uint4 *>(smem + H_OFF + (j % NSLOT) * H_STAGE)[r];
        const float *slot = xs + (j % NSLOT) * (XS_SLOT / 4);
        const float d = f16_bits_to_float(hdr.x & 0xFFFF), dmin = f16_bits_to_float(hdr.x >> 16);
        const uint32_t dbase = trow + D_OFF + (uint32_t)((j % ND) * DS);
#pragma unroll
        for (int kb = 0; kb < 8; kb += KB) {
            // a batch's KB K steps are KB NN consecutive columns, read 32 at a time (a 32-column
            // load costs about what an 8-column one does)
            uint32_t dv[KB][NN];
#pragma unroll
            for (int c = 0; c < KB * NN; c += 32)
                tmem_ld32(dbase + kb * NN + c, *reinterpret_cast<uint32_t(*)[32]>(&dv[c / NN][c % NN]));
            tmem_ld_wait();
            // the batch's scales first, then token by token over its K steps: one branch per token,
            // so a token's loads and conversions for all K steps can overlap (a branch per K step
            // serialised them)
            float dsc[KB], ndm[KB];
#pragma unroll
            for (int i = 0; i < KB; ++i) {
                const int k = kb + i, s = k < 4 ? 2 * k : 2 * (k - 4) + 1;  // K step k is sub-block s
                int scv, mv;
                q4k_scale_min(hdr.y, hdr.z, hdr.w, s, scv, mv);
                dsc[i] = d * (float)scv;
                ndm[i] = -(dmin * (float)mv);
            }
#pragma unroll
            for (int t = 0; t < MT; ++t) {
                if (t >= n) break;
#pragma unroll
                for (int i = 0; i < KB; ++i) {
                    const int k = kb + i, s = k < 4 ? 2 * k : 2 * (k - 4) + 1;
                    const float qx = digit_sum(dv[i][3 * t], dv[i][3 * t + 1], dv[i][3 * t + 2]) * slot[t * 16 + 8 + s];
                    acc[t] = fmaf(dsc[i], qx, fmaf(ndm[i], slot[t * 16 + s], acc[t]));
                }
            }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&d_empty[j % NSLOT]);
        const bool last = st.js == S - 1, donor = S >= 2 && st.js == S - 2;
        if (last || donor) {
            if (p.dual && !up) {  // this set saw only gate rows of the item (one superblock per row)
#pragma unroll
                for (int t = 0; t < MT; ++t) {
                    accg[t] = acc[t];
                    acc[t] = 0.0f;
                }
            }
            // buffer kit % 2, used for the (kit / 2)-th time: written by the donor, read by the finisher
            const int buf = st.kit & 1, use = st.kit >> 1;
            float *rg = red + (size_t)buf * 2 * MAXT * ROWS, *ru = rg + MAXT * ROWS;
            if (donor) {
                if (use >= 1 && !warp_wait(&red_empty[buf], (use - 1) & 1, err, 10)) break;
#pragma unroll
                for (int t = 0; t < MT; ++t)
                    if (t < n) {
                        ru[t * ROWS + r] = acc[t];
                        rg[t * ROWS + r] = accg[t];
                    }
                __syncwarp();
                if (lane == 0) mbar_arrive(&red_full[buf]);
            } else {
                const bool other = S >= 2;  // the other set holds partial sums of this item
                if (other && !warp_wait(&red_full[buf], use & 1, err, 11)) break;
                const int col = st.rt * ROWS + r;
#pragma unroll
                for (int t = 0; t < MT; ++t) {
                    if (t >= n) break;
                    float v = acc[t] + (other ? ru[t * ROWS + r] : 0.0f);
                    if (p.dual) {
                        const float gv = accg[t] + (other ? rg[t * ROWS + r] : 0.0f);
                        const float rw = p.row_w ? p.row_w[st.tl.z + t] : 1.0f;
                        // silu(g) = g / (1 + e^-g), as the grouped GEMM computes it
                        v = __fdividef(gv, 1.0f + __expf(-gv)) * v * rw;
                    }
                    p.out[(size_t)(st.tl.z + t) * p.N + col] = __bfloat16_as_ushort(__float2bfloat16_rn(v));
                }
                __syncwarp();
                if (other && lane == 0) mbar_arrive(&red_empty[buf]);
            }
#pragma unroll
            for (int t = 0; t < MT; ++t) acc[t] = accg[t] = 0.0f;
        }
    }
}

template <int NN>
__global__ void __launch_bounds__(NTHR, 1)
    k_moe_gemv(const __grid_constant__ CUtensorMap m_w0, const __grid_constant__ CUtensorMap m_w1,
               const __grid_constant__ CUtensorMap m_s0, const __grid_constant__ CUtensorMap m_s1, Params p) {
    constexpr int DS = 8 * NN;                          // accumulator columns per step
    constexpr int ND = (int)(TMEM_COLS - D_OFF) / DS;   // accumulator stages
    constexpr uint32_t IDESC = idesc_u8s8(ROWS, NN);
    static_assert(ND >= 1 && ND <= NSLOT, "accumulator stages");
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + BAR_OFF);
    // w_full / w_empty: the weight ring; ops_full[j % NA]: A (four warps) and B (one warp) of step
    // j are in place; mma_done[j % NSLOT]: step j's MMAs have completed (its A and B stages free,
    // its accumulator ready); d_empty[j % NSLOT]: step j's epilogue has read its accumulator, header
    // and x slot; red_full / red_empty: the epilogue halves' hand-over of an item's partial sums
    uint64_t *w_full = bars, *w_empty = w_full + WST, *ops_full = w_empty + WST, *mma_done = ops_full + NA;
    uint64_t *d_empty = mma_done + NSLOT, *red_full = d_empty + NSLOT, *red_empty = red_full + 2, *done = red_empty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
    int *err = reinterpret_cast<int *>(tmem_slot + 1);
    float *xs = reinterpret_cast<float *>(smem + XS_OFF);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    for (uint32_t i = threadIdx.x; i < BST * B_STAGE / 16; i += NTHR)
        reinterpret_cast<uint4 *>(smem + B_OFF)[i] = make_uint4(0u, 0u, 0u, 0u);
    if (threadIdx.x == 0) {
        for (int i = 0; i < WST; ++i) {
            mbar_init(&w_full[i], 1);
            mbar_init(&w_empty[i], 4);
        }
        for (int i = 0; i < NA; ++i) mbar_init(&ops_full[i], 5);
        for (int i = 0; i < NSLOT; ++i) {
            mbar_init(&mma_done[i], 1);
            mbar_init(&d_empty[i], 4);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&red_full[i], 4);
            mbar_init(&red_empty[i], 4);
        }
        mbar_init(done, 1);
        *err = 0;
        fence_barrier_init();
    }
    fence_proxy_async_smem();  // the zeroed B ring is read by the tensor cores
    if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_launch_dependents();
    pdl_wait();  // the tile table and the activations come from the kernels before this one

    const int S = (int)p.nsb * (p.dual ? 2 : 1);
    const int nitems = *p.ntiles * (int)p.rtiles;
    const int mine = (int)blockIdx.x < nitems ? (nitems - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int nj = mine * S;

    if (warp == 0) {
        // ------------------------------------------------------------ weights: TMA producer
        if (lane == 0) {
            prefetch_tmap(&m_w0);
            prefetch_tmap(&m_w1);
            prefetch_tmap(&m_s0);
            prefetch_tmap(&m_s1);
            int issued = 0;
            Step st = {};
            if (nj > 0) st = step_at(p, 0, S);
            for (int j = 0; j < nj; step_advance(st, p, 1, S, ++j < nj)) {
                const int s = j % WST;
                if (!mbar_wait_bounded(&w_empty[s], ((j / WST) & 1) ^ 1, err, 1)) break;
                const bool routed = st.tl.x < (int)p.n_routed;
                const CUtensorMap *map = routed ? (st.m ? &m_w1 : &m_w0) : (st.m ? &m_s1 : &m_s0);
                mbar_arrive_expect_tx(&w_full[s], W_STAGE);
                tma_load_3d(smem + W_OFF + s * W_STAGE, map, &w_full[s], st.sb * Q4K_BYTES, st.rt * ROWS,
                            routed ? st.tl.x : st.tl.x - (int)p.n_routed);
                issued = j + 1;
            }
            // no copy may still be landing when the CTA exits
            for (int j = issued > WST ? issued - WST : 0; j < issued; ++j)
                mbar_wait_bounded(&w_full[j % WST], (j / WST) & 1, nullptr, 0);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        const uint32_t bring = smem_u32(smem + B_OFF);
        for (int j = 0; j < nj; ++j) {
            int ok = 1;
            if (lane == 0)
                ok = mbar_wait_bounded(&ops_full[j % NA], (j / NA) & 1, err, 2) &&
                     (j < ND || mbar_wait_bounded(&d_empty[(j - ND) % NSLOT], ((j - ND) / NSLOT) & 1, err, 3));
            if (!__shfl_sync(0xffffffffu, ok, 0)) break;
            tc_fence_after();
            if (elect_one()) {
                const uint64_t bd0 = sdesc_k_sw128(bring + (j % BST) * B_STAGE), bd1 = bd0 + (B_TILE >> 4);
                const uint32_t dt = tmem + D_OFF + (uint32_t)((j % ND) * DS), at = tmem + A_COLS * (j % NA);
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    umma_i8_ts(dt + k * NN, at + 8 * k, (k < 4 ? bd0 : bd1) + (uint64_t)(2 * (k & 3)), IDESC, 0u);
                umma_commit(&mma_done[j % NSLOT]);
            }
            __syncwarp();
        }
        if (elect_one()) umma_commit(done);
        __syncwarp();
        if (lane == 0) mbar_wait_bounded(done, 0, nullptr, 0);
        __syncwarp();
    } else if (warp < 4) {
        // ------------------------------------------------------------ B builders (alternate steps)
        // lane = 4 s + qt: sub-block s, its activations 8 qt .. 8 qt + 7; sub-block s is K step
        // s / 2 (low nibbles, B tile 0) or 4 + s / 2 (high nibbles, B tile 1), at 32 (s / 2) in the
        // tile's 128-K rows
        const int s = lane >> 2, qt = lane & 3;
        const int kk0 = 32 * (s >> 1) + 8 * qt;
        const uint32_t toff = (uint32_t)(s & 1) * B_TILE;
        // the activations of this warp's next step are staged in shared memory by cp.async while
        // the current one is converted (a register prefetch would unroll the token loop, and the
        // roles share each scheduler's instruction cache)
        uint4 *stg = reinterpret_cast<uint4 *>(smem + STG_OFF + (warp - 2) * 2 * STG_BUF);
        Step nst = {};  // the step the staging reads
        auto stage = [&](const Step &st, int buf) {
            const int n = min(st.tl.w, MAXT);
            const uint16_t *xr = p.x + (size_t)(p.xrow_is_orow ? st.tl.z : st.tl.y) * p.K + st.sb * 256 + 32 * s + 8 * qt;
#pragma unroll 1
            for (int t = 0; t < n; ++t) cp_async16(&stg[(buf * MAXT + t) * 32 + lane], xr + (size_t)t * p.K);
            cp_async_commit();
        };
        if (warp - 2 < nj) {
            nst = step_at(p, warp - 2, S);
            stage(nst, 0);
        }
        int buf = 0;
        for (int j = warp - 2; j < nj; j += 2, buf ^= 1) {
            const int n = min(nst.tl.w, MAXT);
            if (j + 2 < nj) {  // the next step's activations load during this one
                step_advance(nst, p, 2, S, true);
                stage(nst, buf ^ 1);
                cp_async_wait<1>();
            } else {
                cp_async_wait<0>();
            }
            const bool ok = (j < BST || mbar_wait_bounded(&mma_done[(j - BST) % NSLOT], ((j - BST) / NSLOT) & 1, err, 4)) &&
                            (j < NSLOT || mbar_wait_bounded(&d_empty[(j - NSLOT) % NSLOT], ((j - NSLOT) / NSLOT) & 1, err, 5));
            if (!__all_sync(0xffffffffu, ok)) break;
            uint8_t *bt = smem + B_OFF + (j % BST) * B_STAGE + toff;
            float *slot = xs + (j % NSLOT) * (XS_SLOT / 4);
#pragma unroll 1
            for (int t = 0; t < n; ++t) {
                const uint4 c = stg[(buf * MAXT + t) * 32 + lane];
                const uint32_t wv[4] = {c.x, c.y, c.z, c.w};
                float xv[8];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    xv[2 * i] = __uint_as_float(wv[i] << 16);
                    xv[2 * i + 1] = __uint_as_float(wv[i] & 0xFFFF0000u);
                }
                float mx = 0.0f, sum = 0.0f;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    mx = fmaxf(mx, fabsf(xv[i]));
                    sum += xv[i];
                }
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
                sum += __shfl_xor_sync(0xffffffffu, sum, 1);
                sum += __shfl_xor_sync(0xffffffffu, sum, 2);
                const int e = subblock_exponent(mx);
                uint2 w0, w1, w2;
                digits8(xv, e, w0, w1, w2);
                *reinterpret_cast<uint2 *>(bt + b_off(3 * t + 0, kk0)) = w0;
                *reinterpret_cast<uint2 *>(bt + b_off(3 * t + 1, kk0)) = w1;
                *reinterpret_cast<uint2 *>(bt + b_off(3 * t + 2, kk0)) = w2;
                if (qt == 0) {
                    slot[t * 16 + s] = sum;
                    slot[t * 16 + 8 + s] = digit_scale(e, 4 * (s & 1));
                }
            }
            fence_proxy_async_smem();  // generic writes of B, read by the tensor cores
            __syncwarp();
            if (lane == 0) mbar_arrive(&ops_full[j % NA]);
        }
    } else if (warp < 12) {
        // ------------------------------------------------------------ A builders + headers
        const int sub = warp & 3, r = 32 * sub + lane;
        const uint32_t trow = tmem + ((uint32_t)(32 * sub) << 16);
        for (int j = (warp - 4) >> 2; j < nj; j += 2) {
            const bool ok = mbar_wait_bounded(&w_full[j % WST], (j / WST) & 1, err, 6) &&
                            (j < NA || mbar_wait_bounded(&mma_done[(j - NA) % NSLOT], ((j - NA) / NSLOT) & 1, err, 7)) &&
                            (j < NSLOT || mbar_wait_bounded(&d_empty[(j - NSLOT) % NSLOT], ((j - NSLOT) / NSLOT) & 1, err, 8));
            if (!__all_sync(0xffffffffu, ok)) break;  // the tensor-memory stores below need the whole warp
            tc_fence_after();
            const uint8_t *blk = smem + W_OFF + (j % WST) * W_STAGE + r * Q4K_BYTES;
            reinterpret_cast<uint4 *>(smem + H_OFF + (j % NSLOT) * H_STAGE)[r] = *reinterpret_cast<const uint4 *>(blk);
            uint32_t lo[32], hi[32];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const uint4 v = *reinterpret_cast<const uint4 *>(blk + 16 + 16 * i);
                const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    lo[4 * i + u] = w[u] & 0x0F0F0F0Fu;
                    hi[4 * i + u] = w[u] & 0xF0F0F0F0u;
                }
            }
            const uint32_t at = trow + (uint32_t)(A_COLS * (j % NA));
            tmem_st32(at, lo);
            tmem_st32(at + 32, hi);
            tmem_st_wait();
            fence_proxy_async_smem();  // the W stage is refilled by TMA
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&w_empty[j % WST]);
                mbar_arrive(&ops_full[j % NA]);
            }
        }
    } else {
        // ------------------------------------------------------------ epilogue
        // two sets of four warps on alternate steps (one copy of the code for both: a second copy
        // measured slower, the roles already share each scheduler's instruction cache)
        epilogue<NN>(p, S, nj, smem, mma_done, d_empty, red_full, red_empty, err, tmem, (warp - 12) >> 2, warp & 3,
                     lane);
    }
    __syncthreads();
    if (threadIdx.x == 0 && *err) atomicCAS(p.err, 0, *err);
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

template <int NN>
static int launch_nn(const CUtensorMap (&maps)[4], const Params &prm, uint32_t grid, cudaStream_t s) {
    static unsigned long long set = 0;
    if (attr_pending(set)) {
        const cudaError_t e = cudaFuncSetAttribute(k_moe_gemv<NN>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
        if (e != cudaSuccess) return (int)e;
        attr_mark(set);
    }
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(NTHR);
    cfg.dynamicSmemBytes = SMEM;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, k_moe_gemv<NN>, maps[0], maps[1], maps[2], maps[3], prm);
    return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

}  // namespace gmv

bool gemv_moe_ok(const GemmParams &p) {
    const auto al = [](const void *q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
    return !p.a_dense && p.max_tile_tok >= 1 && p.max_tile_tok <= (uint32_t)gmv::MAXT && p.N % gmv::ROWS == 0 &&
           p.K % 256 == 0 && p.K > 0 && p.w0 && p.x && p.out && al(p.w0) && al(p.x) && al(p.out) &&
           p.w_stride % 16 == 0 && (!p.dual || (p.w1 && al(p.w1))) &&
           (p.n_shared == 0 || (p.s0 && al(p.s0) && (!p.dual || (p.s1 && al(p.s1)))));
}

int launch_gemv_moe(const GemmParams &p, cudaStream_t s) {
    if (!gemv_moe_ok(p)) return CK_ERR_SHAPE;
    EncodeTiledFn enc = tensor_map_encoder();
    if (!enc) return CK_ERR_NODEV;
    const uint32_t nsb = p.K / 256, row_bytes = nsb * Q4K_BYTES;
    // a single matrix (one group, w_stride 0) still needs a valid stride for the map's third axis
    const uint64_t wstr = p.w_stride ? p.w_stride : (uint64_t)row_bytes * p.N;
    auto encode = [&](CUtensorMap &m, const uint8_t *base, uint32_t count) {
        cuuint64_t dims[3] = {row_bytes, p.N, count};
        cuuint64_t strides[2] = {row_bytes, wstr};
        cuuint32_t box[3] = {Q4K_BYTES, (cuuint32_t)gmv::ROWS, 1};
        cuuint32_t estr[3] = {1, 1, 1};
        return enc(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint8_t *>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    };
    // the maps a launch never reads (no up matrix, no shared experts) repeat the routed one
    CUtensorMap maps[4];
    const bool shared = p.n_shared > 0;
    if (!encode(maps[0], p.w0, p.n_routed) || !encode(maps[1], p.dual ? p.w1 : p.w0, p.n_routed) ||
        !encode(maps[2], shared ? p.s0 : p.w0, shared ? p.n_shared : p.n_routed) ||
        !encode(maps[3], shared && p.dual ? p.s1 : (shared ? p.s0 : p.w0), shared ? p.n_shared : p.n_routed))
        return CK_ERR_ARG;
    int dev = 0, nsm = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    gmv::Params prm = {reinterpret_cast<const uint16_t *>(p.x), reinterpret_cast<uint16_t *>(p.out), p.row_w, p.tiles,
                       p.ntiles, p.n_routed, p.N, p.K, nsb, p.N / gmv::ROWS, (uint32_t)p.dual, (uint32_t)p.xrow_is_orow,
                       p.err};
    const uint64_t items = (uint64_t)p.max_tiles * prm.rtiles;
    const uint32_t grid = (uint32_t)(items < (uint64_t)nsm ? (items ? items : 1) : (uint64_t)nsm);
    const uint32_t rows3 = 3 * p.max_tile_tok;
    if (rows3 <= 8) return gmv::launch_nn<8>(maps, prm, grid, s);
    if (rows3 <= 16) return gmv::launch_nn<16>(maps, prm, grid, s);
    return gmv::launch_nn<32>(maps, prm, grid, s);
}

}  // namespace ck
