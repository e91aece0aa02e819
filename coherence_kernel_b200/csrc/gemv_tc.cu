// gemv_tc.cu -- Q4_K decode matvec on the tensor cores: y[r] = sum_j W[r, j] x[j], x and y fp32
// (the fused form of form_q4k_matvec_f32, q4k-msl.fk:111-114).
//
// The CUDA-core matvec spends about 2.4 issued instructions per weight (a byte permute per weight
// to make a float, the packed FMA, the per-row scale unpack) and stops near 35% of HBM.  Here the
// 4-bit codes go to an integer MMA almost as they lie in memory, and all scale arithmetic happens
// once per (row, sub-block) on exact integer sums:
//   * A (u8, in tensor memory): per superblock and row, the 128 qs bytes masked twice -- the low
//     nibbles (w & 0x0F0F0F0F) as K 0..127 and the high nibbles in place (w & 0xF0F0F0F0, i.e.
//     16 q) as K 128..255.  One LOP3 per four weights; K step k (32 wide) is exactly one
//     sub-block: 2k for k < 4 (low nibbles of chunk k), 2(k-4)+1 for k >= 4;
//   * B (s8, shared memory, 128-byte swizzle): x of sub-block s as a 22-bit fixed-point integer
//     X = rint(x 2^(22-e_s)) (e_s: the sub-block's power-of-two bound on |x|), split into three
//     balanced base-256 digits X = 65536 l0 + 256 l1 + l2, each in [-128, 127].  Row 4 s + t of
//     B holds digit t at the K positions of sub-block s and zero elsewhere, so one M = 128, N = 32
//     accumulator collects, per row and sub-block, the three exact int32 sums D_st = sum q l_t
//     (|D| <= 32 * 240 * 128 < 2^24, so also exact as floats);
//   * epilogue: sum q x over sub-block s = (65536 D_s0 + 256 D_s1 + D_s2) 2^(e_s-22) (/16 for the
//     high nibbles; combined in fp32, as the weighted sum can exceed int32), and
//     y += d sc_s (that) - dmin m_s X_s with X_s = sum x (fp32).
// The only approximation beyond fp32 roundings of the sums is the 22-bit fixed point of x,
// relative 2^-22 of the sub-block's largest |x|.
//
// One CTA handles a 128-row tile over a range of superblocks; the CTAs of a cluster split a tile's
// superblocks and add their partial row sums through distributed shared memory in rank order (no
// global scratch, deterministic).  Roles (640 threads): warp 0 TMA-loads the 128 rows' 144-byte
// superblock blocks; warp 1 owns tensor memory and issues the MMAs; warps 2-3 write the B tiles of
// alternate superblocks (the zero parts are written once); warps 4-11, two sets of four taking
// alternate superblocks, build A in tensor memory and pass the rows' 16-byte headers on; warps
// 12-19, likewise in two sets, apply the scales.  Every
// wait is bounded (about one second); a CTA whose wait gives up writes NaN to its rows.
#include "ck_common.cuh"
#include "ck_launch.h"
#include "tc_i8.cuh"

#include <initializer_list>
#include <mutex>

namespace ck {
namespace gtc {
using namespace tci8;

constexpr int NTHR = 640;
constexpr int ROWS = 128;  // MMA M: rows per tile
constexpr int NCOL = 32;   // MMA N: 8 sub-blocks x (3 digits + 1 zero row)
constexpr int WST = 6;     // weight stages (one superblock of the 128 rows each)
constexpr int NA = 4;      // operand stages: B tiles in shared memory, A in tensor memory
constexpr int ND = 8;      // accumulator stages in tensor memory, and header slots
constexpr int BST = NA;
constexpr int XSL = 16;    // per-superblock x sums / scale slots (>= ND + NA)
constexpr uint32_t W_STAGE = ROWS * Q4K_BYTES;  // 18432
constexpr uint32_t B_TILE = NCOL * 128;         // [32 rows x 128 K] s8, 128-byte swizzle
constexpr uint32_t B_STAGE = 2 * B_TILE;        // 256 K
constexpr uint32_t H_STAGE = ROWS * 16;         // the rows' superblock headers
constexpr uint32_t W_OFF = 0;
constexpr uint32_t B_OFF = W_OFF + WST * W_STAGE;  // 110592, 1024-aligned
constexpr uint32_t H_OFF = B_OFF + BST * B_STAGE;  // 143360
constexpr uint32_t XS_OFF = H_OFF + ND * H_STAGE;
constexpr uint32_t RED_OFF = XS_OFF + XSL * 64;     // this CTA's row partials, two epilogue sets
constexpr uint32_t INBOX_OFF = RED_OFF + 2 * ROWS * 4;  // rank 0: the peers' row sums and error words
constexpr uint32_t MAX_CLUSTER = 4;
constexpr uint32_t BAR_OFF = INBOX_OFF + (MAX_CLUSTER - 1) * (ROWS + 1) * 4 + 4;
constexpr uint32_t SMEM = BAR_OFF + 512 + 1024;       // + barriers, + alignment slack
constexpr uint32_t A_COLS = 64, D_OFF = NA * A_COLS, TMEM_COLS = 512;
// kind::i8 instruction descriptor: D s32, A u8, B s8, both K-major, M x N
constexpr uint32_t IDESC = idesc_u8s8(ROWS, NCOL);
static_assert(D_OFF + ND * NCOL <= TMEM_COLS, "tensor memory");
static_assert(SMEM <= 227 * 1024, "shared memory");

CK_DEV void tma_load_2d_u8(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"((uint64_t)map), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}
CK_DEV void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
CK_DEV void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
CK_DEV uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
CK_DEV uint32_t peer_addr(const void *local, uint32_t rank) {
    uint32_t pa;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(pa) : "r"(smem_u32(local)), "r"(rank));
    return pa;
}
CK_DEV void st_peer_u32(const void *local, uint32_t rank, uint32_t v) {
    asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(peer_addr(local, rank)), "r"(v) : "memory");
}
// arrive on the mbarrier at the same offset in CTA `rank` of the cluster, releasing this thread's
// earlier stores to it
CK_DEV void mbar_arrive_peer(uint64_t *local, uint32_t rank) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(peer_addr(local, rank))
                 : "memory");
}

constexpr uint32_t MAX_GROUP = 4;  // matrices of one shape sharing x in one launch
struct Params {
    const float *x;
    float *y[MAX_GROUP];       // y of matrix g (maps wmap0 .. wmap3)
    uint32_t rows, cols, nsb;  // nsb: superblocks per row
    uint32_t csize;            // CTAs per cluster (K split)
    uint32_t trows;            // rows per tile (<= ROWS; the MMA's rows past it are discarded)
    uint32_t tiles;            // tiles per matrix
};

__global__ void __launch_bounds__(NTHR, 1) k_gemv_tc(const __grid_constant__ CUtensorMap wmap0,
                                                     const __grid_constant__ CUtensorMap wmap1,
                                                     const __grid_constant__ CUtensorMap wmap2,
                                                     const __grid_constant__ CUtensorMap wmap3, Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + BAR_OFF);
    // ops_full[j % NA]: A (four warps) and B (one warp) of superblock j are in place;
    // mma_done[j % ND]: its MMAs have completed (A and B stages free, accumulator ready);
    // d_empty[j % ND]: its epilogue has read the accumulator and the header
    uint64_t *w_full = bars, *w_empty = w_full + WST, *ops_full = w_empty + WST, *mma_done = ops_full + NA;
    uint64_t *d_empty = mma_done + ND, *done = d_empty + ND;
    uint64_t *inbox_full = done + 1;  // rank 0: every peer thread's row sum has landed
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(inbox_full + 1);
    int *err = reinterpret_cast<int *>(tmem_slot + 1);
    float *red = reinterpret_cast<float *>(smem + RED_OFF);
    float *xs = reinterpret_cast<float *>(smem + XS_OFF);  // per slot: X_s[8], scale_s[8]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // cluster blockIdx / csize is tile `tile` of matrix `mi`
    const uint32_t q = cluster_rank(), mi = blockIdx.x / p.csize / p.tiles, tile = blockIdx.x / p.csize % p.tiles;
    const uint32_t row0 = tile * p.trows;
    const CUtensorMap *wmap = mi == 0 ? &wmap0 : mi == 1 ? &wmap1 : mi == 2 ? &wmap2 : &wmap3;
    float *__restrict__ y = mi == 0 ? p.y[0] : mi == 1 ? p.y[1] : mi == 2 ? p.y[2] : p.y[3];
    // this CTA's superblocks [sb0, sb1)
    const uint32_t sb0 = (uint32_t)((uint64_t)p.nsb * q / p.csize), sb1 = (uint32_t)((uint64_t)p.nsb * (q + 1) / p.csize);
    const int nj = (int)(sb1 - sb0);

    // the B ring starts all zero: the builders only ever rewrite the live spans of each stage
    for (uint32_t i = threadIdx.x; i < BST * B_STAGE / 16; i += NTHR)
        reinterpret_cast<uint4 *>(smem + B_OFF)[i] = make_uint4(0u, 0u, 0u, 0u);
    if (threadIdx.x == 0) {
        for (int i = 0; i < WST; ++i) {
            mbar_init(&w_full[i], 1);
            mbar_init(&w_empty[i], 4);
        }
        for (int i = 0; i < NA; ++i) mbar_init(&ops_full[i], 5);
        for (int i = 0; i < ND; ++i) {
            mbar_init(&mma_done[i], 1);
            mbar_init(&d_empty[i], 4);
        }
        mbar_init(done, 1);
        mbar_init(inbox_full, p.csize > 1 ? (p.csize - 1) * ROWS : 1);
        *err = 0;
        fence_barrier_init();
    }
    fence_proxy_async_smem();  // the zeroed B ring is read by the tensor cores (async proxy)
    if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // every CTA of the cluster has initialised its barriers once this phase completes; the wait
    // comes at the very end, before the first remote arrive
    cluster_arrive();
    const uint32_t tmem = *tmem_slot;
    pdl_launch_dependents();
    // x may be written by the kernel before this one, and y read by it: every warp but the weight
    // producer waits for it here.  The packed weights are never written by the kernel before (no
    // kernel of this library writes them), so the producer fills the first stages first and waits
    // after, and those loads overlap the previous kernel's tail.
    if (warp != 0) pdl_wait();

    if (warp == 0) {
        // ------------------------------------------------------------ weights: TMA producer
        if (lane == 0) {
            prefetch_tmap(wmap);
            int issued = 0;
            const int early = nj < WST ? nj : WST;
            for (int j = 0; j < early; ++j) {
                mbar_arrive_expect_tx(&w_full[j], p.trows * Q4K_BYTES);
                tma_load_2d_u8(smem + W_OFF + j * W_STAGE, wmap, &w_full[j], (int)((sb0 + j) * Q4K_BYTES),
                               (int)row0);
                issued = j + 1;
            }
            pdl_wait();
            for (int j = early; j < nj; ++j) {
                const int s = j % WST;
                if (!mbar_wait_bounded(&w_empty[s], ((j / WST) & 1) ^ 1, err, 1)) break;
                mbar_arrive_expect_tx(&w_full[s], p.trows * Q4K_BYTES);
                tma_load_2d_u8(smem + W_OFF + s * W_STAGE, wmap, &w_full[s], (int)((sb0 + j) * Q4K_BYTES),
                               (int)row0);
                issued = j + 1;
            }
            // no copy may still be landing when the CTA exits (only the last load of each stage can
            // be outstanding; after a normal run all of them have long completed)
            for (int j = issued > WST ? issued - WST : 0; j < issued; ++j)
                mbar_wait_bounded(&w_full[j % WST], (j / WST) & 1, nullptr, 0);
        } else {
            pdl_wait();
        }
        __syncwarp();  // the warp reaches the CTA barrier below as a whole
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        // The whole warp runs the loop and one elected lane issues: a tcgen05.mma from a lone
        // diverged thread issues several times slower than its N = 32 tile takes to compute.
        const uint32_t bring = smem_u32(smem + B_OFF);
        for (int j = 0; j < nj; ++j) {
            const int a = j % NA, bs = a, ds = j % ND;
            int ok = 1;
            // the A builders waited for the epilogue of superblock j - ND before arriving, so the
            // accumulator stage is free too
            if (lane == 0) ok = mbar_wait_bounded(&ops_full[a], (j / NA) & 1, err, 2);
            if (!__shfl_sync(0xffffffffu, ok, 0)) break;
            tc_fence_after();
            if (elect_one()) {
                const uint64_t bd0 = sdesc_k_sw128(bring + bs * B_STAGE), bd1 = bd0 + (B_TILE >> 4);
                const uint32_t dt = tmem + D_OFF + NCOL * ds, at = tmem + A_COLS * a;
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    umma_i8_ts(dt, at + 8 * k, (k < 4 ? bd0 : bd1) + (uint64_t)(2 * (k & 3)), IDESC, k > 0 ? 1u : 0u);
                umma_commit(&mma_done[ds]);
            }
            __syncwarp();
        }
        // every MMA has finished before tensor memory is released
        if (elect_one()) umma_commit(done);
        __syncwarp();
        if (lane == 0) mbar_wait_bounded(done, 0, nullptr, 0);
        __syncwarp();
    } else if (warp < 4) {
        // ------------------------------------------------------------ B builders (alternate superblocks)
        // lane = 4 s + qt: sub-block s, weights 8 qt .. 8 qt + 7 of it
        const int s = lane >> 2, qt = lane & 3;
        const int kk0 = 32 * (s >> 1) + 8 * qt;  // K of the first weight within its 128-K tile
        const uint32_t toff = (uint32_t)(s & 1) * B_TILE;
        // this lane's eight x of superblock j, loaded one iteration ahead
        const float *xl = p.x + (size_t)sb0 * 256 + 32 * s + 8 * qt;
        float4 n0 = make_float4(0.f, 0.f, 0.f, 0.f), n1 = n0;
        if (warp - 2 < nj) {
            n0 = __ldg(reinterpret_cast<const float4 *>(xl + (size_t)(warp - 2) * 256));
            n1 = __ldg(reinterpret_cast<const float4 *>(xl + (size_t)(warp - 2) * 256) + 1);
        }
        for (int j = warp - 2; j < nj; j += 2) {
            const int bs = j % BST;
            const float4 v0 = n0, v1 = n1;
            if (j + 2 < nj) {
                n0 = __ldg(reinterpret_cast<const float4 *>(xl + (size_t)(j + 2) * 256));
                n1 = __ldg(reinterpret_cast<const float4 *>(xl + (size_t)(j + 2) * 256) + 1);
            }
            // B stage bs was last read by the MMAs of superblock j - NA
            const bool ok = j < NA || mbar_wait_bounded(&mma_done[(j - NA) % ND], ((j - NA) / ND) & 1, err, 5);
            if (!__all_sync(0xffffffffu, ok)) break;
            const float xv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
            float mx = 0.0f, sum = 0.0f;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                mx = fmaxf(mx, fabsf(xv[e]));
                sum += xv[e];
            }
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            sum += __shfl_xor_sync(0xffffffffu, sum, 2);
            const int e = subblock_exponent(mx);
            uint2 w0, w1, w2;
            digits8(xv, e, w0, w1, w2);
            uint8_t *st = smem + B_OFF + bs * B_STAGE + toff;
            *reinterpret_cast<uint2 *>(st + b_off(4 * s + 0, kk0)) = w0;
            *reinterpret_cast<uint2 *>(st + b_off(4 * s + 1, kk0)) = w1;
            *reinterpret_cast<uint2 *>(st + b_off(4 * s + 2, kk0)) = w2;
            if (qt == 0) {
                float *slot = xs + (j % XSL) * 16;
                slot[s] = sum;
                // 2^(e-22), and 2^(e-26) for the high nibbles (A holds 16 q there)
                slot[8 + s] = digit_scale(e, 4 * (s & 1));
            }
            fence_proxy_async_smem();  // generic writes of B, read by the tensor cores
            __syncwarp();
            if (lane == 0) mbar_arrive(&ops_full[bs]);
        }
    } else if (warp < 12) {
        // ------------------------------------------------------------ A builders + headers
        // two sets of four warps (one per tensor-memory sub-partition) take alternate superblocks
        const int sub = warp & 3, r = 32 * sub + lane;
        const uint32_t trow = tmem + ((uint32_t)(32 * sub) << 16);
        for (int j = (warp - 4) >> 2; j < nj; j += 2) {
            const int ws = j % WST, a = j % NA, ds = j % ND;
            // A stage a was last read by the MMAs of superblock j - NA; header slot ds by the
            // epilogue of superblock j - ND (waiting for it also frees the accumulator stage)
            const bool ok = mbar_wait_bounded(&w_full[ws], (j / WST) & 1, err, 6) &&
                            (j < NA || mbar_wait_bounded(&mma_done[(j - NA) % ND], ((j - NA) / ND) & 1, err, 7)) &&
                            mbar_wait_bounded(&d_empty[ds], ((j / ND) & 1) ^ 1, err, 8);
            if (!__all_sync(0xffffffffu, ok)) break;  // the tensor-memory stores below need the whole warp
            tc_fence_after();
            const uint8_t *blk = smem + W_OFF + ws * W_STAGE + r * Q4K_BYTES;
            reinterpret_cast<uint4 *>(smem + H_OFF + ds * H_STAGE)[r] = *reinterpret_cast<const uint4 *>(blk);
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
            tmem_st32(trow + (uint32_t)(A_COLS * a), lo);
            tmem_st32(trow + (uint32_t)(A_COLS * a + 32), hi);
            tmem_st_wait();
            fence_proxy_async_smem();  // the W stage is refilled by TMA (async proxy)
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&w_empty[ws]);
                mbar_arrive(&ops_full[a]);
            }
        }
    } else {
        // ------------------------------------------------------------ epilogue
        // two sets of four warps take alternate superblocks, all eight sub-blocks each
        const int sub = warp & 3, g = (warp - 12) >> 2, r = 32 * sub + lane;
        const uint32_t trow = tmem + ((uint32_t)(32 * sub) << 16);
        float acc = 0.0f;
        for (int j = g; j < nj; j += 2) {
            const int ds = j % ND;
            if (!__all_sync(0xffffffffu, mbar_wait_bounded(&mma_done[ds], (j / ND) & 1, err, 9))) break;
            tc_fence_after();
            uint32_t dv[32];
            tmem_ld32(trow + D_OFF + NCOL * ds, dv);
            const uint4 hdr = reinterpret_cast<const uint4 *>(smem + H_OFF + ds * H_STAGE)[r];
            const float *slot = xs + (j % XSL) * 16;
            tmem_ld_wait();
            const float d = f16_bits_to_float(hdr.x & 0xFFFF), dmin = f16_bits_to_float(hdr.x >> 16);
#pragma unroll
            for (int s = 0; s < 8; ++s) {
                const int i = s;
                int scv, mv;
                q4k_scale_min(hdr.y, hdr.z, hdr.w, s, scv, mv);
                const float qx = digit_sum(dv[4 * i], dv[4 * i + 1], dv[4 * i + 2]) * slot[8 + s];  // sum q x
                acc = fmaf(d * (float)scv, qx, fmaf(-(dmin * (float)mv), slot[s], acc));
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&d_empty[ds]);
        }
        red[g * ROWS + r] = acc;
    }
    __syncthreads();
    cluster_wait();
    // the row sums of the cluster's CTAs, added in rank order by rank 0: the peers push theirs into
    // rank 0's inbox and leave; rank 0 waits for all of them (bounded) and writes y
    float *inbox = reinterpret_cast<float *>(smem + INBOX_OFF);
    int *inbox_err = reinterpret_cast<int *>(inbox + (MAX_CLUSTER - 1) * ROWS);
    if (threadIdx.x < ROWS) {
        const uint32_t r = threadIdx.x, row = row0 + r;
        float v = red[r] + red[ROWS + r];
        if (q != 0) {
            st_peer_u32(&inbox[(q - 1) * ROWS + r], 0, __float_as_uint(v));
            if (r == 0) st_peer_u32(&inbox_err[q - 1], 0, (uint32_t)*err);
            mbar_arrive_peer(inbox_full, 0);
        } else {
            bool bad = *err != 0;
            if (p.csize > 1) {
                bad |= !mbar_wait_bounded(inbox_full, 0, nullptr, 0);
                for (uint32_t c = 1; c < p.csize; ++c) {
                    v += inbox[(c - 1) * ROWS + r];
                    bad |= inbox_err[c - 1] != 0;
                }
            }
            if (r < p.trows && row < p.rows) y[row] = bad ? __int_as_float(0x7FC00000) : v;
        }
    }
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

// Tile height and K split.  Within one wave of CTAs the time follows the superblocks each CTA
// streams (its pipeline's cadence), not the bytes: so full 128-row tiles, and the largest split in
// {1, 2, 4} that keeps every CTA resident and gives each at least two superblocks.  (Clusters of 8
// CTAs, each needing a whole SM, schedule poorly.)
static void plan(uint32_t rows, uint32_t nsb, uint32_t nsm, uint32_t &trows, uint32_t &csize) {
    trows = ROWS;
    const uint32_t tiles = (rows + ROWS - 1) / ROWS;
    csize = 1;
    for (uint32_t c : {2u, 4u})
        if (tiles * c <= nsm && nsb >= 2 * c) csize = c;
}

}  // namespace gtc

EncodeTiledFn tensor_map_encoder() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult qr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &qr) == cudaSuccess &&
            qr == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(f);
    });
    return fn;
}

bool gemv_tc_ok(const void *qb, const float *x, uint32_t rows, uint32_t cols) {
    return cols % 256 == 0 && cols >= 256 && rows >= 1 && (reinterpret_cast<uintptr_t>(qb) & 15) == 0 &&
           (reinterpret_cast<uintptr_t>(x) & 15) == 0;
}

namespace gtc {
// ng matrices qb[0 .. ng) of one shape, all against x, in one launch: every matrix's tiles and K
// split are those of its own single launch (so each y is bit-identical to it), one after another in
// the grid
static int launch(uint32_t ng, const uint8_t *const *qb, const float *x, float *const *y, uint32_t rows,
                  uint32_t cols, uint32_t trows, uint32_t csize, cudaStream_t s) {
    if (trows == 0 || trows > ROWS || csize == 0 || csize > MAX_CLUSTER || ng == 0 || ng > MAX_GROUP)
        return CK_ERR_ARG;
    EncodeTiledFn enc = tensor_map_encoder();
    if (!enc) return CK_ERR_NODEV;
    const uint32_t nsb = cols / 256, row_bytes = nsb * Q4K_BYTES;
    CUtensorMap maps[MAX_GROUP];
    for (uint32_t g = 0; g < MAX_GROUP; ++g) {
        if (g >= ng) {
            maps[g] = maps[0];  // never read
            continue;
        }
        cuuint64_t dims[2] = {row_bytes, rows};
        cuuint64_t strides[1] = {row_bytes};
        cuuint32_t box[2] = {Q4K_BYTES, trows};
        cuuint32_t estr[2] = {1, 1};
        if (enc(&maps[g], CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t *>(qb[g]), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return CK_ERR_ARG;
    }
    const uint32_t tiles = (rows + trows - 1) / trows;
    static unsigned long long set = 0;
    if (attr_pending(set)) {
        cudaError_t e = cudaFuncSetAttribute(gtc::k_gemv_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, gtc::SMEM);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(gtc::k_gemv_tc, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) return (int)e;
        attr_mark(set);
    }
    gtc::Params p = {};
    p.x = x;
    for (uint32_t g = 0; g < MAX_GROUP; ++g) p.y[g] = y[g < ng ? g : 0];
    p.rows = rows;
    p.cols = cols;
    p.nsb = nsb;
    p.csize = csize;
    p.trows = trows;
    p.tiles = tiles;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = csize;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ng * tiles * csize);
    cfg.blockDim = dim3(gtc::NTHR);
    cfg.dynamicSmemBytes = gtc::SMEM;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, gtc::k_gemv_tc, maps[0], maps[1], maps[2], maps[3], p);
    return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}
}  // namespace gtc

int launch_gemv_tc(const uint8_t *qb, const float *x, float *y, uint32_t rows, uint32_t cols, cudaStream_t s) {
    return launch_gemv_tc_group(1, &qb, x, &y, rows, cols, s);
}

int launch_gemv_tc_group(uint32_t ng, const uint8_t *const *qb, const float *x, float *const *y, uint32_t rows,
                         uint32_t cols, cudaStream_t s) {
    for (uint32_t g = 0; g < ng; ++g)
        if (!gemv_tc_ok(qb[g], x, rows, cols)) return CK_ERR_SHAPE;
    int dev = 0, nsm = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    uint32_t trows, csize;
    gtc::plan(rows, cols / 256, (uint32_t)nsm, trows, csize);
    return gtc::launch(ng, qb, x, y, rows, cols, trows, csize, s);
}

}  // namespace ck
