// moe_kernels.cu -- token permute (dispatch) and weighted combine for the MoE layer.
//
// The reference gathers an expert's weights on the host per token (t.off + e*nb02,
// form/form-stdlib/moe-msl.fk:24-35) or per slot on the device (ids[slot]*stride,
// ds4-order-match.fk:251-252) and never batches tokens by expert.  Here the batch is sorted by
// expert with a deterministic counting sort (histogram -> prefix sum -> scatter, stable in the
// (token, slot) order), so every expert's tokens form one contiguous block of rows that the
// grouped tensor-core GEMM consumes in tiles, and the combine reads them back per token in the
// reference's own summation order.
#include "ck_common.cuh"
#include "ck_launch.h"

namespace ck {

constexpr int PERM_CHUNK = 1024;  // (token, slot) pairs per histogram chunk
constexpr int MAX_EXPERTS = 1024;

struct PermWs {
    int32_t *chunk_hist;   // [nchunks, E]
    int32_t *local_rank;   // [A]
    int32_t *expert_off;   // [E]
};

static inline uint32_t n_pairs(const PermuteParams &p) { return p.ntok * p.nsel; }
static inline uint32_t n_chunks(const PermuteParams &p) { return (n_pairs(p) + PERM_CHUNK - 1) / PERM_CHUNK; }

size_t permute_workspace_bytes(const PermuteParams &p) {
    size_t a = (size_t)n_chunks(p) * p.n_experts * 4;
    size_t b = (size_t)n_pairs(p) * 4;
    size_t c = (size_t)p.n_experts * 4;
    return ((a + 255) & ~(size_t)255) + ((b + 255) & ~(size_t)255) + ((c + 255) & ~(size_t)255);
}
static PermWs carve(void *ws, const PermuteParams &p) {
    uint8_t *b = (uint8_t *)ws;
    PermWs w;
    size_t a = ((size_t)n_chunks(p) * p.n_experts * 4 + 255) & ~(size_t)255;
    size_t r = ((size_t)n_pairs(p) * 4 + 255) & ~(size_t)255;
    w.chunk_hist = (int32_t *)b;
    w.local_rank = (int32_t *)(b + a);
    w.expert_off = (int32_t *)(b + a + r);
    return w;
}

// K1: per chunk, one warp walks the pairs in order; __match_any_sync ranks equal experts inside
// each 32-pair step and a shared counter per expert carries the rank across steps, so the rank of
// a pair among its expert's pairs in this chunk follows the (token, slot) order exactly.
__global__ void k_perm_hist(const int32_t *__restrict__ ids, uint32_t npairs, uint32_t E, int32_t *__restrict__ chunk_hist,
                            int32_t *__restrict__ local_rank) {
    grid_dep_trigger_small();
    grid_dep_wait();
    __shared__ int32_t cnt[MAX_EXPERTS];
    const int lane = threadIdx.x;
    for (uint32_t e = lane; e < E; e += 32) cnt[e] = 0;
    __syncwarp();
    const uint32_t p0 = blockIdx.x * PERM_CHUNK;
    const uint32_t p1 = min(p0 + PERM_CHUNK, npairs);
    const unsigned lt = (1u << lane) - 1u;
    for (uint32_t base = p0; base < p1; base += 32) {
        const uint32_t p = base + lane;
        const bool valid = p < p1;
        int e = valid ? ids[p] : -1;
        if (valid && (e < 0 || (uint32_t)e >= E)) e = -2;  // an out-of-range id is counted nowhere
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        const int rank = __popc(peers & lt);
        const int c = e >= 0 ? cnt[e] : 0;
        __syncwarp();
        if (valid) local_rank[p] = e >= 0 ? c + rank : -1;
        if (e >= 0 && lane == __ffs(peers) - 1) cnt[e] = c + __popc(peers);
        __syncwarp();
    }
    for (uint32_t e = lane; e < E; e += 32) chunk_hist[(size_t)blockIdx.x * E + e] = cnt[e];
}

// exclusive scan of one value per thread over a block of up to 1024 threads
__device__ int block_excl_scan(int v, int *total) {
    __shared__ int warp_sums[32];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[w] = x;
    __syncthreads();
    if (w == 0) {
        int s = lane < (int)(blockDim.x >> 5) ? warp_sums[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += y;
        }
        warp_sums[lane] = s;  // inclusive over warps
    }
    __syncthreads();
    const int before = (w > 0 ? warp_sums[w - 1] : 0) + x - v;
    if (total) *total = warp_sums[(blockDim.x >> 5) - 1];
    __syncthreads();
    return before;
}

// token tiles of one segment of c rows: ceil(c/bn) tiles of equal size rounded up to 16
__device__ __forceinline__ int seg_tiles(int c, int bn, int &base) {
    if (c <= 0) { base = 0; return 0; }
    const int nt = (c + bn - 1) / bn;
    int b = (c + nt - 1) / nt;
    b = ((b + 15) / 16) * 16;
    base = b < bn ? b : bn;
    return nt;
}

// K2: one block.  Per expert: chunk offsets (in chunk order), count, expert offset; then the
// token-tile table of the grouped GEMM, routed experts first (in expert order), shared after.
__global__ void __launch_bounds__(1024) k_perm_scan(int32_t *__restrict__ chunk_hist, uint32_t nchunks, PermuteParams p,
                                                    int32_t *__restrict__ expert_off, int32_t *__restrict__ counts,
                                                    int4 *__restrict__ tiles, int32_t *__restrict__ ntiles) {
    grid_dep_trigger_small();
    grid_dep_wait();
    const int e = threadIdx.x;
    int c = 0;
    if (e < (int)p.n_experts) {
        for (uint32_t k = 0; k < nchunks; ++k) {
            const int h = chunk_hist[(size_t)k * p.n_experts + e];
            chunk_hist[(size_t)k * p.n_experts + e] = c;  // becomes the chunk's offset inside the expert
            c += h;
        }
        counts[e] = c;
    }
    int total = 0;
    const int off = block_excl_scan(e < (int)p.n_experts ? c : 0, &total);
    if (e < (int)p.n_experts) expert_off[e] = off;
    int base = 0;
    const int nt = e < (int)p.n_experts ? seg_tiles(c, (int)p.bn, base) : 0;
    int ntot = 0;
    const int toff = block_excl_scan(nt, &ntot);
    for (int i = 0; i < nt; ++i) {
        const int r0 = off + i * base;
        const int n = min(base, c - i * base);
        tiles[toff + i] = make_int4(e, r0, r0, n);
    }
    // shared experts: all tokens, x rows after the routed block, output rows per shared expert
    const int A = (int)(p.ntok * p.nsel);
    int sbase = 0;
    const int snt = seg_tiles((int)p.ntok, (int)p.bn, sbase);
    for (int i = threadIdx.x; i < (int)p.n_shared * snt; i += blockDim.x) {
        const int s = i / snt, m = i % snt;
        const int n = min(sbase, (int)p.ntok - m * sbase);
        tiles[ntot + i] = make_int4((int)p.n_experts + s, A + m * sbase, A + s * (int)p.ntok + m * sbase, n);
    }
    if (threadIdx.x == 0) *ntiles = ntot + (int)p.n_shared * snt;
}

// K3: one warp per row of xp.  Routed pair p lands at expert_off[e] + chunk offset + local rank;
// the warp copies token p/nsel's activation row there with 16-byte loads.  When there are shared
// experts, rows A .. A+ntok-1 are the tokens themselves (the shared experts' input).
__global__ void k_perm_scatter(const int32_t *__restrict__ ids, const float *__restrict__ wts,
                               const uint16_t *__restrict__ x, uint16_t *__restrict__ xp, float *__restrict__ row_w,
                               int32_t *__restrict__ pair_pos, const int32_t *__restrict__ chunk_off,
                               const int32_t *__restrict__ local_rank, const int32_t *__restrict__ expert_off,
                               PermuteParams p) {
    grid_dep_trigger_small();
    grid_dep_wait();
    const uint32_t A = p.ntok * p.nsel;
    const uint32_t wid = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (wid >= A + (p.n_shared ? p.ntok : 0u)) return;
    uint32_t src_tok, dst;
    if (wid < A) {
        const int e = ids[wid];
        const int lr = local_rank[wid];
        if (e < 0 || (uint32_t)e >= p.n_experts || lr < 0) {
            if (lane == 0) pair_pos[wid] = -1;
            return;
        }
        dst = (uint32_t)(expert_off[e] + chunk_off[(size_t)(wid / PERM_CHUNK) * p.n_experts + e] + lr);
        src_tok = wid / p.nsel;
        if (lane == 0) {
            pair_pos[wid] = (int32_t)dst;
            row_w[dst] = p.weight_in_mid ? wts[wid] : 1.0f;
        }
    } else {
        src_tok = wid - A;
        dst = wid;
        if (lane == 0)
            for (uint32_t s = 0; s < p.n_shared; ++s) row_w[A + s * p.ntok + src_tok] = 1.0f;
    }
    const uint4 *s4 = reinterpret_cast<const uint4 *>(x + (size_t)src_tok * p.hidden);
    uint4 *d4 = reinterpret_cast<uint4 *>(xp + (size_t)dst * p.hidden);
    for (uint32_t v = lane; v < p.hidden / 8; v += 32) d4[v] = __ldg(s4 + v);
}

int launch_permute(const int32_t *ids, const float *wts, const uint16_t *x, uint16_t *xp, float *row_w,
                   int32_t *pair_pos, int32_t *counts, int4 *tiles, int32_t *ntiles, void *workspace,
                   const PermuteParams &p, cudaStream_t s) {
    // tiles of up to 8 tokens (the few-token matvec's), or a multiple of 8 up to the GEMM's tile
    if (p.n_experts == 0 || p.n_experts > MAX_EXPERTS || p.nsel == 0 || p.hidden % 8 != 0 || p.bn == 0 ||
        (p.bn > 8 && p.bn % 8 != 0) || p.bn > GEMM_TILE_TOKENS)
        return CK_ERR_SHAPE;
    if (!ids || !x || !xp || !row_w || !pair_pos || !counts || !tiles || !ntiles || !workspace) return CK_ERR_ARG;
    PermWs w = carve(workspace, p);
    const uint32_t npairs = n_pairs(p), nch = n_chunks(p);
    cudaError_t e = cudaSuccess;
    if (nch) e = launch_pdl(k_perm_hist, dim3(nch), dim3(32), 0, s, ids, npairs, p.n_experts, w.chunk_hist, w.local_rank);
    if (e == cudaSuccess)
        e = launch_pdl(k_perm_scan, dim3(1), dim3(1024), 0, s, w.chunk_hist, nch, p, w.expert_off, counts, tiles, ntiles);
    const uint64_t warps = (uint64_t)npairs + (p.n_shared ? p.ntok : 0u);
    if (e == cudaSuccess && warps)
        e = launch_pdl(k_perm_scatter, dim3((unsigned)((warps * 32 + 255) / 256)), dim3(256), 0, s, ids, wts, x, xp,
                       row_w, pair_pos, w.chunk_hist, w.local_rank, w.expert_off, p);
    return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

// The token tiles of a single matrix over ntok rows (a prefill GEMM): group 0, rows in order.
__global__ void k_single_tiles(int4 *__restrict__ tiles, int32_t *__restrict__ ntiles, uint32_t ntok, uint32_t bn) {
    int base = 0;
    const int nt = seg_tiles((int)ntok, (int)bn, base);
    for (int i = threadIdx.x; i < nt; i += blockDim.x)
        tiles[i] = make_int4(0, i * base, i * base, min(base, (int)ntok - i * base));
    if (threadIdx.x == 0) *ntiles = nt;
}
int launch_single_tiles(int4 *tiles, int32_t *ntiles, uint32_t ntok, uint32_t bn, cudaStream_t s) {
    if (!tiles || !ntiles || bn == 0 || (bn > 8 && bn % 16) || bn > GEMM_TILE_TOKENS) return CK_ERR_ARG;
    k_single_tiles<<<1, 256, 0, s>>>(tiles, ntiles, ntok, bn);
    return (int)cudaGetLastError();
}

// dst[i] = src[idx[i]] for rows of row_bytes (a multiple of 16); idx < 0 leaves the row alone.
__global__ void k_gather_rows(const uint4 *__restrict__ src, const int32_t *__restrict__ idx, uint4 *__restrict__ dst,
                              uint32_t nrows, uint32_t vecs) {
    const uint32_t w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (w >= nrows) return;
    const int r = idx[w];
    if (r < 0) return;
    for (uint32_t v = lane; v < vecs; v += 32) dst[(size_t)w * vecs + v] = __ldg(src + (size_t)r * vecs + v);
}
int launch_gather_rows(const void *src, const int32_t *idx, void *dst, uint32_t nrows, uint32_t row_bytes,
                       cudaStream_t s) {
    if (row_bytes % 16) return CK_ERR_SHAPE;
    if (!src || !idx || !dst) return CK_ERR_ARG;
    if (nrows)
        k_gather_rows<<<(unsigned)(((uint64_t)nrows * 32 + 255) / 256), 256, 0, s>>>(
            (const uint4 *)src, idx, (uint4 *)dst, nrows, row_bytes / 16);
    return (int)cudaGetLastError();
}

// Expert-parallel dispatch plan, one CTA (the reference runs its MoE on one device; there is no
// counterpart).  Rank d owns experts [d*el, (d+1)*el).  A token crosses to each rank that holds
// at least one of its experts once: the rows of the dispatch are the (rank, token) pairs in
// (rank, token) order, each carrying its slots' local experts (-1 for slots whose expert lives
// elsewhere) and route weights (0 there) as one metadata row of 2K int32.  The (token, slot) pairs
// come back rank by rank, in (token, slot) order inside a rank; ret_pos gives each pair's row in
// that return.  Pass 1 totals rows and pairs per rank (and pairs per expert) with shared-memory
// atomics; pass 2 walks the tokens in chunks of 1024 in order and places every row and pair with
// warp ballots / scans and a scan over the warps, so all positions follow token order exactly.
constexpr int PLAN_THREADS = 1024;
constexpr uint32_t PLAN_MAX_RANKS = 32, PLAN_MAX_SLOTS = 16;
__global__ void __launch_bounds__(PLAN_THREADS) k_ep_plan(const int32_t *__restrict__ ids, const float *__restrict__ wts,
                                                       uint32_t T, uint32_t K, uint32_t E, uint32_t W,
                                                       int32_t *__restrict__ counts, long long *__restrict__ sizes,
                                                       int32_t *__restrict__ send_tok, int32_t *__restrict__ meta,
                                                       int32_t *__restrict__ ret_pos) {
    __shared__ int cnt[MAX_EXPERTS];
    __shared__ int tot_rows[PLAN_MAX_RANKS], tot_pairs[PLAN_MAX_RANKS], base_rows[PLAN_MAX_RANKS],
        base_pairs[PLAN_MAX_RANKS];
    __shared__ int wrow[PLAN_THREADS / 32][PLAN_MAX_RANKS], wpair[PLAN_THREADS / 32][PLAN_MAX_RANKS];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t el = E / W;
    for (uint32_t e = tid; e < E; e += PLAN_THREADS) cnt[e] = 0;
    if (tid < (int)PLAN_MAX_RANKS) tot_rows[tid] = tot_pairs[tid] = 0;
    __syncthreads();
    for (uint32_t t = tid; t < T; t += PLAN_THREADS) {
        uint32_t seen = 0;
        for (uint32_t k = 0; k < K; ++k) {
            const int e = ids[(size_t)t * K + k];
            if (e < 0 || (uint32_t)e >= E) continue;
            const uint32_t d = (uint32_t)e / el;
            atomicAdd(&cnt[e], 1);
            atomicAdd(&tot_pairs[d], 1);
            seen |= 1u << d;
        }
        for (; seen; seen &= seen - 1) atomicAdd(&tot_rows[__ffs(seen) - 1], 1);
    }
    __syncthreads();
    if (tid == 0) {
        int r = 0, q = 0;
        for (uint32_t d = 0; d < W; ++d) {
            base_rows[d] = r;
            base_pairs[d] = q;
            sizes[2 * d] = tot_rows[d];
            sizes[2 * d + 1] = tot_pairs[d];
            r += tot_rows[d];
            q += tot_pairs[d];
        }
    }
    for (uint32_t e = tid; e < E; e += PLAN_THREADS) counts[e] = cnt[e];
    __syncthreads();
    const unsigned lt = (1u << lane) - 1u;
    for (uint32_t c0 = 0; c0 < T; c0 += PLAN_THREADS) {
        const uint32_t t = c0 + tid;
        int er[PLAN_MAX_SLOTS];
#pragma unroll
        for (uint32_t k = 0; k < PLAN_MAX_SLOTS; ++k) {
            const int e = (t < T && k < K) ? ids[(size_t)t * K + k] : -1;
            er[k] = (e >= 0 && (uint32_t)e < E) ? (int)((uint32_t)e / el) : -1;
        }
        // per rank: this warp's rows and pairs
        for (uint32_t d = 0; d < W; ++d) {
            int c = 0;
#pragma unroll
            for (uint32_t k = 0; k < PLAN_MAX_SLOTS; ++k) c += er[k] == (int)d;
            const unsigned bal = __ballot_sync(0xffffffffu, c > 0);
            int sc = c;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, sc, o);
                if (lane >= o) sc += v;
            }
            if (lane == 31) {
                wrow[warp][d] = __popc(bal);
                wpair[warp][d] = sc;
            }
        }
        __syncthreads();
        int cr = 0, cp = 0;  // this chunk's totals for rank tid
        if (tid < (int)W) {
            for (int w = 0; w < PLAN_THREADS / 32; ++w) {
                const int a = wrow[w][tid], b = wpair[w][tid];
                wrow[w][tid] = cr;
                wpair[w][tid] = cp;
                cr += a;
                cp += b;
            }
        }
        __syncthreads();
        for (uint32_t d = 0; d < W; ++d) {
            int c = 0;
#pragma unroll
            for (uint32_t k = 0; k < PLAN_MAX_SLOTS; ++k) c += er[k] == (int)d;
            const unsigned bal = __ballot_sync(0xffffffffu, c > 0);
            int sc = c;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, sc, o);
                if (lane >= o) sc += v;
            }
            if (c > 0) {
                const int row = base_rows[d] + wrow[warp][d] + __popc(bal & lt);
                send_tok[row] = (int32_t)t;
                int32_t *m = meta + (size_t)row * 2 * K;
                int q = base_pairs[d] + wpair[warp][d] + (sc - c);
#pragma unroll
                for (uint32_t k = 0; k < PLAN_MAX_SLOTS; ++k) {
                    if (k >= K) break;
                    const bool mine = er[k] == (int)d;
                    const size_t i = (size_t)t * K + k;
                    m[k] = mine ? ids[i] - (int)(d * el) : -1;
                    m[K + k] = mine ? __float_as_int(wts[i]) : 0;
                    if (mine) ret_pos[i] = q++;
                }
            }
        }
        if (t < T) {
#pragma unroll
            for (uint32_t k = 0; k < PLAN_MAX_SLOTS; ++k)
                if (k < K && er[k] < 0) ret_pos[(size_t)t * K + k] = -1;
        }
        __syncthreads();
        if (tid < (int)W) {
            base_rows[tid] += cr;
            base_pairs[tid] += cp;
        }
        __syncthreads();
    }
}
int launch_ep_plan(const int32_t *ids, const float *wts, uint32_t ntok, uint32_t nsel, uint32_t n_experts,
                   uint32_t world, int32_t *counts, long long *sizes, int32_t *send_tok, int32_t *meta,
                   int32_t *ret_pos, cudaStream_t s) {
    if (world == 0 || world > PLAN_MAX_RANKS || nsel == 0 || nsel > PLAN_MAX_SLOTS || n_experts == 0 ||
        n_experts > (uint32_t)MAX_EXPERTS || n_experts % world)
        return CK_ERR_SHAPE;
    if (!ids || !wts || !counts || !sizes || !send_tok || !meta || !ret_pos) return CK_ERR_ARG;
    k_ep_plan<<<1, PLAN_THREADS, 0, s>>>(ids, wts, ntok, nsel, n_experts, world, counts, sizes, send_tok, meta,
                                         ret_pos);
    return (int)cudaGetLastError();
}

// Combine: a token's row is split over gridDim.y blocks of CMB_THREADS threads, 8-column vectors
// strided over them (small batches: one vector per thread; large ones: one block per token, which
// sets the token's slots up once).  order_by_expert = 1 is moe-mix (moe-gate.fk:32-37): the chosen experts in ascending
// index, acc + g*y.  order_by_expert = 0 is dsv4-moe-acc (dsv4-forward.fk:100-103): the slots in
// list order, acc + y (the weight was applied inside the expert).  Shared experts are added after,
// in index order.  fp32 accumulation, bf16 out.  The token's slots (row position and weight, in
// summation order) are set up once per block in shared memory, and a thread issues all its rows'
// loads before it adds them in that order: per-slot dependent loads made a decode-sized combine a
// chain of memory round trips.
constexpr int CMB_THREADS = 256;
__global__ void __launch_bounds__(CMB_THREADS) k_combine(const uint16_t *__restrict__ y, const int32_t *__restrict__ ids,
                                                         const float *__restrict__ wts, const int32_t *__restrict__ pair_pos,
                                                         uint16_t *__restrict__ out, float *__restrict__ out_f32,
                                                         PermuteParams p, int order_by_expert) {
    grid_dep_trigger_small();
    grid_dep_wait();
    const uint32_t t = blockIdx.x;
    const uint32_t A = p.ntok * p.nsel;
    const int ns = (int)min(p.nsel, 16u);
    __shared__ int s_id[16], s_pos[16], s_ord[16];
    __shared__ float s_g[16];
    if ((int)threadIdx.x < ns) {
        const int k = (int)threadIdx.x;
        s_id[k] = ids[t * p.nsel + k];
        s_pos[k] = pair_pos[t * p.nsel + k];
        s_g[k] = order_by_expert ? wts[t * p.nsel + k] : 1.0f;
    }
    __syncthreads();
    if ((int)threadIdx.x < ns) {
        // the summation order: ascending expert, ties in list order (a stable sort), or the list
        // order; slot k's place is the number of slots that come before it
        const int k = (int)threadIdx.x;
        int rank = k;
        if (order_by_expert) {
            rank = 0;
            for (int i = 0; i < ns; ++i) rank += s_id[i] < s_id[k] || (s_id[i] == s_id[k] && i < k);
        }
        s_ord[rank] = k;
    }
    __syncthreads();
    for (uint32_t v = blockIdx.y * CMB_THREADS + threadIdx.x; v < p.hidden / 8; v += gridDim.y * CMB_THREADS) {
        float acc[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
        // eight slots' loads at a time, then their adds in order
        for (int k0 = 0; k0 < ns; k0 += 8) {
            uint4 q[8];
            int pos[8];
            float g[8];
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
                pos[kk] = -1;
                if (k0 + kk < ns) {
                    pos[kk] = s_pos[s_ord[k0 + kk]];
                    g[kk] = s_g[s_ord[k0 + kk]];
                    if (pos[kk] >= 0) q[kk] = __ldg(reinterpret_cast<const uint4 *>(y + (size_t)pos[kk] * p.hidden) + v);
                }
            }
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
                if (pos[kk] < 0) continue;  // a slot this layer did not compute (another rank's expert)
                const uint32_t qq[4] = {q[kk].x, q[kk].y, q[kk].z, q[kk].w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float lo = __uint_as_float(qq[i] << 16), hi = __uint_as_float(qq[i] & 0xFFFF0000u);
                    if (order_by_expert) {
                        acc[2 * i] = __fadd_rn(acc[2 * i], __fmul_rn(g[kk], lo));
                        acc[2 * i + 1] = __fadd_rn(acc[2 * i + 1], __fmul_rn(g[kk], hi));
                    } else {
                        acc[2 * i] = __fadd_rn(acc[2 * i], lo);
                        acc[2 * i + 1] = __fadd_rn(acc[2 * i + 1], hi);
                    }
                }
            }
        }
        for (uint32_t sh = 0; sh < p.n_shared; ++sh) {
            const uint4 qs = __ldg(reinterpret_cast<const uint4 *>(y + ((size_t)A + (size_t)sh * p.ntok + t) * p.hidden) + v);
            const uint32_t qq[4] = {qs.x, qs.y, qs.z, qs.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                acc[2 * i] = __fadd_rn(acc[2 * i], __uint_as_float(qq[i] << 16));
                acc[2 * i + 1] = __fadd_rn(acc[2 * i + 1], __uint_as_float(qq[i] & 0xFFFF0000u));
            }
        }
        if (out) {
            uint4 o;
            o.x = pack_bf16x2(acc[0], acc[1]);
            o.y = pack_bf16x2(acc[2], acc[3]);
            o.z = pack_bf16x2(acc[4], acc[5]);
            o.w = pack_bf16x2(acc[6], acc[7]);
            reinterpret_cast<uint4 *>(out + (size_t)t * p.hidden)[v] = o;
        }
        if (out_f32) {
            float4 *o4 = reinterpret_cast<float4 *>(out_f32 + (size_t)t * p.hidden + v * 8);
            o4[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
            o4[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
        }
    }
}

int launch_combine(const uint16_t *y, const int32_t *ids, const float *wts, const int32_t *pair_pos, uint16_t *out,
                   float *out_f32, const PermuteParams &p, int order_by_expert, cudaStream_t s) {
    if (p.hidden % 8 != 0 || p.nsel > 16) return CK_ERR_SHAPE;
    if (!y || !ids || !pair_pos || (!out && !out_f32) || (order_by_expert && !wts)) return CK_ERR_ARG;
    if (p.ntok) {
        const uint32_t split = p.ntok <= 256 ? (p.hidden / 8 + CMB_THREADS - 1) / CMB_THREADS : 1;
        const cudaError_t e = launch_pdl(k_combine, dim3(p.ntok, split),
                                         dim3(CMB_THREADS), 0, s, y, ids, wts, pair_pos, out, out_f32, p, order_by_expert);
        if (e != cudaSuccess) return (int)e;
    }
    return (int)cudaGetLastError();
}

}  // namespace ck
