// ep_peer.cu -- the expert-parallel exchange over NVLink peer memory (no counterpart in the
// reference, whose MoE runs on one device).
//
// Every rank owns one device arena that its peers map through CUDA IPC: W receive regions (one per
// source rank; each `cap` rows of bf16 activations with their slots' local experts, route weights
// and source-token numbers), a return buffer indexed by (token, slot), two flag arrays (dispatch and
// return, one 64-bit slot per source rank) and a step counter.  One forward:
//
//   k_ep_begin           the rank's step counter += 1 (a device value, so a captured graph replays)
//   k_ep_dispatch        every dispatch row of the plan (ck_ep_dispatch_plan: (rank, token) order)
//                        is stored straight into region `me` of its destination's arena, and the
//                        rows of that region the step does not use get expert -1
//   k_ep_signal          system fence, then each peer's flag[me] = step (release)
//   k_ep_wait            the rank's flags[s] >= step for every s, bounded; a timeout sets err
//   ... the receiver regroups its W * cap rows by local expert and runs the expert GEMMs ...
//   k_ep_return          every (row, slot) pair the rank computed is stored into its source's return
//                        buffer at (token, slot), followed by a second signal / wait -- or, when the
//                        down projection runs on the grouped GEMM, k_ep_return_rows gives that GEMM
//                        each output row's address in its source's return buffer and the GEMM's
//                        epilogue stores the rows there itself (ck_moe_expert_gemm_rows)
//
// The host never waits and no size crosses to the host, so a forward can be captured in a CUDA
// graph.  Single buffering is safe: a rank writes step i+1 rows into a peer only after the return
// barrier of step i, which that peer passes only after it has finished reading step i's rows; and
// a peer writes step i+1 returns only after the dispatch barrier of step i+1, which this rank
// signals only after its step-i combine.
#include "../../include/ck_b200.h"
#include "ck_common.cuh"
#include "ck_launch.h"

#include <string.h>

namespace {

CK_DEV unsigned long long ld_acquire_sys(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
CK_DEV void st_release_sys(unsigned long long *p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__global__ void k_ep_begin(unsigned long long *ctr) {
    if (threadIdx.x == 0 && blockIdx.x == 0) *ctr += 1ull;
}

// One warp per dispatch row: 16-byte copies of the token's activations into the destination's
// region, then its slots' experts, weights and the token number.  Rows past the plan's total and
// the unused tail of every destination's region (expert -1) are handled by the same grid.
__global__ void k_ep_dispatch(ck_ep_peers P, const uint4 *__restrict__ x, const int32_t *__restrict__ send_tok,
                              const int32_t *__restrict__ meta, const long long *__restrict__ sizes,
                              uint32_t max_rows) {
    const uint32_t K = P.nsel, vecs = P.hidden / 8, W = P.world;
    const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const uint32_t nwarps = (gridDim.x * blockDim.x) >> 5;
    // the prefix of rows per destination (W <= 32: one value per lane)
    const long long nd = lane < W ? sizes[2 * lane] : 0;
    long long pre = nd;
    for (int o = 1; o < 32; o <<= 1) {
        const long long v = __shfl_up_sync(0xffffffffu, pre, o);
        if ((int)lane >= o) pre += v;
    }
    const long long total = __shfl_sync(0xffffffffu, pre, 31);
    for (uint32_t r = warp; r < max_rows; r += nwarps) {
        if ((long long)r >= total) break;
        // the destination: the first d whose inclusive prefix exceeds r
        const unsigned ball = __ballot_sync(0xffffffffu, lane < W && pre > (long long)r);
        const uint32_t d = __ffs(ball) - 1;
        const long long base = __shfl_sync(0xffffffffu, pre - nd, d);
        const uint32_t i = (uint32_t)((long long)r - base);
        const int32_t t = send_tok[r];
        uint4 *dst = reinterpret_cast<uint4 *>(P.recv_x[d]) + (size_t)i * vecs;
        const uint4 *src = x + (size_t)t * vecs;
        for (uint32_t v = lane; v < vecs; v += 32) dst[v] = __ldg(src + v);
        const int32_t *m = meta + (size_t)r * 2 * K;
        if (lane < K) {
            P.recv_ids[d][(size_t)i * K + lane] = m[lane];
            P.recv_w[d][(size_t)i * K + lane] = __int_as_float(m[K + lane]);
        }
        if (lane == 0) P.recv_tok[d][i] = t;
    }
    // the unused rows of region `me` in every destination: no expert
    for (uint32_t d = 0; d < W; ++d) {
        const long long n = __shfl_sync(0xffffffffu, nd, d);
        const size_t first = (size_t)n * K, last = (size_t)P.cap * K;
        for (size_t j = (size_t)(blockIdx.x * blockDim.x + threadIdx.x) + first; j < last;
             j += (size_t)gridDim.x * blockDim.x)
            P.recv_ids[d][j] = -1;
    }
}

// After the work before it on the stream: make this rank's stores visible system-wide, then tell
// every peer (flag slot `me` of its `which` array) that step *ctr is in place.
__global__ void k_ep_signal(ck_ep_peers P, int which) {
    __threadfence_system();
    const unsigned long long step = *P.ctr;
    const uint32_t d = threadIdx.x;
    if (d < P.world) st_release_sys(which ? P.rflag[d] : P.dflag[d], step);
}

// Every source's flag of the `which` array has reached this rank's step; bounded at limit_ns.
__global__ void k_ep_wait(ck_ep_peers P, int which, uint64_t limit_ns) {
    const unsigned long long step = *P.ctr;
    const unsigned long long *flags = which ? P.my_rflags : P.my_dflags;
    const uint32_t s = threadIdx.x;
    if (s < P.world) {
        const uint64_t t0 = ck::globaltimer_ns();
        for (uint32_t i = 0;; ++i) {
            if (ld_acquire_sys(flags + s) >= step) break;
            if ((i & 255u) == 255u) {
                if (*(volatile int *)P.err) break;  // another wait of this rank already gave up
                if (ck::globaltimer_ns() - t0 > limit_ns) {
                    atomicCAS(P.err, 0, 20 + which);
                    break;
                }
            }
        }
    }
    __syncthreads();
}

// One warp per (received row, slot) pair with a local expert: its output row (y2 at the permute's
// pair position) goes to the source rank's return buffer at (token, slot).
__global__ void k_ep_return(ck_ep_peers P, const uint4 *__restrict__ y2, const int32_t *__restrict__ pair_pos2,
                            const int32_t *__restrict__ ids_own, const int32_t *__restrict__ tok_own) {
    const uint32_t K = P.nsel, vecs = P.hidden / 8;
    const size_t npairs = (size_t)P.world * P.cap * K;
    const size_t warp = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const uint32_t lane = threadIdx.x & 31;
    const size_t nwarps = ((size_t)gridDim.x * blockDim.x) >> 5;
    for (size_t q = warp; q < npairs; q += nwarps) {
        if (ids_own[q] < 0) continue;
        const size_t row = q / K;
        const uint32_t k = (uint32_t)(q - row * K), s = (uint32_t)(row / P.cap);
        const int32_t t = tok_own[row];
        const int32_t pos = pair_pos2[q];
        uint4 *dst = reinterpret_cast<uint4 *>(P.ret_y[s]) + ((size_t)t * K + k) * vecs;
        const uint4 *src = y2 + (size_t)pos * vecs;
        for (uint32_t v = lane; v < vecs; v += 32) dst[v] = src[v];
    }
}

// The destinations of the down projection's rows when its epilogue writes the return itself: for
// every (received row, slot) pair with a local expert, row_dst[its permute position] = the address
// of row token * nsel + slot in its source's return buffer (k_ep_return's mapping).
__global__ void k_ep_return_rows(ck_ep_peers P, const int32_t *__restrict__ pair_pos2,
                                 const int32_t *__restrict__ ids_own, const int32_t *__restrict__ tok_own,
                                 unsigned long long *__restrict__ row_dst) {
    const uint32_t K = P.nsel;
    const size_t npairs = (size_t)P.world * P.cap * K;
    for (size_t q = (size_t)blockIdx.x * blockDim.x + threadIdx.x; q < npairs; q += (size_t)gridDim.x * blockDim.x) {
        if (ids_own[q] < 0) continue;
        const size_t row = q / K;
        const uint32_t k = (uint32_t)(q - row * K), s = (uint32_t)(row / P.cap);
        const int32_t t = tok_own[row];
        row_dst[pair_pos2[q]] = reinterpret_cast<unsigned long long>(P.ret_y[s]) +
                                ((unsigned long long)t * K + k) * P.hidden * 2ull;
    }
}

inline cudaStream_t S(void *s) { return reinterpret_cast<cudaStream_t>(s); }

int check(const ck_ep_peers *P) {
    if (!P || P->world == 0 || P->world > CK_EP_MAX_RANKS || P->rank >= P->world || P->cap == 0 || P->nsel == 0 ||
        P->nsel > 16 || P->hidden == 0 || P->hidden % 8 || !P->ctr || !P->err || !P->my_dflags || !P->my_rflags)
        return CK_EARG;
    for (uint32_t d = 0; d < P->world; ++d)
        if (!P->recv_x[d] || !P->recv_ids[d] || !P->recv_w[d] || !P->recv_tok[d] || !P->ret_y[d] || !P->dflag[d] ||
            !P->rflag[d])
            return CK_EARG;
    return 0;
}
int grid_for(size_t warps) {
    const size_t blocks = (warps * 32 + 255) / 256;
    return (int)(blocks < 1 ? 1 : blocks > 4 * 148 ? 4 * 148 : blocks);
}

}  // namespace

extern "C" {

int ck_ep_arena_alloc(size_t bytes, void **dev_ptr_out) {
    if (!dev_ptr_out || bytes == 0) return CK_EARG;
    cudaError_t e = cudaMalloc(dev_ptr_out, bytes);
    if (e == cudaSuccess) e = cudaMemset(*dev_ptr_out, 0, bytes);
    return (int)e;
}
int ck_ep_arena_free(void *dev_ptr) { return dev_ptr ? (int)cudaFree(dev_ptr) : CK_EARG; }

int ck_ipc_get_handle(const void *dev_ptr, void *handle_out) {
    if (!dev_ptr || !handle_out) return CK_EARG;
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void *>(dev_ptr));
    if (e != cudaSuccess) return (int)e;
    memcpy(handle_out, &h, sizeof(h));
    return 0;
}
int ck_ipc_open_handle(const void *handle, void **dev_ptr_out) {
    if (!handle || !dev_ptr_out) return CK_EARG;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    return (int)cudaIpcOpenMemHandle(dev_ptr_out, h, cudaIpcMemLazyEnablePeerAccess);
}
int ck_ipc_close(void *dev_ptr) { return dev_ptr ? (int)cudaIpcCloseMemHandle(dev_ptr) : CK_EARG; }

int ck_ep_peer_status(const ck_ep_peers *P, void *s) {
    if (int rc = check(P)) return rc;
    int e = 0;
    cudaError_t r = cudaMemcpyAsync(&e, P->err, 4, cudaMemcpyDeviceToHost, S(s));
    if (r == cudaSuccess) r = cudaStreamSynchronize(S(s));
    if (r != cudaSuccess) return (int)r;
    return e ? CK_ETIMEOUT : 0;
}
int ck_ep_peer_begin(const ck_ep_peers *P, void *s) {
    if (int rc = check(P)) return rc;
    k_ep_begin<<<1, 32, 0, S(s)>>>(P->ctr);
    return (int)cudaGetLastError();
}
int ck_ep_peer_dispatch(const ck_ep_peers *P, const void *x_bf16_dev, const int32_t *send_tok_dev,
                        const int32_t *meta_dev, const int64_t *sizes_dev, uint32_t ntok, void *s) {
    if (int rc = check(P)) return rc;
    if (!x_bf16_dev || !send_tok_dev || !meta_dev || !sizes_dev || ntok > P->cap) return CK_EARG;
    const uint32_t max_rows = ntok * (P->world < P->nsel ? P->world : P->nsel);
    const int g = grid_for(max_rows > P->cap ? max_rows : P->cap);
    k_ep_dispatch<<<g, 256, 0, S(s)>>>(*P, reinterpret_cast<const uint4 *>(x_bf16_dev), send_tok_dev, meta_dev,
                                      reinterpret_cast<const long long *>(sizes_dev), max_rows);
    return (int)cudaGetLastError();
}
int ck_ep_peer_signal(const ck_ep_peers *P, int which, void *s) {
    if (int rc = check(P)) return rc;
    k_ep_signal<<<1, CK_EP_MAX_RANKS, 0, S(s)>>>(*P, which ? 1 : 0);
    return (int)cudaGetLastError();
}
int ck_ep_peer_wait(const ck_ep_peers *P, int which, uint64_t limit_ns, void *s) {
    if (int rc = check(P)) return rc;
    if (limit_ns == 0 || limit_ns > 10000000000ull) return CK_EARG;
    k_ep_wait<<<1, CK_EP_MAX_RANKS, 0, S(s)>>>(*P, which ? 1 : 0, limit_ns);
    return (int)cudaGetLastError();
}
int ck_ep_peer_return(const ck_ep_peers *P, const void *y2_bf16_dev, const int32_t *pair_pos2_dev,
                      const int32_t *ids_own_dev, const int32_t *tok_own_dev, void *s) {
    if (int rc = check(P)) return rc;
    if (!y2_bf16_dev || !pair_pos2_dev || !ids_own_dev || !tok_own_dev) return CK_EARG;
    const size_t npairs = (size_t)P->world * P->cap * P->nsel;
    k_ep_return<<<grid_for(npairs), 256, 0, S(s)>>>(*P, reinterpret_cast<const uint4 *>(y2_bf16_dev), pair_pos2_dev,
                                                   ids_own_dev, tok_own_dev);
    return (int)cudaGetLastError();
}

int ck_ep_peer_return_rows(const ck_ep_peers *P, const int32_t *pair_pos2_dev, const int32_t *ids_own_dev,
                           const int32_t *tok_own_dev, unsigned long long *row_dst_dev, void *s) {
    if (int rc = check(P)) return rc;
    if (!pair_pos2_dev || !ids_own_dev || !tok_own_dev || !row_dst_dev) return CK_EARG;
    const size_t npairs = (size_t)P->world * P->cap * P->nsel;
    k_ep_return_rows<<<grid_for((npairs + 31) / 32), 256, 0, S(s)>>>(*P, pair_pos2_dev, ids_own_dev, tok_own_dev,
                                                                     row_dst_dev);
    return (int)cudaGetLastError();
}

}  // extern "C"
