// ep_group.cu -- one process driving the expert-parallel MoE layer over several GPUs of one box.
//
// The reference's MoE runs on one device (there is no counterpart).  A host that owns the box's
// GPUs in a single process -- the reference runtime with this carrier linked in is one, since its
// Form ABI sees one device -- creates a group: every member GPU gets its share of the experts
// (E / world of them, copied once from a full set of weights anywhere in device memory), replicas
// of the router and shared expert(s), its own stream and one block of device memory, and the
// members reach each other's exchange arenas through peer access (cudaDeviceEnablePeerAccess).
// A forward splits the caller's tokens evenly over the members, runs on each member exactly the
// sequence a rank of PeerExpertParallelMoE runs (route, dispatch plan, shared expert, dispatch
// stores, barrier, regroup, expert GEMMs, return stores, barrier, combine; ep_peer.cu), and
// gathers ids, weights, per-expert counts and outputs back to the caller's device.  The host
// issues every member's work without waiting, phase by phase across the members (member_forward):
// members meet only at the bounded device barriers.
#include "../../include/ck_b200.h"
#include "ck_common.cuh"
#include "ck_launch.h"

#include <stdlib.h>
#include <string.h>

namespace {

inline size_t al(size_t b) { return (b + 255) & ~(size_t)255; }
constexpr uint64_t WAIT_NS = 10000000000ull;

struct Member {
    int dev;
    cudaStream_t st;
    cudaEvent_t done;
    uint8_t *mem;
    // weights
    uint8_t *wg, *wu, *wd, *sg, *su, *sd;
    float *router, *bias;
    // source side
    uint16_t *x, *out;
    float *logits, *wts;
    int32_t *ids, *send_tok, *send_meta, *ret_pos, *counts, *iota;
    int64_t *sizes;
    uint8_t *route_ws;
    size_t route_ws_bytes;
    uint16_t *h_sh;
    int4 *sh_tiles;
    int32_t *sh_ntiles;
    // receiver side
    uint16_t *xp2, *h2, *y2;
    float *row_w2;
    int32_t *pair_pos2, *counts2, *ntiles2;
    int4 *tiles2;
    uint8_t *perm_ws2;
    uint32_t mt2;
    // exchange arena: flags | recv_x | recv_ids | recv_w | recv_tok | ret_y
    uint8_t *arena;
    size_t a_recv_x, a_recv_ids, a_recv_w, a_recv_tok, a_ret_y;
    ck_ep_peers peers;
};

__global__ void k_iota(int32_t *v, uint32_t n) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) v[i] = (int32_t)i;
}
__global__ void k_sum_counts(const int32_t *__restrict__ parts, int32_t *__restrict__ out, uint32_t world,
                             uint32_t E) {
    const uint32_t e = blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= E) return;
    int32_t s = 0;
    for (uint32_t d = 0; d < world; ++d) s += parts[(size_t)d * E + e];
    out[e] = s;
}

}  // namespace

struct ck_ep_group {
    uint32_t world, cap, el;
    ck_moe_config cfg;
    Member m[CK_EP_MAX_RANKS];
    int32_t *count_parts;  // on the first member's device: [world][E]
    int loaded;
};

namespace {

int setup_member(ck_ep_group *g, uint32_t d, int dev) {
    Member &m = g->m[d];
    const ck_moe_config &c = g->cfg;
    const uint32_t W = g->world, T = g->cap, K = c.nsel, H = c.hidden, I = c.inter, E = c.n_experts,
                   NS = c.n_shared;
    const size_t mb = (size_t)I * H / 256 * 144;
    const size_t R = (size_t)W * T, P = R * K, SR = (size_t)T * (W < K ? W : K);
    m.dev = dev;
    cudaError_t e = cudaSetDevice(dev);
    if (e != cudaSuccess) return (int)e;
    m.route_ws_bytes = ck_moe_route_workspace_bytes(&c, T);
    m.mt2 = ck_moe_max_tiles((uint32_t)R, K, g->el, 0);
    const size_t perm2 = ck_moe_permute_workspace_bytes((uint32_t)R, K, g->el);
    // one allocation per member, carved in this order
    size_t o = 0;
    struct Part {
        void **p;
        size_t bytes;
    } parts[] = {
        {(void **)&m.wg, g->el * mb}, {(void **)&m.wu, g->el * mb}, {(void **)&m.wd, g->el * mb},
        {(void **)&m.sg, NS * mb}, {(void **)&m.su, NS * mb}, {(void **)&m.sd, NS * mb},
        {(void **)&m.router, (size_t)E * H * 4}, {(void **)&m.bias, (size_t)E * 4},
        {(void **)&m.x, (size_t)T * H * 2}, {(void **)&m.out, (size_t)T * H * 2},
        {(void **)&m.logits, (size_t)T * E * 4}, {(void **)&m.ids, (size_t)T * K * 4},
        {(void **)&m.wts, (size_t)T * K * 4}, {(void **)&m.send_tok, SR * 4}, {(void **)&m.send_meta, SR * 2 * K * 4},
        {(void **)&m.sizes, (size_t)W * 16}, {(void **)&m.ret_pos, (size_t)T * K * 4}, {(void **)&m.counts, (size_t)E * 4},
        {(void **)&m.iota, (size_t)T * K * 4}, {(void **)&m.route_ws, m.route_ws_bytes},
        {(void **)&m.h_sh, (size_t)(NS ? NS : 1) * T * I * 2}, {(void **)&m.sh_tiles, ((size_t)T / 5 + 2) * 16},
        {(void **)&m.sh_ntiles, 4}, {(void **)&m.xp2, P * H * 2}, {(void **)&m.row_w2, P * 4},
        {(void **)&m.pair_pos2, P * 4}, {(void **)&m.counts2, (size_t)g->el * 4}, {(void **)&m.tiles2, (size_t)m.mt2 * 16},
        {(void **)&m.ntiles2, 4}, {(void **)&m.perm_ws2, perm2}, {(void **)&m.h2, P * I * 2},
        {(void **)&m.y2, P * H * 2}, {(void **)&m.arena, 0},
    };
    const size_t nparts = sizeof(parts) / sizeof(parts[0]);
    size_t offs[64];
    for (size_t i = 0; i + 1 < nparts; ++i) {
        offs[i] = o;
        o += al(parts[i].bytes);
    }
    offs[nparts - 1] = o;
    // the arena
    size_t a = 0;
    const size_t a_flags = a;
    a += 1024;
    m.a_recv_x = a;
    a += al(R * H * 2);
    m.a_recv_ids = a;
    a += al(R * K * 4);
    m.a_recv_w = a;
    a += al(R * K * 4);
    m.a_recv_tok = a;
    a += al(R * 4);
    m.a_ret_y = a;
    a += al((size_t)T * (K + NS) * H * 2);
    (void)a_flags;
    e = cudaMalloc(&m.mem, o + a);
    if (e != cudaSuccess) return (int)e;
    for (size_t i = 0; i < nparts; ++i) *parts[i].p = m.mem + offs[i];
    e = cudaMemset(m.arena, 0, a);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&m.st, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&m.done, cudaEventDisableTiming);
    if (e != cudaSuccess) return (int)e;
    k_iota<<<(T * K + 255) / 256, 256, 0, m.st>>>(m.iota, T * K);
    return (int)cudaGetLastError();
}

void fill_peers(ck_ep_group *g) {
    const uint32_t W = g->world, T = g->cap, K = g->cfg.nsel, H = g->cfg.hidden;
    for (uint32_t me = 0; me < W; ++me) {
        ck_ep_peers &p = g->m[me].peers;
        memset(&p, 0, sizeof(p));
        p.world = W;
        p.rank = me;
        p.cap = T;
        p.nsel = K;
        p.hidden = H;
        for (uint32_t d = 0; d < W; ++d) {
            uint8_t *b = g->m[d].arena;
            p.recv_x[d] = b + g->m[d].a_recv_x + (size_t)me * T * H * 2;
            p.recv_ids[d] = (int32_t *)(b + g->m[d].a_recv_ids + (size_t)me * T * K * 4);
            p.recv_w[d] = (float *)(b + g->m[d].a_recv_w + (size_t)me * T * K * 4);
            p.recv_tok[d] = (int32_t *)(b + g->m[d].a_recv_tok + (size_t)me * T * 4);
            p.ret_y[d] = b + g->m[d].a_ret_y;
            p.dflag[d] = (unsigned long long *)(b + 8 * me);
            p.rflag[d] = (unsigned long long *)(b + 256 + 8 * me);
        }
        uint8_t *own = g->m[me].arena;
        p.my_dflags = (unsigned long long *)own;
        p.my_rflags = (unsigned long long *)(own + 256);
        p.ctr = (unsigned long long *)(own + 512);
        p.err = (int *)(own + 520);
    }
}

// One member's forward over its T tokens, issued on its stream in three phases: 0 up to the
// dispatch signal, 1 from the dispatch barrier to the return signal, 2 from the return barrier on.
// The group issues phase p of every member before phase p + 1 of any: a member's barrier then only
// ever waits on work already queued on its peers, so no host call that blocks until a device is
// idle (a kernel's first launch on a device loads its module) can wait on a barrier whose signal
// the host has not issued yet.
int member_forward(ck_ep_group *g, uint32_t d, uint32_t T, int phase) {
    Member &m = g->m[d];
    const ck_moe_config &c = g->cfg;
    const uint32_t W = g->world, K = c.nsel, H = c.hidden, I = c.inter, E = c.n_experts, NS = c.n_shared;
    const uint32_t R = W * g->cap;
    const uint64_t mb = (uint64_t)I * H / 256 * 144;
    void *s = m.st;
    const ck_ep_peers *pe = &m.peers;
    int rc = cudaSetDevice(m.dev);
    uint8_t *ret_y = m.arena + m.a_ret_y;
    int32_t *rids = (int32_t *)(m.arena + m.a_recv_ids);
    if (phase == 2) {
        if (!rc) rc = ck_ep_peer_wait(pe, 1, WAIT_NS, s);
        if (!rc && T)
            rc = ck_moe_combine(ret_y, m.ids, m.wts, m.iota, T, K, NS, H, c.mode == 3, m.out, nullptr, s);
        return rc;
    }
    if (phase == 1) {
        if (!rc) rc = ck_ep_peer_wait(pe, 0, WAIT_NS, s);
        if (!rc)
            rc = ck_moe_permute(rids, (const float *)(m.arena + m.a_recv_w), m.arena + m.a_recv_x, R, K, g->el, 0, H,
                                c.mode == 4, m.xp2, m.row_w2, m.pair_pos2, m.counts2, m.tiles2, m.ntiles2, m.perm_ws2,
                                s);
        const uint32_t bound = R <= CK_MOE_DECODE_TOKENS ? (R < CK_MOE_FEW_TOKENS ? R : CK_MOE_FEW_TOKENS) : 0;
        if (!rc)
            rc = ck_moe_expert_gemm_bounded(1, m.wg, m.wu, nullptr, nullptr, mb, g->el, 0, m.xp2, R * K, m.h2, R * K,
                                            m.row_w2, m.tiles2, m.ntiles2, m.mt2, I, H, 0, bound, pe->err, s);
        const int32_t *rtok = (const int32_t *)(m.arena + m.a_recv_tok);
        if (bound) {
            if (!rc)
                rc = ck_moe_expert_gemm_bounded(0, m.wd, nullptr, nullptr, nullptr, mb, g->el, 0, m.h2, R * K, m.y2,
                                                R * K, nullptr, m.tiles2, m.ntiles2, m.mt2, H, I, 1, bound, pe->err, s);
            if (!rc) rc = ck_ep_peer_return(pe, m.y2, m.pair_pos2, rids, rtok, s);
        } else {
            // the down projection stores every row in its source's return buffer itself; the row
            // table (8 bytes a pair) lives in the y2 block, which it does not otherwise need
            unsigned long long *row_dst = reinterpret_cast<unsigned long long *>(m.y2);
            if (!rc) rc = ck_ep_peer_return_rows(pe, m.pair_pos2, rids, rtok, row_dst, s);
            if (!rc)
                rc = ck_moe_expert_gemm_rows(m.wd, mb, g->el, m.h2, R * K, row_dst, R * K, m.tiles2, m.ntiles2, m.mt2,
                                             H, I, 1, pe->err, s);
        }
        if (!rc) rc = ck_ep_peer_signal(pe, 1, s);
        return rc;
    }
    if (!rc) rc = ck_ep_peer_begin(pe, s);
    if (!rc && T) rc = ck_moe_route(&c, m.x, T, m.router, m.bias, m.logits, m.ids, m.wts, m.route_ws, m.route_ws_bytes, s);
    if (!rc) rc = ck_ep_dispatch_plan(m.ids, m.wts, T, K, E, W, m.counts, m.sizes, m.send_tok, m.send_meta, m.ret_pos, s);
    if (!rc && NS && T) {
        const uint32_t bound = T <= CK_MOE_DECODE_TOKENS ? (T < CK_MOE_FEW_TOKENS ? T : CK_MOE_FEW_TOKENS) : 0;
        rc = ck_token_tiles_n(m.sh_tiles, m.sh_ntiles, T, bound ? CK_MOE_FEW_TOKENS : 192, s);
        const uint32_t ntab = T / 5 + 2;
        for (uint32_t sh = 0; !rc && sh < NS; ++sh) {
            uint16_t *hs = m.h_sh + (size_t)sh * T * I;
            uint8_t *ys = ret_y + ((size_t)T * K + (size_t)sh * T) * H * 2;
            rc = ck_moe_expert_gemm_bounded(1, m.sg + sh * mb, m.su + sh * mb, nullptr, nullptr, 0, 1, 0, m.x, T, hs, T,
                                            nullptr, m.sh_tiles, m.sh_ntiles, ntab, I, H, 0, bound, pe->err, s);
            if (!rc)
                rc = ck_moe_expert_gemm_bounded(0, m.sd + sh * mb, nullptr, nullptr, nullptr, 0, 1, 0, hs, T, ys, T,
                                                nullptr, m.sh_tiles, m.sh_ntiles, ntab, H, I, 0, bound, pe->err, s);
        }
    }
    if (!rc) rc = ck_ep_peer_dispatch(pe, m.x, m.send_tok, m.send_meta, m.sizes, T, s);
    if (!rc) rc = ck_ep_peer_signal(pe, 0, s);
    return rc;
}

}  // namespace

extern "C" {

ck_ep_group *ck_ep_group_create(const ck_moe_config *cfg, uint32_t world, const int *devices, uint32_t cap) {
    if (!cfg || !devices || world < 1 || world > CK_EP_MAX_RANKS || cap == 0) return nullptr;
    if (ck_moe_workspace_bytes(cfg, cap) == 0 || cfg->n_experts % world || cfg->hidden % 256 || cfg->inter % 256)
        return nullptr;
    int prev = 0;
    cudaGetDevice(&prev);
    ck_ep_group *g = (ck_ep_group *)calloc(1, sizeof(ck_ep_group));
    if (!g) return nullptr;
    g->world = world;
    g->cap = cap;
    g->el = cfg->n_experts / world;
    g->cfg = *cfg;
    bool ok = true;
    for (uint32_t d = 0; d < world && ok; ++d) ok = setup_member(g, d, devices[d]) == 0;
    for (uint32_t a = 0; a < world && ok; ++a) {
        cudaSetDevice(devices[a]);
        for (uint32_t b = 0; b < world; ++b) {
            if (a == b || devices[a] == devices[b]) continue;
            int can = 0;
            cudaDeviceCanAccessPeer(&can, devices[a], devices[b]);
            if (!can) {
                ok = false;
                break;
            }
            const cudaError_t e = cudaDeviceEnablePeerAccess(devices[b], 0);
            if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled) ok = false;
            cudaGetLastError();
        }
    }
    if (ok) {
        cudaSetDevice(devices[0]);
        ok = cudaMalloc(&g->count_parts, (size_t)world * cfg->n_experts * 4) == cudaSuccess;
    }
    if (ok) fill_peers(g);
    for (uint32_t d = 0; d < world && ok; ++d) {
        cudaSetDevice(devices[d]);
        ok = cudaDeviceSynchronize() == cudaSuccess;
    }
    cudaSetDevice(prev);
    if (!ok) {
        ck_ep_group_destroy(g);
        return nullptr;
    }
    return g;
}

int ck_ep_group_load(ck_ep_group *g, const void *w_gate, const void *w_up, const void *w_down, const void *s_gate,
                     const void *s_up, const void *s_down, const float *router_w, const float *bias) {
    if (!g || !w_gate || !w_up || !w_down || !router_w || (g->cfg.mode == 4 && !bias) ||
        (g->cfg.n_shared && (!s_gate || !s_up || !s_down)))
        return CK_EARG;
    const ck_moe_config &c = g->cfg;
    const size_t mb = (size_t)c.inter * c.hidden / 256 * 144, sh = (size_t)g->el * mb;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaError_t e = cudaSuccess;
    for (uint32_t d = 0; d < g->world && e == cudaSuccess; ++d) {
        Member &m = g->m[d];
        cudaSetDevice(m.dev);
        const size_t off = (size_t)d * sh;
        e = cudaMemcpy(m.wg, (const uint8_t *)w_gate + off, sh, cudaMemcpyDefault);
        if (e == cudaSuccess) e = cudaMemcpy(m.wu, (const uint8_t *)w_up + off, sh, cudaMemcpyDefault);
        if (e == cudaSuccess) e = cudaMemcpy(m.wd, (const uint8_t *)w_down + off, sh, cudaMemcpyDefault);
        if (e == cudaSuccess && c.n_shared) {
            e = cudaMemcpy(m.sg, s_gate, c.n_shared * mb, cudaMemcpyDefault);
            if (e == cudaSuccess) e = cudaMemcpy(m.su, s_up, c.n_shared * mb, cudaMemcpyDefault);
            if (e == cudaSuccess) e = cudaMemcpy(m.sd, s_down, c.n_shared * mb, cudaMemcpyDefault);
        }
        if (e == cudaSuccess) e = cudaMemcpy(m.router, router_w, (size_t)c.n_experts * c.hidden * 4, cudaMemcpyDefault);
        if (e == cudaSuccess && bias) e = cudaMemcpy(m.bias, bias, (size_t)c.n_experts * 4, cudaMemcpyDefault);
    }
    cudaSetDevice(prev);
    if (e == cudaSuccess) g->loaded = 1;
    return (int)e;
}

int ck_ep_group_forward(ck_ep_group *g, const void *x_bf16, uint32_t ntok, int32_t *ids, float *wts, int32_t *counts,
                        void *out_bf16, void *stream) {
    if (!g || !g->loaded) return CK_EARG;
    if (ntok == 0) return 0;
    if (!x_bf16 || !ids || !wts || !counts || !out_bf16) return CK_EARG;
    const uint32_t W = g->world, K = g->cfg.nsel, H = g->cfg.hidden, E = g->cfg.n_experts;
    if (ntok > W * g->cap) return CK_ESHAPE;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
    cudaEvent_t start;
    cudaEventCreateWithFlags(&start, cudaEventDisableTiming);
    cudaEventRecord(start, cs);
    int rc = 0;
    uint32_t off[CK_EP_MAX_RANKS + 1];
    off[0] = 0;
    for (uint32_t d = 0; d < W; ++d) off[d + 1] = (uint32_t)(((uint64_t)ntok * (d + 1)) / W);
    for (int phase = 0; phase < 3 && !rc; ++phase) {
        for (uint32_t d = 0; d < W && !rc; ++d) {
            Member &m = g->m[d];
            const uint32_t T = off[d + 1] - off[d];
            cudaSetDevice(m.dev);
            if (phase == 0) {
                rc = (int)cudaStreamWaitEvent(m.st, start, 0);
                if (!rc && T)
                    rc = (int)cudaMemcpyAsync(m.x, (const uint8_t *)x_bf16 + (size_t)off[d] * H * 2, (size_t)T * H * 2,
                                              cudaMemcpyDefault, m.st);
            }
            if (!rc) rc = member_forward(g, d, T, phase);
            if (phase < 2) continue;
            if (!rc && T) {
                rc = (int)cudaMemcpyAsync((uint8_t *)out_bf16 + (size_t)off[d] * H * 2, m.out, (size_t)T * H * 2,
                                          cudaMemcpyDefault, m.st);
                if (!rc)
                    rc = (int)cudaMemcpyAsync(ids + (size_t)off[d] * K, m.ids, (size_t)T * K * 4, cudaMemcpyDefault,
                                              m.st);
                if (!rc)
                    rc = (int)cudaMemcpyAsync(wts + (size_t)off[d] * K, m.wts, (size_t)T * K * 4, cudaMemcpyDefault,
                                              m.st);
            }
            if (!rc)
                rc = (int)cudaMemcpyAsync(g->count_parts + (size_t)d * E, m.counts, (size_t)E * 4, cudaMemcpyDefault,
                                          m.st);
            if (!rc) rc = (int)cudaEventRecord(m.done, m.st);
        }
    }
    cudaSetDevice(prev);
    for (uint32_t d = 0; d < W && !rc; ++d) rc = (int)cudaStreamWaitEvent(cs, g->m[d].done, 0);
    if (!rc) {
        k_sum_counts<<<(E + 255) / 256, 256, 0, cs>>>(g->count_parts, counts, W, E);
        rc = (int)cudaGetLastError();
    }
    cudaEventDestroy(start);
    return rc;
}

int ck_ep_group_status(ck_ep_group *g) {
    if (!g) return CK_EARG;
    int prev = 0, worst = 0;
    cudaGetDevice(&prev);
    for (uint32_t d = 0; d < g->world; ++d) {
        cudaSetDevice(g->m[d].dev);
        const int rc = ck_ep_peer_status(&g->m[d].peers, g->m[d].st);
        if (rc && !worst) worst = rc;
    }
    cudaSetDevice(prev);
    return worst;
}

void ck_ep_group_destroy(ck_ep_group *g) {
    if (!g) return;
    int prev = 0;
    cudaGetDevice(&prev);
    for (uint32_t d = 0; d < g->world; ++d) {
        Member &m = g->m[d];
        if (!m.mem) continue;
        cudaSetDevice(m.dev);
        if (m.st) cudaStreamSynchronize(m.st);
        cudaFree(m.mem);
        if (m.st) cudaStreamDestroy(m.st);
        if (m.done) cudaEventDestroy(m.done);
    }
    if (g->count_parts) {
        cudaSetDevice(g->m[0].dev);
        cudaFree(g->count_parts);
    }
    cudaSetDevice(prev);
    free(g);
}

}  // extern "C"
