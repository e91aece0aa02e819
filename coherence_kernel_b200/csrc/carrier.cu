// carrier.cu -- the CUDA carrier behind coherence-kernel's handle door.
//
// The reference runtime (runtime/fkwu-uni.c:951-1009) declares the door as weak C symbols and its
// Metal carrier (form/native/metal/fk-metal-carrier.m) supplies the strong ones.  This file supplies
// the same symbols for a B200: linking it into the runtime overrides the weak stubs, and Form cells
// that drive metal_pipeline / metal_buf_* / metal_enqueue / metal_sync run on sm_100a kernels with
// their argument layouts unchanged.
//
// The contract kept from the Metal carrier (fk-metal-carrier.m:29-151, 337-1071):
//   * buffer handles are (generation << 16) | slot, slot 1-based, 0 never live; freeing bumps the
//     generation so stale handles are refused;
//   * the binding string is little-endian u32: n_buf, handle[n_buf], n_const, value[n_const],
//     optionally + (threads_per_group, threadgroup_bytes) or + those and (dispatch_mode,
//     barrier_before) -- exactly three legal lengths;
//   * enqueue never waits; sync drains everything and answers the number of dispatches drained;
//     submit / fence_wait double-buffer; buf_read syncs first and answers all `len` bytes or -1;
//     buf_free only at a quiescent point; barrier_before is legal only in a concurrent batch;
//   * every failure records last_error and metal_status speaks it.
// What differs, because the memory is not unified: buffers are device allocations, and
// buf_from_file copies the file region into HBM once (a writable file region, len < 0, is written
// back at every sync).  A pipeline name resolves to a prebuilt sm_100a kernel; the MSL text is kept
// only for identity (same text + same name = same handle).  Each registered kernel checks that
// its buffers hold what its constants say it will read or write, and refuses the dispatch
// otherwise, so a wrong size in a Form cell is an error string, not a device fault.
#include "../../include/ck_b200.h"
#include "../../include/fk_cuda_carrier.h"
#include "ck_launch.h"
#include "form_kernels.h"

#include <cuda_runtime.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <map>
#include <string>
#include <vector>

namespace {

constexpr int MAX_BUF = 8192;
constexpr int MAX_PIPE = 512;

struct Buf {
    void *dev = nullptr;
    unsigned long long len = 0;
    bool live = false;
    bool file_rw = false;
    std::string path;
    long long file_off = 0;
};

struct State {
    bool up = false;
    int dev = 0;
    cudaStream_t stream = nullptr;
    char devname[256] = "none";
    std::vector<Buf> bufs;  // slot s at index s-1
    unsigned gen[MAX_BUF] = {};
    std::vector<long long> free_slots;
    std::vector<int> pipes;  // handle h -> registry index at h-1
    std::map<std::string, long long> pipe_by_key;
    bool batch_open = false;
    int batch_concurrent = 0, next_concurrent = 0;
    long long pending = 0, total_dispatch = 0, total_sync = 0;
    cudaEvent_t batch_start = nullptr;
    struct Fence {
        cudaEvent_t start, end;
        long long n;
    };
    std::map<long long, Fence> inflight;
    long long fence_next = 1;
    double gpu_busy_us = 0.0;
    std::string last_err = "none";
} g;

void err(const std::string &s) { g.last_err = s; }

bool carrier_up() {
    if (g.up) return true;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        err("no CUDA device");
        return false;
    }
    cudaGetDevice(&g.dev);
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, g.dev) == cudaSuccess) snprintf(g.devname, sizeof(g.devname), "%s", prop.name);
    if (cudaStreamCreateWithFlags(&g.stream, cudaStreamNonBlocking) != cudaSuccess) {
        err("cannot create a CUDA stream");
        return false;
    }
    g.up = true;
    return true;
}

long long buf_slot(long long h) {
    const long long slot = h & 0xFFFF, gen = h >> 16;
    if (slot < 1 || slot > (long long)g.bufs.size()) return 0;
    if (gen < 0 || gen != (long long)g.gen[slot - 1]) return 0;
    if (!g.bufs[slot - 1].live) return 0;
    return slot;
}

long long buf_register(const Buf &b) {
    long long slot;
    if (!g.free_slots.empty()) {
        slot = g.free_slots.back();
        g.free_slots.pop_back();
        g.bufs[slot - 1] = b;
    } else {
        if ((int)g.bufs.size() >= MAX_BUF) {
            err("buffer table full at 8192 live slots");
            return 0;
        }
        g.bufs.push_back(b);
        slot = (long long)g.bufs.size();
    }
    g.bufs[slot - 1].live = true;
    return ((long long)g.gen[slot - 1] << 16) | slot;
}

unsigned le32(const unsigned char *p) {
    return (unsigned)p[0] | ((unsigned)p[1] << 8) | ((unsigned)p[2] << 16) | ((unsigned)p[3] << 24);
}
float f32_of(unsigned v) {
    float f;
    memcpy(&f, &v, 4);
    return f;
}

// ------------------------------------------------------------------------------ kernel registry
struct Call {
    void *b[16];
    unsigned long long blen[16];
    unsigned c[16];
    long long threads;
    cudaStream_t s;
};
typedef int (*Launch)(const Call &, std::string &why);
struct Entry {
    const char *name;
    unsigned nbuf, nconst;
    Launch fn;
};

bool need(const Call &k, int i, unsigned long long bytes, std::string &why, const char *what) {
    if (k.blen[i] < bytes) {
        char m[256];
        snprintf(m, sizeof(m), "buffer %d (%s) holds %llu bytes, the dispatch needs %llu", i, what, k.blen[i], bytes);
        why = m;
        return false;
    }
    return true;
}
unsigned long long q80b(unsigned long long n) { return (n + 31) / 32 * 34; }
unsigned long long q4kb(unsigned long long n) { return (n + 255) / 256 * 144; }

int L_q80_dequant(const Call &k, std::string &w) {
    const unsigned long long off = k.c[0], n = k.c[1];
    if (!need(k, 0, q80b(off + n), w, "qb") || !need(k, 1, n * 4, w, "w")) return CK_ERR_ARG;
    return ck::launch_q80_dequant((const uint8_t *)k.b[0], (float *)k.b[1], off, n, k.s);
}
int L_q4k_dequant(const Call &k, std::string &w) {
    const unsigned long long off = k.c[0], n = k.c[1];
    if (!need(k, 0, q4kb(off + n), w, "qb") || !need(k, 1, n * 4, w, "w")) return CK_ERR_ARG;
    return ck::launch_q4k_dequant((const uint8_t *)k.b[0], (float *)k.b[1], off, n, k.s);
}
bool mv_check(const Call &k, bool q8, std::string &w) {
    const unsigned long long rows = k.c[0], cols = k.c[1];
    return need(k, 0, q8 ? q80b(rows * cols) : q4kb(rows * cols), w, "qb") && need(k, 1, cols * 4, w, "x") &&
           need(k, 2, rows * 4, w, "y");
}
int L_q80_attestant(const Call &k, std::string &w) {
    if (k.c[1] % 32) { w = "cols must be a multiple of 32"; return CK_ERR_SHAPE; }
    if (!mv_check(k, true, w)) return CK_ERR_ARG;
    return ck::launch_matvec_ordered(8, (const uint8_t *)k.b[0], (const float *)k.b[1], (float *)k.b[2], k.c[0], k.c[1], k.s);
}
int L_q80_fast(const Call &k, std::string &w) {
    if (k.c[1] % 32) { w = "cols must be a multiple of 32"; return CK_ERR_SHAPE; }
    if (!mv_check(k, true, w)) return CK_ERR_ARG;
    return ck::launch_q80_matvec((const uint8_t *)k.b[0], (const float *)k.b[1], (float *)k.b[2], k.c[0], k.c[1], k.s);
}
int L_q4k_attestant(const Call &k, std::string &w) {
    if (((unsigned long long)k.c[0] * k.c[1]) % 256) { w = "rows*cols must be whole superblocks"; return CK_ERR_SHAPE; }
    if (!mv_check(k, false, w)) return CK_ERR_ARG;
    return ck::launch_matvec_ordered(12, (const uint8_t *)k.b[0], (const float *)k.b[1], (float *)k.b[2], k.c[0], k.c[1], k.s);
}
int L_q4k_fast(const Call &k, std::string &w) {
    if (k.c[1] % 64) { w = "cols must be a multiple of 64"; return CK_ERR_SHAPE; }
    if (!mv_check(k, false, w)) return CK_ERR_ARG;
    return ck::launch_q4k_matvec((const uint8_t *)k.b[0], (const float *)k.b[1], (float *)k.b[2], k.c[0], k.c[1], 1, k.s);
}
int L_q4k_part(const Call &k, std::string &w) {
    const unsigned long long rows = k.c[0], cols = k.c[1], parts = k.c[2];
    if (parts == 0) { w = "parts must be positive"; return CK_ERR_ARG; }
    if (!need(k, 0, q4kb(rows * cols), w, "qb") || !need(k, 1, cols * 4, w, "x") || !need(k, 2, rows * parts * 4, w, "part"))
        return CK_ERR_ARG;
    return ck::launch_q4k_part((const uint8_t *)k.b[0], (const float *)k.b[1], (float *)k.b[2], k.c[0], k.c[1], k.c[2], k.s);
}
int L_part_combine(const Call &k, std::string &w) {
    const unsigned long long rows = k.c[0], parts = k.c[1];
    if (!need(k, 0, rows * parts * 4, w, "part") || !need(k, 1, rows * 4, w, "y")) return CK_ERR_ARG;
    return ck::launch_part_combine((const float *)k.b[0], (float *)k.b[1], k.c[0], k.c[1], k.s);
}
int L_q4k_matmul_batch(const Call &k, std::string &w) {
    const unsigned long long rows = k.c[0], cols = k.c[1], ntok = k.c[2];
    if (cols % 64 || ntok == 0) { w = "cols must be a multiple of 64 and ntok positive"; return CK_ERR_SHAPE; }
    if (!need(k, 0, q4kb(rows * cols), w, "qb") || !need(k, 1, ntok * cols * 4, w, "x") ||
        !need(k, 2, ntok * rows * 4, w, "y"))
        return CK_ERR_ARG;
    return ck::launch_q4k_matvec((const uint8_t *)k.b[0], (const float *)k.b[1], (float *)k.b[2], k.c[0], k.c[1], k.c[2], k.s);
}
// ---- Q6_K (q6k-msl.fk, qk-matvec-lane.fk, qk-matvec-slot.fk, qk-matvec-split.fk, qk-matmul-batch.fk)
unsigned long long q6kb(unsigned long long n) { return (n + 255) / 256 * 210; }
int L_q6k_dequant(const Call &k, std::string &w) {
    const unsigned long long off = k.c[0], n = k.c[1];
    if (!need(k, 0, q6kb(off + n), w, "qb") || !need(k, 1, n * 4, w, "w")) return CK_ERR_ARG;
    return ck::launch_q6k_dequant((const uint8_t *)k.b[0], (float *)k.b[1], off, n, k.s);
}
bool q6_mv_check(const Call &k, std::string &w) {
    const unsigned long long rows = k.c[0], cols = k.c[1];
    if ((rows * cols) % 256) { w = "rows*cols must be whole superblocks"; return false; }
    return need(k, 0, q6kb(rows * cols), w, "qb") && need(k, 1, cols * 4, w, "x") && need(k, 2, rows * 4, w, "y");
}
int L_q6k_attestant(const Call &k, std::string &w) {
    if (!q6_mv_check(k, w)) return CK_ERR_ARG;
    return ck::launch_q6k_ordered((const uint8_t *)k.b[0], (const float *)k.b[1], (float *)k.b[2], k.c[0], k.c[1], k.s);
}
int L_q6k_fast(const Call &k, std::string &w) {
    if (!q6_mv_check(k, w)) return CK_ERR_ARG;
    return ck::launch_q6k_matvec((const uint8_t *)k.b[0], (const float *)k.b[1], (float *)k.b[2], k.c[0], k.c[1], 1,
                                 k.s);
}
int L_q6k_part(const Call &k, std::string &w) {
    const unsigned long long rows = k.c[0], cols = k.c[1], parts = k.c[2];
    if (parts == 0) { w = "parts must be positive"; return CK_ERR_ARG; }
    if ((rows * cols) % 256) { w = "rows*cols must be whole superblocks"; return CK_ERR_SHAPE; }
    if (!need(k, 0, q6kb(rows * cols), w, "qb") || !need(k, 1, cols * 4, w, "x") || !need(k, 2, rows * parts * 4, w, "part"))
        return CK_ERR_ARG;
    return ck::launch_q6k_part((const uint8_t *)k.b[0], (const float *)k.b[1], (float *)k.b[2], k.c[0], k.c[1], k.c[2],
                               k.s);
}
int L_q6k_matmul_batch(const Call &k, std::string &w) {
    const unsigned long long rows = k.c[0], cols = k.c[1], ntok = k.c[2];
    if ((rows * cols) % 256 || ntok == 0) { w = "rows*cols must be whole superblocks and ntok positive"; return CK_ERR_SHAPE; }
    if (!need(k, 0, q6kb(rows * cols), w, "qb") || !need(k, 1, ntok * cols * 4, w, "x") ||
        !need(k, 2, ntok * rows * 4, w, "y"))
        return CK_ERR_ARG;
    return ck::launch_q6k_matvec((const uint8_t *)k.b[0], (const float *)k.b[1], (float *)k.b[2], k.c[0], k.c[1],
                                 k.c[2], k.s);
}
int L_f16_matvec(const Call &k, std::string &w) {
    const unsigned long long rows = k.c[0], cols = k.c[1];
    if (!need(k, 0, rows * cols * 2, w, "qb") || !need(k, 1, cols * 4, w, "x") || !need(k, 2, rows * 4, w, "y"))
        return CK_ERR_ARG;
    return ck::launch_f16_matvec((const uint16_t *)k.b[0], (const float *)k.b[1], (float *)k.b[2], k.c[0], k.c[1], k.s);
}
int route_common(const Call &k, unsigned cap, std::string &w) {
    const unsigned ne = k.c[0], nsel = k.c[1];
    if (ne > cap || nsel > 8 || nsel > ne || ne == 0 || nsel == 0) {
        w = "router needs 0 < nsel <= 8, nsel <= ne <= " + std::to_string(cap);
        return CK_ERR_SHAPE;
    }
    if (!need(k, 0, (unsigned long long)ne * 4, w, "logits") || !need(k, 1, nsel * 4ull, w, "ids") ||
        !need(k, 2, nsel * 4ull, w, "wts"))
        return CK_ERR_ARG;
    return ck::launch_route_softmax_tokens((const float *)k.b[0], (uint32_t *)k.b[1], (float *)k.b[2], ne, nsel, 1, 1, k.s);
}
int L_route(const Call &k, std::string &w) { return route_common(k, 64, w); }
int L_route_wide(const Call &k, std::string &w) { return route_common(k, 256, w); }
int L_dsv4_router(const Call &k, std::string &w) {
    const unsigned ne = k.c[0], nused = k.c[1];
    if (ne > 256 || nused > 8 || nused > ne || ne == 0 || nused == 0) { w = "dsv4 router needs nused <= 8, ne <= 256"; return CK_ERR_SHAPE; }
    if (!need(k, 0, ne * 4ull, w, "logits") || !need(k, 1, ne * 4ull, w, "bias") || !need(k, 2, nused * 4ull, w, "ids") ||
        !need(k, 3, nused * 4ull, w, "wts"))
        return CK_ERR_ARG;
    return ck::launch_route_dsv4_tokens((const float *)k.b[0], (const float *)k.b[1], (uint32_t *)k.b[2], (float *)k.b[3],
                                        ne, nused, f32_of(k.c[2]), 1, k.s);
}
int L_dsv4_swiglu(const Call &k, std::string &w) {
    const unsigned long long n = k.c[0];
    if (!need(k, 0, n * 4, w, "gate") || !need(k, 1, n * 4, w, "up") || !need(k, 2, n * 4, w, "out")) return CK_ERR_ARG;
    return ck::launch_swiglu((const float *)k.b[0], (const float *)k.b[1], (float *)k.b[2], k.c[0], f32_of(k.c[1]),
                             f32_of(k.c[2]), k.s);
}
int L_swiglu(const Call &k, std::string &w) {
    const unsigned long long n = k.c[0];
    if (!need(k, 0, n * 4, w, "g") || !need(k, 1, n * 4, w, "u") || !need(k, 2, n * 4, w, "y")) return CK_ERR_ARG;
    return ck::launch_swiglu_plain((const float *)k.b[0], (const float *)k.b[1], (float *)k.b[2], k.c[0], k.s);
}
int L_scale(const Call &k, std::string &w) {
    const unsigned long long n = k.c[1];
    if (!need(k, 0, n * 4, w, "x") || !need(k, 1, n * 4, w, "y")) return CK_ERR_ARG;
    return ck::launch_scale((const float *)k.b[0], (float *)k.b[1], f32_of(k.c[0]), k.c[1], k.s);
}
int L_axpy(const Call &k, std::string &w) {
    const unsigned long long n = k.c[1];
    if (!need(k, 0, n * 4, w, "x") || !need(k, 1, n * 4, w, "y")) return CK_ERR_ARG;
    return ck::launch_axpy((const float *)k.b[0], (float *)k.b[1], f32_of(k.c[0]), k.c[1], k.s);
}
int L_f32_matvec(const Call &k, std::string &w) {
    const unsigned long long rows = k.c[0], cols = k.c[1];
    if (!need(k, 0, rows * cols * 4, w, "W") || !need(k, 1, cols * 4, w, "x") || !need(k, 2, rows * 4, w, "y"))
        return CK_ERR_ARG;
    return ck::launch_f32_matvec((const float *)k.b[0], (const float *)k.b[1], (float *)k.b[2], k.c[0], k.c[1], k.s);
}
int L_swiglu_experts(const Call &k, std::string &w) {
    const unsigned long long n = k.c[0], ne = k.c[1];
    if (!need(k, 0, n * ne * 4, w, "gate") || !need(k, 1, n * ne * 4, w, "up") || !need(k, 2, n * ne * 4, w, "out") ||
        !need(k, 3, ne * 4, w, "wts"))
        return CK_ERR_ARG;
    return ck::launch_swiglu_experts((const float *)k.b[0], (const float *)k.b[1], (float *)k.b[2], (const float *)k.b[3],
                                     k.c[0], k.c[1], f32_of(k.c[2]), k.s);
}
int L_moe_reduce(const Call &k, std::string &w) {
    const unsigned long long n = k.c[0], ne = k.c[1];
    if (!need(k, 0, n * ne * 4, w, "parts") || !need(k, 1, n * 4, w, "out")) return CK_ERR_ARG;
    return ck::launch_moe_reduce((const float *)k.b[0], (float *)k.b[1], k.c[0], k.c[1], k.s);
}
// ck_moe_layer_bf16: buffers x wg wu wd sg su sd router bias ids wts counts out workspace;
// constants hidden inter ne nshared nsel mode ngroups topk_groups wscale(f32) tau(f32) ntok
int L_moe_layer(const Call &k, std::string &w) {
    ck_moe_config c = {k.c[0], k.c[1], k.c[2], k.c[3], k.c[4], k.c[5], k.c[6], k.c[7], f32_of(k.c[8]), f32_of(k.c[9])};
    const unsigned long long T = k.c[10], H = c.hidden, I = c.inter, E = c.n_experts, NS = c.n_shared, K = c.nsel;
    const size_t ws = ck_moe_workspace_bytes(&c, (uint32_t)T);
    if (ws == 0) { w = "unsupported MoE configuration"; return CK_ERR_SHAPE; }
    const unsigned long long mb = q4kb(I * H);
    if (!need(k, 0, T * H * 2, w, "x") || !need(k, 1, E * mb, w, "w_gate") || !need(k, 2, E * mb, w, "w_up") ||
        !need(k, 3, E * mb, w, "w_down") || !need(k, 4, NS * mb, w, "s_gate") || !need(k, 5, NS * mb, w, "s_up") ||
        !need(k, 6, NS * mb, w, "s_down") || !need(k, 7, E * H * 4, w, "router") ||
        !need(k, 8, c.mode == 4 ? E * 4 : 0, w, "bias") || !need(k, 9, T * K * 4, w, "ids") ||
        !need(k, 10, T * K * 4, w, "wts") || !need(k, 11, E * 4, w, "counts") || !need(k, 12, T * H * 2, w, "out") ||
        !need(k, 13, ws, w, "workspace"))
        return CK_ERR_ARG;
    return ck_moe_layer_bf16(&c, k.b[0], (uint32_t)T, k.b[1], k.b[2], k.b[3], k.b[4], k.b[5], k.b[6], (const float *)k.b[7],
                             (const float *)k.b[8], (int32_t *)k.b[9], (float *)k.b[10], (int32_t *)k.b[11], k.b[12],
                             k.b[13], k.blen[13], k.s);
}
// ck_moe_layer_ep_bf16: the same 14 buffers and 11 constants as ck_moe_layer_bf16, then `world`:
// the layer over GPUs carrier_dev .. carrier_dev + world - 1 (modulo the device count) as one
// expert-parallel group.  The group is built at the first dispatch for a set of weight buffers
// (experts shared out to the members once) and kept for later dispatches with the same weights,
// configuration and width; the workspace buffer is not used.
struct EpKey {
    const void *wg, *wu, *wd;
    unsigned world, ntok_cap;
    ck_moe_config cfg;
};
struct EpEntry {
    EpKey key;
    ck_ep_group *g;
};
std::vector<EpEntry> g_ep_groups;
int L_moe_layer_ep(const Call &k, std::string &w) {
    ck_moe_config c = {k.c[0], k.c[1], k.c[2], k.c[3], k.c[4], k.c[5], k.c[6], k.c[7], f32_of(k.c[8]), f32_of(k.c[9])};
    const unsigned long long T = k.c[10], H = c.hidden, I = c.inter, E = c.n_experts, NS = c.n_shared, K = c.nsel;
    const unsigned world = k.c[11];
    int ndev = 0, dev = 0;
    cudaGetDeviceCount(&ndev);
    cudaGetDevice(&dev);
    if (world == 0 || world > CK_EP_MAX_RANKS || (int)world > ndev || E % world) {
        w = "ck_moe_layer_ep_bf16 needs 1 <= world <= the device count with the experts dividing evenly";
        return CK_ERR_SHAPE;
    }
    if (ck_moe_workspace_bytes(&c, 1) == 0) { w = "unsupported MoE configuration"; return CK_ERR_SHAPE; }
    const unsigned long long mb = q4kb(I * H);
    if (!need(k, 0, T * H * 2, w, "x") || !need(k, 1, E * mb, w, "w_gate") || !need(k, 2, E * mb, w, "w_up") ||
        !need(k, 3, E * mb, w, "w_down") || !need(k, 4, NS * mb, w, "s_gate") || !need(k, 5, NS * mb, w, "s_up") ||
        !need(k, 6, NS * mb, w, "s_down") || !need(k, 7, E * H * 4, w, "router") ||
        !need(k, 8, c.mode == 4 ? E * 4 : 0, w, "bias") || !need(k, 9, T * K * 4, w, "ids") ||
        !need(k, 10, T * K * 4, w, "wts") || !need(k, 11, E * 4, w, "counts") || !need(k, 12, T * H * 2, w, "out"))
        return CK_ERR_ARG;
    const unsigned cap = (unsigned)((T + world - 1) / world);
    ck_ep_group *grp = nullptr;
    for (auto &e : g_ep_groups)
        if (e.key.wg == k.b[1] && e.key.wu == k.b[2] && e.key.wd == k.b[3] && e.key.world == world &&
            e.key.ntok_cap >= cap && !memcmp(&e.key.cfg, &c, sizeof(c)))
            grp = e.g;
    if (!grp) {
        int devs[CK_EP_MAX_RANKS];
        for (unsigned d = 0; d < world; ++d) devs[d] = (dev + (int)d) % ndev;
        grp = ck_ep_group_create(&c, world, devs, cap);
        if (!grp) { w = "expert-parallel group could not be built (peer access or memory)"; return CK_ERR_ARG; }
        const int rc = ck_ep_group_load(grp, k.b[1], k.b[2], k.b[3], k.b[4], k.b[5], k.b[6], (const float *)k.b[7],
                                        (const float *)k.b[8]);
        if (rc) {
            ck_ep_group_destroy(grp);
            w = "expert-parallel group could not load the weights";
            return rc;
        }
        g_ep_groups.push_back({{k.b[1], k.b[2], k.b[3], world, cap, c}, grp});
    }
    return ck_ep_group_forward(grp, k.b[0], (uint32_t)T, (int32_t *)k.b[9], (float *)k.b[10], (int32_t *)k.b[11],
                               k.b[12], k.s);
}
// ck_q4k_gemm_bf16: buffers qb x y workspace; constants rows cols ntok
int L_q4k_gemm(const Call &k, std::string &w) {
    const unsigned long long rows = k.c[0], cols = k.c[1], ntok = k.c[2];
    if (cols % 64 || (rows * cols) % 256) { w = "cols % 64 and rows*cols % 256 must be 0"; return CK_ERR_SHAPE; }
    if (!need(k, 0, q4kb(rows * cols), w, "qb") || !need(k, 1, ntok * cols * 2, w, "x") ||
        !need(k, 2, ntok * rows * 2, w, "y") || !need(k, 3, ck_q4k_gemm_workspace_bytes((uint32_t)ntok), w, "workspace"))
        return CK_ERR_ARG;
    return ck_q4k_gemm_bf16(k.b[0], k.b[1], k.b[2], k.c[0], k.c[1], k.c[2], k.b[3], k.blen[3], k.s);
}

const Entry REGISTRY[] = {
    {"form_q8_0_dequant_f32", 2, 2, L_q80_dequant},
    {"form_q8_0_matvec_f32", 3, 2, L_q80_attestant},
    {"form_q8_0_matvec_lane_f32", 3, 2, L_q80_fast},
    {"form_q8_0_matvec_wide_f32", 3, 2, L_q80_fast},
    {"form_q4k_dequant_f32", 2, 2, L_q4k_dequant},
    {"form_q4k_matvec_f32", 3, 2, L_q4k_attestant},
    {"form_q4k_matvec_part_f32", 3, 3, L_q4k_part},
    {"form_q4k_matvec_hoist_f32", 3, 3, L_q4k_part},
    {"form_part_combine_f32", 2, 2, L_part_combine},
    {"form_q4k_matvec_lane_f32", 3, 2, L_q4k_fast},
    {"form_q4k_matvec_slot_f32", 3, 2, L_q4k_fast},
    {"form_q4k_matvec_slot4_f32", 3, 2, L_q4k_fast},
    {"form_q4k_matmul_batch_f32", 3, 3, L_q4k_matmul_batch},
    {"form_q6k_dequant_f32", 2, 2, L_q6k_dequant},
    {"form_q6k_matvec_f32", 3, 2, L_q6k_attestant},
    {"form_q6k_matvec_part_f32", 3, 3, L_q6k_part},
    {"form_q6k_matvec_hoist_f32", 3, 3, L_q6k_part},
    {"form_q6k_matvec_lane_f32", 3, 2, L_q6k_fast},
    {"form_q6k_matvec_slot_f32", 3, 2, L_q6k_fast},
    {"form_q6k_matmul_batch_f32", 3, 3, L_q6k_matmul_batch},
    {"form_f16_matvec_f32", 3, 2, L_f16_matvec},
    {"form_moe_route_f32", 3, 2, L_route},
    {"form_moe_route_wide_f32", 3, 2, L_route_wide},
    {"form_dsv4_router_f32", 4, 3, L_dsv4_router},
    {"form_dsv4_swiglu_f32", 3, 3, L_dsv4_swiglu},
    {"form_swiglu_f32", 3, 1, L_swiglu},
    {"form_scale_f32", 2, 2, L_scale},
    {"form_axpy_f32", 2, 2, L_axpy},
    {"form_dsv4_scale_f32", 2, 2, L_scale},
    {"form_dsv4_axpy_f32", 2, 2, L_axpy},
    {"form_dsv4_matvec_f32", 3, 2, L_f32_matvec},
    {"form_dsv4_swiglu_experts", 4, 3, L_swiglu_experts},
    {"form_dsv4_moe_reduce", 2, 2, L_moe_reduce},
    {"ck_moe_layer_bf16", 14, 11, L_moe_layer},
    {"ck_moe_layer_ep_bf16", 14, 12, L_moe_layer_ep},
    {"ck_q4k_gemm_bf16", 4, 3, L_q4k_gemm},
};
constexpr int NREG = sizeof(REGISTRY) / sizeof(REGISTRY[0]);

long long emit(char *out, long long cap, const std::string &s) {
    long long n = (long long)s.size();
    if (n > cap) n = cap;
    if (n > 0) memcpy(out, s.data(), (size_t)n);
    return n;
}

void open_batch() {
    if (g.batch_open) return;
    g.batch_open = true;
    g.batch_concurrent = g.next_concurrent;
    g.next_concurrent = 0;
    if (!g.batch_start) cudaEventCreate(&g.batch_start);
    cudaEventRecord(g.batch_start, g.stream);
}

int writeback_files() {
    for (auto &b : g.bufs) {
        if (!b.live || !b.file_rw) continue;
        std::vector<char> host(b.len);
        if (cudaMemcpy(host.data(), b.dev, b.len, cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
        FILE *f = fopen(b.path.c_str(), "r+b");
        if (!f) return -1;
        if (fseek(f, b.file_off, SEEK_SET) != 0 || fwrite(host.data(), 1, b.len, f) != b.len) {
            fclose(f);
            return -1;
        }
        fclose(f);
    }
    return 0;
}

}  // namespace

extern "C" {

long long fk_metal_pipeline_external(const char *msl, long long msl_len, const char *name, long long name_len) {
    if (!carrier_up()) return 0;
    if (!name || name_len <= 0 || name_len > 256) {
        err("pipeline: kernel name length out of range");
        return 0;
    }
    const std::string fn(name, (size_t)name_len);
    const std::string key = fn + "\n" + std::string(msl ? msl : "", msl && msl_len > 0 ? (size_t)msl_len : 0);
    auto it = g.pipe_by_key.find(key);
    if (it != g.pipe_by_key.end()) return it->second;
    int idx = -1;
    for (int i = 0; i < NREG; ++i)
        if (fn == REGISTRY[i].name) idx = i;
    if (idx < 0) {
        err("pipeline: no sm_100a kernel is registered under the name " + fn);
        return 0;
    }
    if ((int)g.pipes.size() >= MAX_PIPE) {
        err("pipeline table full at 512");
        return 0;
    }
    g.pipes.push_back(idx);
    const long long h = (long long)g.pipes.size();
    g.pipe_by_key[key] = h;
    return h;
}

long long fk_metal_buf_alloc_external(long long nbytes) {
    if (!carrier_up()) return 0;
    if (nbytes <= 0) {
        err("buf_alloc needs a positive length");
        return 0;
    }
    Buf b;
    if (cudaMalloc(&b.dev, (size_t)nbytes) != cudaSuccess) {
        cudaGetLastError();
        err("buffer allocation failed");
        return 0;
    }
    cudaMemset(b.dev, 0, (size_t)nbytes);
    b.len = (unsigned long long)nbytes;
    long long h = buf_register(b);
    if (!h) cudaFree(b.dev);
    return h;
}

long long fk_metal_buf_from_file_external(const char *path, long long path_len, long long off, long long len) {
    if (!carrier_up()) return 0;
    if (len == (-9223372036854775807LL - 1LL)) {
        err("buf_from_file length is out of range");
        return 0;
    }
    const bool rw = len < 0;
    if (rw) len = -len;
    if (off < 0 || len <= 0) {
        err("buf_from_file needs off>=0 and len>0");
        return 0;
    }
    if (!path || path_len <= 0 || path_len >= 4096) {
        err("buf_from_file path length out of range");
        return 0;
    }
    std::string p(path, (size_t)path_len);
    FILE *f = fopen(p.c_str(), rw ? "r+b" : "rb");
    if (!f && rw) {
        f = fopen(p.c_str(), "w+b");
    }
    if (!f) {
        err("cannot open " + p);
        return 0;
    }
    fseek(f, 0, SEEK_END);
    long long size = ftell(f);
    if (rw && off + len > size) {
        // extend the file, as the writable mapping does
        fseek(f, off + len - 1, SEEK_SET);
        fputc(0, f);
        size = off + len;
    }
    if (off + len > size) {
        char m[256];
        snprintf(m, sizeof(m), "file is %lld bytes, asked for [%lld,%lld)", size, off, off + len);
        err(m);
        fclose(f);
        return 0;
    }
    std::vector<char> host((size_t)len);
    fseek(f, off, SEEK_SET);
    size_t got = fread(host.data(), 1, (size_t)len, f);
    fclose(f);
    if ((long long)got != len) {
        err("short read from " + p);
        return 0;
    }
    Buf b;
    if (cudaMalloc(&b.dev, (size_t)len) != cudaSuccess) {
        cudaGetLastError();
        err("buffer allocation failed");
        return 0;
    }
    if (cudaMemcpy(b.dev, host.data(), (size_t)len, cudaMemcpyHostToDevice) != cudaSuccess) {
        cudaFree(b.dev);
        err("copy of the file region into device memory failed");
        return 0;
    }
    b.len = (unsigned long long)len;
    b.file_rw = rw;
    b.path = p;
    b.file_off = off;
    long long h = buf_register(b);
    if (!h) cudaFree(b.dev);
    return h;
}

long long fk_metal_buf_write_external(long long h, long long off, const char *bytes, long long len) {
    const long long slot = buf_slot(h);
    if (!slot) {
        err("buf_write: bad handle " + std::to_string(h));
        return -1;
    }
    if (off < 0 || len < 0) {
        err("buf_write: negative off or len");
        return -1;
    }
    Buf &b = g.bufs[slot - 1];
    if ((unsigned long long)(off + len) > b.len) {
        err("buf_write: range past the buffer's length");
        return -1;
    }
    // stream-ordered, so a write lands after the dispatches enqueued before it
    if (len > 0 &&
        cudaMemcpyAsync((char *)b.dev + off, bytes, (size_t)len, cudaMemcpyHostToDevice, g.stream) != cudaSuccess) {
        err("buf_write: copy failed");
        return -1;
    }
    if (len > 0) cudaStreamSynchronize(g.stream);
    return len;
}

long long fk_metal_enqueue_external(long long pipe, const char *binding, long long binding_len, long long threads) {
    if (!carrier_up()) return -1;
    if (pipe < 1 || pipe > (long long)g.pipes.size()) {
        err("enqueue: bad pipeline handle " + std::to_string(pipe));
        return -1;
    }
    if (threads <= 0) {
        err("enqueue: threads must be positive");
        return -1;
    }
    const unsigned char *bp = (const unsigned char *)binding;
    if (!bp || binding_len < 4) {
        err("enqueue: binding shorter than its first count");
        return -1;
    }
    const unsigned nbuf = le32(bp);
    if (nbuf > 64 || binding_len < (long long)(4 + 4 * nbuf + 4)) {
        err("enqueue: binding truncated before its constant count");
        return -1;
    }
    const unsigned nconst = le32(bp + 4 + 4 * nbuf);
    if (nconst > 64) {
        err("enqueue: more than 64 constants");
        return -1;
    }
    const long long base = (long long)(4 + 4 * nbuf + 4 + 4 * nconst);
    unsigned tpg = 0, tgmem = 0, mode = 0, barrier = 0;
    if (binding_len == base + 8 || binding_len == base + 16) {
        tpg = le32(bp + base);
        tgmem = le32(bp + base + 4);
        if (binding_len == base + 16) {
            mode = le32(bp + base + 8);
            barrier = le32(bp + base + 12);
        }
    } else if (binding_len != base) {
        char m[320];
        snprintf(m, sizeof(m),
                 "enqueue: binding is %lld bytes; n_buf=%u n_const=%u makes %lld (no tail), %lld "
                 "(threads_per_group + threadgroup_bytes), or %lld (+ dispatch_mode + barrier_before)",
                 binding_len, nbuf, nconst, base, base + 8, base + 16);
        err(m);
        return -1;
    }
    const int concurrent = g.batch_open ? g.batch_concurrent : g.next_concurrent;
    if (mode > 1) {
        err("enqueue: dispatch_mode " + std::to_string(mode) + " is not 0 or 1");
        return -1;
    }
    if (barrier > 1) {
        err("enqueue: barrier_before " + std::to_string(barrier) + " is not 0 or 1");
        return -1;
    }
    if (mode == 1 && tpg == 0) {
        err("enqueue: dispatch_mode 1 (threadgroups) needs threads_per_group nonzero");
        return -1;
    }
    if (barrier == 1 && !concurrent) {
        err("enqueue: barrier_before is only legal in a concurrent batch");
        return -1;
    }
    if (mode == 1 && tpg > 1024) {
        err("enqueue: threads_per_group " + std::to_string(tpg) + " past this pipeline's max 1024");
        return -1;
    }
    (void)tgmem;
    const Entry &e = REGISTRY[g.pipes[(size_t)(pipe - 1)]];
    if (nbuf != e.nbuf || nconst != e.nconst) {
        char m[256];
        snprintf(m, sizeof(m), "enqueue: %s binds %u buffers and %u constants, the binding has %u and %u", e.name,
                 e.nbuf, e.nconst, nbuf, nconst);
        err(m);
        return -1;
    }
    Call k = {};
    for (unsigned i = 0; i < nbuf; ++i) {
        const long long bh = (long long)le32(bp + 4 + 4 * i);
        const long long bs = buf_slot(bh);
        if (!bs) {
            err("enqueue: bad buffer handle " + std::to_string(bh) + " at slot " + std::to_string(i));
            return -1;
        }
        k.b[i] = g.bufs[bs - 1].dev;
        k.blen[i] = g.bufs[bs - 1].len;
    }
    for (unsigned i = 0; i < nconst; ++i) k.c[i] = le32(bp + 4 + 4 * nbuf + 4 + 4 * i);
    k.threads = threads;
    k.s = g.stream;
    const bool opened_here = !g.batch_open;
    const int armed = g.next_concurrent;
    open_batch();
    std::string why;
    const int rc = e.fn(k, why);
    if (rc != 0) {
        // a refused dispatch leaves no half-open batch behind it (the batch's mode stays armed)
        if (opened_here && g.pending == 0) {
            g.batch_open = false;
            g.batch_concurrent = 0;
            g.next_concurrent = armed;
        }
        err(std::string("enqueue: ") + e.name + ": " + (why.empty() ? (rc > 0 ? cudaGetErrorString((cudaError_t)rc) : ck_last_error()) : why));
        return -1;
    }
    g.pending++;
    g.total_dispatch++;
    return 1;
}

long long fk_metal_sync_external(void) {
    if (!g.up) return 0;
    long long n = 0;
    bool had = false;
    for (auto &kv : g.inflight) {
        cudaEventSynchronize(kv.second.end);
        float ms = 0.0f;
        if (cudaEventElapsedTime(&ms, kv.second.start, kv.second.end) == cudaSuccess) g.gpu_busy_us += ms * 1000.0;
        cudaEventDestroy(kv.second.start);
        cudaEventDestroy(kv.second.end);
        n += kv.second.n;
        had = true;
    }
    g.inflight.clear();
    if (g.batch_open) {
        cudaEvent_t end;
        cudaEventCreate(&end);
        cudaEventRecord(end, g.stream);
        cudaError_t r = cudaEventSynchronize(end);
        float ms = 0.0f;
        if (cudaEventElapsedTime(&ms, g.batch_start, end) == cudaSuccess) g.gpu_busy_us += ms * 1000.0;
        cudaEventDestroy(end);
        n += g.pending;
        g.pending = 0;
        g.batch_open = false;
        g.batch_concurrent = 0;
        had = true;
        if (r != cudaSuccess) {
            err(std::string("dispatch: ") + cudaGetErrorString(r));
            return -1;
        }
    }
    if (had) {
        g.total_sync++;
        if (writeback_files() != 0) {
            err("sync: writing a writable file region back failed");
            return -1;
        }
    }
    const cudaError_t r = cudaGetLastError();
    if (r != cudaSuccess) {
        err(std::string("dispatch: ") + cudaGetErrorString(r));
        return -1;
    }
    return n;
}

long long fk_metal_buf_read_external(long long h, long long off, long long len, char *out, long long cap) {
    if (g.batch_open || !g.inflight.empty())
        if (fk_metal_sync_external() < 0) return -1;
    const long long slot = buf_slot(h);
    if (!slot) {
        err("buf_read: bad handle " + std::to_string(h));
        return -1;
    }
    if (off < 0 || len < 0 || len > cap) {
        err("buf_read: off/len out of range");
        return -1;
    }
    Buf &b = g.bufs[slot - 1];
    if ((unsigned long long)(off + len) > b.len) {
        err("buf_read: range past the buffer's length");
        return -1;
    }
    if (len > 0 && cudaMemcpy(out, (const char *)b.dev + off, (size_t)len, cudaMemcpyDeviceToHost) != cudaSuccess) {
        err("buf_read: copy failed");
        return -1;
    }
    return len;
}

long long fk_metal_status_external(char *out, long long cap) {
    if (!carrier_up()) {
        return emit(out, cap, "metal_owner=fkwu-form-cli\nmetal_linked=false\nmetal_door=handle\ncarrier=cuda\nlast_error=" +
                                  g.last_err + "\n");
    }
    long long live = 0;
    for (auto &b : g.bufs) live += b.live ? 1 : 0;
    char s[2048];
    snprintf(s, sizeof(s),
             "metal_owner=fkwu-form-cli\nmetal_linked=true\nmetal_door=handle\ncarrier=cuda-sm100a\ndevice=%s\n"
             "unified_memory=0\nbuffers=%lld\npipelines=%zu\nbuffer_slots=%zu\nfree_slots=%zu\npending=%lld\n"
             "batch=%s\nin_flight=%zu\ntotal_dispatch=%lld\ntotal_sync=%lld\ngpu_busy_us_total=%lld\nlast_error=%s\n",
             g.devname, live, g.pipes.size(), g.bufs.size(), g.free_slots.size(), g.pending,
             !g.batch_open ? "none" : (g.batch_concurrent ? "concurrent" : "serial"), g.inflight.size(),
             g.total_dispatch, g.total_sync, (long long)g.gpu_busy_us, g.last_err.c_str());
    return emit(out, cap, s);
}

long long fk_metal_batch_concurrent_external(void) {
    if (!carrier_up()) return 0;
    if (g.batch_open) {
        err("batch_concurrent: a batch is already open; sync or submit it first");
        return 0;
    }
    g.next_concurrent = 1;
    return 1;
}

long long fk_metal_buf_free_external(long long h) {
    const long long slot = buf_slot(h);
    if (!slot) {
        err("buf_free: bad handle " + std::to_string(h));
        return -1;
    }
    if (g.batch_open || !g.inflight.empty()) {
        err("buf_free: work is open or in flight; sync first");
        return -1;
    }
    Buf &b = g.bufs[slot - 1];
    cudaFree(b.dev);
    b = Buf();
    g.gen[slot - 1] = (g.gen[slot - 1] + 1) & 0xFFFF;
    g.free_slots.push_back(slot);
    return 1;
}

long long fk_metal_submit_external(void) {
    if (!g.batch_open) {
        err("submit: no open batch");
        return 0;
    }
    if (g.pending == 0) {
        g.batch_open = false;
        g.batch_concurrent = 0;
        err("submit: batch had no dispatches");
        return 0;
    }
    State::Fence f;
    cudaEventCreate(&f.start);
    cudaEventCreate(&f.end);
    // the batch's start event is reused for the next batch, so copy its position by recording the
    // fence start right after it: both mark the same point in the stream
    cudaEventRecord(f.end, g.stream);
    float ms = 0.0f;
    (void)ms;
    std::swap(f.start, g.batch_start);
    f.n = g.pending;
    const long long id = g.fence_next++;
    g.inflight[id] = f;
    g.pending = 0;
    g.batch_open = false;
    g.batch_concurrent = 0;
    return id;
}

long long fk_metal_fence_wait_external(long long fence) {
    auto it = g.inflight.find(fence);
    if (it == g.inflight.end()) {
        err("fence_wait: no in-flight fence " + std::to_string(fence));
        return 0;
    }
    State::Fence f = it->second;
    g.inflight.erase(it);
    const cudaError_t r = cudaEventSynchronize(f.end);
    float ms = 0.0f;
    if (cudaEventElapsedTime(&ms, f.start, f.end) == cudaSuccess) g.gpu_busy_us += ms * 1000.0;
    cudaEventDestroy(f.start);
    cudaEventDestroy(f.end);
    if (r != cudaSuccess) {
        err(std::string("dispatch: ") + cudaGetErrorString(r));
        return -1;
    }
    g.total_sync++;
    return f.n;
}

// The one-shot text doors (fkwu-uni.c:910-929 weak stubs; fk-metal-carrier.m:192-335).
long long fk_metal_matvec_fixture_external(char *out, long long cap) {
    if (!carrier_up())
        return emit(out, cap, "SKIP fkwu-form-cli-metal-direct: " + g.last_err +
                                  "\nmetal_owner=fkwu-form-cli\nmetal_linked=false\n");
    return emit(out, cap, std::string("PASS fkwu-form-cli-metal-direct\nmetal_owner=fkwu-form-cli\nmetal_linked=true\n"
                                      "device=") + g.devname + "\nunified_memory=0\nmax_threadgroup=1024\n");
}

long long fk_metal_matvec_f32_external(const char *msl, long long msl_len, const char *kernel, long long kernel_len,
                                       const char *model, long long model_len, char *out, long long cap) {
    (void)msl;
    (void)msl_len;
    if (!carrier_up())
        return emit(out, cap, "SKIP fkwu-form-cli-metal-matvec-f32: " + g.last_err +
                                  "\nmetal_owner=fkwu-form-cli\nmetal_linked=false\n");
    if (model_len < 8) return emit(out, cap, "FAIL fkwu-form-cli-metal-matvec-f32 model shorter than its 8-byte header\n");
    uint32_t rows = 0, cols = 0;
    memcpy(&rows, model, 4);
    memcpy(&cols, model + 4, 4);
    if (rows == 0 || cols == 0) return emit(out, cap, "FAIL fkwu-form-cli-metal-matvec-f32 rows or cols is zero\n");
    const long long need_b = 8 + (long long)rows * cols * 4 + (long long)cols * 4;
    if (model_len < need_b) {
        char m[256];
        snprintf(m, sizeof(m), "FAIL fkwu-form-cli-metal-matvec-f32 model is %lld bytes, rows=%u cols=%u needs %lld\n",
                 model_len, rows, cols, need_b);
        return emit(out, cap, m);
    }
    float *W = nullptr, *x = nullptr, *y = nullptr;
    cudaMalloc(&W, (size_t)rows * cols * 4);
    cudaMalloc(&x, (size_t)cols * 4);
    cudaMalloc(&y, (size_t)rows * 4);
    cudaMemcpy(W, model + 8, (size_t)rows * cols * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(x, model + 8 + (long long)rows * cols * 4, (size_t)cols * 4, cudaMemcpyHostToDevice);
    ck::launch_f32_matvec(W, x, y, rows, cols, g.stream);
    std::vector<float> hy(rows);
    cudaMemcpyAsync(hy.data(), y, (size_t)rows * 4, cudaMemcpyDeviceToHost, g.stream);
    const cudaError_t r = cudaStreamSynchronize(g.stream);
    cudaFree(W);
    cudaFree(x);
    cudaFree(y);
    if (r != cudaSuccess) return emit(out, cap, std::string("FAIL fkwu-form-cli-metal-matvec-f32 ") + cudaGetErrorString(r) + "\n");
    double sum = 0.0;
    for (uint32_t i = 0; i < rows; ++i) sum += hy[i];
    std::string s = "PASS fkwu-form-cli-metal-matvec-f32\nmetal_owner=fkwu-form-cli\nmetal_linked=true\n";
    s += std::string("device=") + g.devname + "\nkernel=" + std::string(kernel, (size_t)(kernel_len > 0 ? kernel_len : 0)) + "\n";
    char m[128];
    snprintf(m, sizeof(m), "rows=%u\ncols=%u\nsum=%.9g\ny=", rows, cols, sum);
    s += m;
    for (uint32_t i = 0; i < rows; ++i) {
        if ((long long)s.size() > cap - 64) {
            s += " ...";
            break;
        }
        snprintf(m, sizeof(m), "%s%.9g", i ? " " : "", (double)hy[i]);
        s += m;
    }
    s += "\n";
    return emit(out, cap, s);
}

}  // extern "C"
