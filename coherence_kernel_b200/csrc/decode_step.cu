// decode_step.cu -- one decode step of a transformer block with an MoE feed-forward, resident on
// the device and replayable as one CUDA graph.
//
// The reference measured its decode token at 51.9 ms of which 44.6 ms were the joins between
// operations -- 396 host dispatches per forward at about 113 us each -- not the arithmetic
// (receipts/2026-07-22-ship-the-slot-map.md:135-145).  Here the whole step is issued once into a
// stream and, once captured, replays as a single graph launch:
//
//   a  = rmsnorm(h, g_attn)                    ln-rmsnorm, llama-numerics.fk:40-50
//   q  = Wq a,  k = Wk a,  v = Wv a            Q4_K matvecs (the decode matvec of this library)
//   h += Wo v                                  attention at one position: softmax of one score is 1,
//                                              so its output is v exactly
//   b  = bf16(rmsnorm(h, g_ffn))
//   h += moe(b)                                ck_moe_layer_bf16 (route, permute, experts, combine)
//
// h is fp32 [ntok, hidden] and is updated in place; q, k, v are fp32 [ntok, hidden] outputs (the
// rows a KV cache stores).  Every buffer the step needs beyond its inputs and outputs is carved
// from one caller workspace.
#include "../../include/ck_b200.h"
#include "ck_common.cuh"
#include "ck_launch.h"

#include <stdlib.h>
#include <string.h>

namespace {

constexpr int NORM_THREADS = 512;

// One CTA per token: the sum of squares in fp32 (per-thread strided partials, then the warps in a
// fixed order), s = 1 / sqrt(mean + eps) correctly rounded, out = (x * s) * g.
__global__ void __launch_bounds__(NORM_THREADS) k_rmsnorm(const float *__restrict__ x, const float *__restrict__ g,
                                                          float *__restrict__ out_f32, uint16_t *__restrict__ out_bf16,
                                                          uint32_t H, float eps) {
    __shared__ float part[NORM_THREADS / 32];
    __shared__ float scale;
    const float *xr = x + (size_t)blockIdx.x * H;
    float acc = 0.0f;
    for (uint32_t i = threadIdx.x; i < H; i += NORM_THREADS) acc = fmaf(xr[i], xr[i], acc);
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        float s = 0.0f;
        for (int w = 0; w < NORM_THREADS / 32; ++w) s += part[w];
        scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s, (float)H), eps)));
    }
    __syncthreads();
    const float s = scale;
    for (uint32_t i = threadIdx.x; i < H; i += NORM_THREADS) {
        const float v = __fmul_rn(__fmul_rn(xr[i], s), g[i]);
        if (out_f32) out_f32[(size_t)blockIdx.x * H + i] = v;
        if (out_bf16) out_bf16[(size_t)blockIdx.x * H + i] = __bfloat16_as_ushort(__float2bfloat16_rn(v));
    }
}

__global__ void k_add_f32(float *__restrict__ h, const float *__restrict__ y, size_t n) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) h[i] = __fadd_rn(h[i], y[i]);
}
__global__ void k_add_bf16(float *__restrict__ h, const uint16_t *__restrict__ m, size_t n) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) h[i] = __fadd_rn(h[i], __uint_as_float((uint32_t)m[i] << 16));
}

inline size_t al(size_t b) { return (b + 255) & ~(size_t)255; }

struct Carve {
    float *a, *o;
    uint16_t *b, *m;
    int32_t *ids, *counts;
    float *wts;
    void *moe_ws;
    size_t moe_ws_bytes, total;
};
Carve carve(const ck_decode_config *c, uint8_t *base) {
    Carve w;
    const size_t T = c->max_tokens, H = c->hidden;
    size_t o = 0;
    auto take = [&](size_t bytes) { uint8_t *p = base ? base + o : nullptr; o += al(bytes); return p; };
    w.a = (float *)take(T * H * 4);
    w.o = (float *)take(T * H * 4);
    w.b = (uint16_t *)take(T * H * 2);
    w.m = (uint16_t *)take(T * H * 2);
    w.ids = (int32_t *)take(T * c->moe.nsel * 4);
    w.wts = (float *)take(T * c->moe.nsel * 4);
    w.counts = (int32_t *)take((size_t)c->moe.n_experts * 4);
    w.moe_ws_bytes = ck_moe_workspace_bytes(&c->moe, c->max_tokens);
    w.moe_ws = take(w.moe_ws_bytes);
    w.total = o;
    return w;
}

}  // namespace

struct ck_decode_step {
    ck_decode_config cfg;
    const void *wq, *wk, *wv, *wo;
    const float *g_attn, *g_ffn;
    const void *wg, *wu, *wd, *sg, *su, *sd;
    const float *router, *bias;
    Carve w;
    cudaGraphExec_t exec;
};

extern "C" {

size_t ck_decode_step_workspace_bytes(const ck_decode_config *c) {
    if (!c || c->moe.hidden != c->hidden || c->max_tokens == 0 || ck_moe_workspace_bytes(&c->moe, c->max_tokens) == 0)
        return 0;
    return carve(c, nullptr).total;
}

ck_decode_step *ck_decode_step_create(const ck_decode_config *c, const void *wq_dev, const void *wk_dev,
                                      const void *wv_dev, const void *wo_dev, const float *g_attn_dev,
                                      const float *g_ffn_dev, const void *w_gate_dev, const void *w_up_dev,
                                      const void *w_down_dev, const void *s_gate_dev, const void *s_up_dev,
                                      const void *s_down_dev, const float *router_w_dev, const float *bias_dev,
                                      void *workspace_dev, size_t workspace_bytes) {
    const size_t need = ck_decode_step_workspace_bytes(c);
    if (need == 0 || workspace_bytes < need || !workspace_dev || c->hidden % 256) return nullptr;
    if (!wq_dev || !wk_dev || !wv_dev || !wo_dev || !g_attn_dev || !g_ffn_dev || !w_gate_dev || !w_up_dev ||
        !w_down_dev || !router_w_dev || (c->moe.mode == 4 && !bias_dev) ||
        (c->moe.n_shared && (!s_gate_dev || !s_up_dev || !s_down_dev)))
        return nullptr;
    ck_decode_step *s = (ck_decode_step *)calloc(1, sizeof(ck_decode_step));
    if (!s) return nullptr;
    s->cfg = *c;
    s->wq = wq_dev;
    s->wk = wk_dev;
    s->wv = wv_dev;
    s->wo = wo_dev;
    s->g_attn = g_attn_dev;
    s->g_ffn = g_ffn_dev;
    s->wg = w_gate_dev;
    s->wu = w_up_dev;
    s->wd = w_down_dev;
    s->sg = s_gate_dev;
    s->su = s_up_dev;
    s->sd = s_down_dev;
    s->router = router_w_dev;
    s->bias = bias_dev;
    s->w = carve(c, (uint8_t *)workspace_dev);
    return s;
}

int ck_decode_step_run(ck_decode_step *s, float *h_dev, float *q_dev, float *k_dev, float *v_dev, uint32_t ntok,
                       void *stream) {
    if (!s || !h_dev || !q_dev || !k_dev || !v_dev) return CK_EARG;
    if (ntok == 0) return 0;
    if (ntok > s->cfg.max_tokens) return CK_ESHAPE;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const uint32_t H = s->cfg.hidden;
    const size_t n = (size_t)ntok * H;
    const unsigned eb = (unsigned)((n + 255) / 256);
    k_rmsnorm<<<ntok, NORM_THREADS, 0, st>>>(h_dev, s->g_attn, s->w.a, nullptr, H, s->cfg.eps);
    int rc = (int)cudaGetLastError();
    // Q, K and V read the same a: one launch for the three where the tensor-core matvec applies
    const uint8_t *wqkv[3] = {(const uint8_t *)s->wq, (const uint8_t *)s->wk, (const uint8_t *)s->wv};
    float *yqkv[3] = {q_dev, k_dev, v_dev};
    if (!rc) rc = ck::launch_q4k_matvec_group(3, wqkv, s->w.a, yqkv, H, H, ntok, st);
    if (!rc) rc = ck::launch_q4k_matvec((const uint8_t *)s->wo, v_dev, s->w.o, H, H, ntok, st);
    if (rc) return rc;
    k_add_f32<<<eb, 256, 0, st>>>(h_dev, s->w.o, n);
    k_rmsnorm<<<ntok, NORM_THREADS, 0, st>>>(h_dev, s->g_ffn, nullptr, s->w.b, H, s->cfg.eps);
    rc = (int)cudaGetLastError();
    if (rc) return rc;
    rc = ck_moe_layer_bf16(&s->cfg.moe, s->w.b, ntok, s->wg, s->wu, s->wd, s->sg, s->su, s->sd, s->router, s->bias,
                           s->w.ids, s->w.wts, s->w.counts, s->w.m, s->w.moe_ws, s->w.moe_ws_bytes, stream);
    if (rc) return rc;
    k_add_bf16<<<eb, 256, 0, st>>>(h_dev, s->w.m, n);
    return (int)cudaGetLastError();
}

int ck_decode_step_capture(ck_decode_step *s, float *h_dev, float *q_dev, float *k_dev, float *v_dev, uint32_t ntok,
                           void *stream) {
    if (!s || !stream) return CK_EARG;  // the legacy default stream cannot be captured
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (s->exec) {
        cudaGraphExecDestroy(s->exec);
        s->exec = nullptr;
    }
    cudaError_t e = cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal);
    if (e != cudaSuccess) return (int)e;
    const int rc = ck_decode_step_run(s, h_dev, q_dev, k_dev, v_dev, ntok, stream);
    cudaGraph_t g = nullptr;
    e = cudaStreamEndCapture(st, &g);
    if (rc) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    if (e != cudaSuccess) return (int)e;
    e = cudaGraphInstantiate(&s->exec, g, 0);
    cudaGraphDestroy(g);
    return (int)e;
}

int ck_decode_step_replay(ck_decode_step *s, void *stream) {
    if (!s || !s->exec) return CK_EARG;
    return (int)cudaGraphLaunch(s->exec, reinterpret_cast<cudaStream_t>(stream));
}

int ck_decode_step_status(ck_decode_step *s, uint32_t ntok, void *stream) {
    if (!s) return CK_EARG;
    return ck_moe_layer_status(&s->cfg.moe, ntok, s->w.moe_ws, stream);
}

void ck_decode_step_destroy(ck_decode_step *s) {
    if (!s) return;
    if (s->exec) cudaGraphExecDestroy(s->exec);
    free(s);
}

}  // extern "C"
