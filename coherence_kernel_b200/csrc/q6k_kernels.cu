// q6k_kernels.cu -- GGUF Q6_K (210 bytes / 256 weights) dequant and matvecs.
//
// Layout and unpack follow the reference's flat-index transcription q6m-flat-at
// (form/form-stdlib/q6k-msl.fk:62-81, over q6k-dequant.fk:29-61): block = idx / 256 at a 210-byte
// stride; ql[128] @ +0, qh[64] @ +128, scales[16] (signed int8) @ +192, d (f16) @ +208;
// i = idx % 256, h = i / 128, wi = i % 128, l = wi % 32, g = wi / 32, is = l / 16;
// code = (low nibble of ql[64h + l + 32 (g % 2)] for g < 2, else the high one) + 16 * ((qh[32h + l] >> 2g) & 3);
// w = (d * sc) * (code - 32), sc = scales[8h + is + 2g].  d * sc needs at most 19 significant bits
// and (d * sc) * q at most 25, so the fp32 weight is the fp64 weight rounded once: bit-exact.
//
// Kernels:
//   k_q6k_dequant         w[i] = weight(off + i)                      (form_q6k_dequant_f32)
//   k_q6k_ordered         one thread per row, j counting down, acc = w*x + acc, no FMA
//                                                                      (form_q6k_matvec_f32, q6k-msl.fk:118-123)
//   k_q6k_part            the same fold over `parts` column chunks    (form_q6k_matvec_part/hoist_f32,
//                                                                      qk-matvec-split.fk:114-121,
//                                                                      qk-matvec-lane.fk:213-222)
//   k_q6k_stream          the decode matvec: stages of whole rows copied into shared memory with 16-byte
//                         cp.async, every thread owning fixed 16-weight column units whose activations
//                         stay in registers for every row it folds (form_q6k_matvec_lane/slot_f32)
//   k_q6k_lane            any shape (flat rows that straddle superblocks): one warp per row
#include "ck_common.cuh"
#include "ck_launch.h"

namespace ck {

constexpr uint32_t Q6K_BYTES = 210;

CK_DEV float q6k_weight(const uint8_t *__restrict__ qb, uint64_t idx) {
    const uint8_t *b = qb + (idx >> 8) * Q6K_BYTES;
    const int i = (int)(idx & 255);
    const int h = i >> 7, wi = i & 127, l = wi & 31, g = wi >> 5, is = l >> 4;
    const int qlb = b[64 * h + l + 32 * (g & 1)];
    const int nib = (g >> 1) ? (qlb >> 4) : (qlb & 15);
    const int hi = (b[128 + 32 * h + l] >> (2 * g)) & 3;
    const int q = nib + 16 * hi - 32;
    const int sc = (int)(int8_t)b[192 + 8 * h + is + 2 * g];
    const float d = f16_bits_to_float((uint32_t)b[208] | ((uint32_t)b[209] << 8));
    return __fmul_rn(d * (float)sc, (float)q);
}

__global__ void k_q6k_dequant(const uint8_t *__restrict__ qb, float *__restrict__ w, uint64_t off, uint64_t n) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) w[i] = q6k_weight(qb, off + i);
}

__global__ void k_q6k_ordered(const uint8_t *__restrict__ qb, const float *__restrict__ x, float *__restrict__ y,
                              uint32_t rows, uint32_t cols) {
    const uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    float acc = 0.0f;
    for (uint32_t j = cols; j > 0;) {
        --j;
        acc = __fadd_rn(__fmul_rn(q6k_weight(qb, (uint64_t)r * cols + j), x[j]), acc);
    }
    y[r] = acc;
}

__global__ void k_q6k_part(const uint8_t *__restrict__ qb, const float *__restrict__ x, float *__restrict__ part,
                           uint32_t rows, uint32_t cols, uint32_t parts) {
    const uint64_t gid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= (uint64_t)rows * parts) return;
    const uint32_t r = (uint32_t)(gid / parts), p = (uint32_t)(gid - (uint64_t)r * parts);
    const uint32_t chunk = (cols + parts - 1) / parts;
    uint32_t lo = p * chunk, hi = lo + chunk;
    if (lo > cols) lo = cols;
    if (hi > cols) hi = cols;
    float acc = 0.0f;
    for (uint32_t j = hi; j > lo;) {
        --j;
        acc = __fadd_rn(__fmul_rn(q6k_weight(qb, (uint64_t)r * cols + j), x[j]), acc);
    }
    part[gid] = acc;
}

// One warp per row for any flat shape: lanes stride the columns, then a butterfly sum.
__global__ void k_q6k_lane(const uint8_t *__restrict__ qb, const float *__restrict__ x, float *__restrict__ y,
                           uint32_t rows, uint32_t cols) {
    const uint32_t r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (r >= rows) return;
    float acc = 0.0f;
    for (uint32_t j = lane; j < cols; j += 32) acc = fmaf(q6k_weight(qb, (uint64_t)r * cols + j), x[j], acc);
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) y[r] = acc;
}

namespace q6 {

constexpr int NTHR = 256;
constexpr int MAX_UPT = 4;  // column units (16 weights) per thread: cols <= 16384
constexpr int MAX_RPT = 8;  // rows a thread folds per stage
constexpr uint32_t SMEM_MAX = 110 * 1024;  // two CTAs per SM

struct Geo {
    uint32_t rows, cols, nsb, rb;  // rb: bytes per row
    uint32_t U, tpr, slots, upt;   // units per row, threads per row slot, row slots, units per thread
    uint32_t rs, rpt;              // rows per stage, rows a thread folds per stage (rs / slots)
    uint32_t stage_alloc;          // bytes of one stage buffer (16 bytes of slack past the rows)
    uint32_t red_off;              // cross-warp partials
};

CK_DEV void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
CK_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
CK_DEV void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// four bytes at any byte address of shared memory (the buffers carry 16 bytes of slack)
CK_DEV uint32_t lds32(const uint8_t *p) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t *w = reinterpret_cast<const uint32_t *>(a & ~(uintptr_t)3);
    return __funnelshift_r(w[0], w[1], (uint32_t)(a & 3) * 8);
}

// Byte B of w (< 128) over the float 2.0: 2 + byte / 64, exactly.
template <int B>
CK_DEV float two_plus(uint32_t w) { return __uint_as_float(__byte_perm(w, 0x40000000u, 0x7054u + (B << 8))); }

// The 16 activations of a unit (l0..l0+3 of each of the four 32-wide groups of a half superblock)
// and -160 times the sum of each group's four.
struct XUnit {
    float2 x[8];
    float c[4];
};

// The stage of row group `grp` into buffer `buf`: 16-byte copies of the aligned part (the
// stage's first byte is 16-byte aligned: rs * rb % 16 == 0), plain loads of a ragged tail.
CK_DEV void load_stage(const Geo &g, const uint8_t *__restrict__ qb, uint8_t *buf, uint32_t grp) {
    const uint32_t r0 = grp * g.rs, nr = min(g.rs, g.rows - r0);
    const uint8_t *src = qb + (uint64_t)r0 * g.rb;
    const uint32_t bytes = nr * g.rb, nv = bytes >> 4, tail = bytes & 15;
    for (uint32_t i = threadIdx.x; i < nv; i += NTHR) cp_async16(buf + 16 * i, src + 16 * i);
    if (threadIdx.x < tail) buf[16 * nv + threadIdx.x] = src[16 * nv + threadIdx.x];
    cp_async_commit();
}

// UPT: the units each thread owns (1 up to 4096 columns, 2 up to 8192, 4 up to 16384)
template <int UPT>
__global__ void __launch_bounds__(NTHR, UPT <= 2 ? 2 : 1)
    k_q6k_stream(const uint8_t *__restrict__ qb, const float *__restrict__ x, float *__restrict__ y, Geo g) {
    extern __shared__ __align__(128) uint8_t smem[];
    float *red = reinterpret_cast<float *>(smem + g.red_off);
    const uint32_t t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const uint32_t slot = t / g.tpr, lt = t % g.tpr;
    const uint32_t ngrp = (g.rows + g.rs - 1) / g.rs;

    // this thread's units: u = lt + tpr * k; unit u = (superblock u / 16, sub = u % 16), sub = 8 ip + il
    XUnit xu[UPT];
    uint32_t uoff[UPT], hoff[UPT], soff[UPT], doff[UPT];
#pragma unroll
    for (int k = 0; k < UPT; ++k) {
        const uint32_t u = lt + g.tpr * k;
        const bool live = k < (int)g.upt && u < g.U;
        const uint32_t sb = live ? u >> 4 : 0, sub = u & 15, ip = sub >> 3, il = sub & 7;
        uoff[k] = sb * Q6K_BYTES + 64 * ip + 4 * il;   // ql bytes of groups 0 / 2 (and +32: 1 / 3)
        hoff[k] = sb * Q6K_BYTES + 128 + 32 * ip + 4 * il;  // qh bytes
        soff[k] = sb * Q6K_BYTES + 192 + 8 * ip + (il >> 2);  // the unit's four scales: +0, +2, +4, +6
        doff[k] = sb * Q6K_BYTES + 208;                       // d (f16)
        const float *xs = x + sb * 256 + 128 * ip + 4 * il;
#pragma unroll
        for (int gq = 0; gq < 4; ++gq) {
            const float4 v = live ? __ldg(reinterpret_cast<const float4 *>(xs + 32 * gq)) : make_float4(0, 0, 0, 0);
            xu[k].x[2 * gq] = make_float2(v.x, v.y);
            xu[k].x[2 * gq + 1] = make_float2(v.z, v.w);
            xu[k].c[gq] = -160.0f * ((v.x + v.y) + (v.z + v.w));
        }
    }

    uint8_t *bufs[2] = {smem, smem + g.stage_alloc};
    if (blockIdx.x < ngrp) load_stage(g, qb, bufs[0], blockIdx.x);
    if (blockIdx.x + gridDim.x < ngrp) load_stage(g, qb, bufs[1], blockIdx.x + gridDim.x);
    uint32_t k = 0;
    for (uint32_t grp = blockIdx.x; grp < ngrp; grp += gridDim.x, ++k) {
        const uint8_t *buf = bufs[k & 1];
        const uint32_t r0 = grp * g.rs, nr = min(g.rs, g.rows - r0);
        if (grp + gridDim.x < ngrp) cp_async_wait<1>();
        else cp_async_wait<0>();
        __syncthreads();
        float acc[MAX_RPT];
#pragma unroll
        for (int j = 0; j < MAX_RPT; ++j) acc[j] = 0.0f;
#pragma unroll
        for (int ku = 0; ku < UPT; ++ku) {
            if (ku >= (int)g.upt || lt + g.tpr * ku >= g.U) break;
#pragma unroll
            for (int j = 0; j < MAX_RPT; ++j) {
                const uint32_t i = slot + g.slots * j;
                if (j >= (int)g.rpt) break;
                if (i >= nr) break;
                const uint8_t *row = buf + i * g.rb;
                const uint32_t A = lds32(row + uoff[ku]), B = lds32(row + uoff[ku] + 32), H = lds32(row + hoff[ku]);
                // d * sc of the unit's four sub-blocks (exact in fp32): scales at +0, +2, +4, +6 of
                // soff, d the f16 at byte 208 of the superblock (the stage carries 16 bytes of slack)
                const uint32_t S0 = lds32(row + soff[ku]), S1 = lds32(row + soff[ku] + 4);
                const float d = f16_bits_to_float(lds32(row + doff[ku]) & 0xFFFFu);
                const float4 ds = make_float4(d * (float)(int)(int8_t)(S0 & 0xFFu), d * (float)(int)(int8_t)(S0 >> 16),
                                              d * (float)(int)(int8_t)(S1 & 0xFFu), d * (float)(int)(int8_t)(S1 >> 16));
                const uint32_t q0 = (A & 0x0F0F0F0Fu) | ((H << 4) & 0x30303030u);
                const uint32_t q1 = (B & 0x0F0F0F0Fu) | ((H << 2) & 0x30303030u);
                const uint32_t q2 = ((A >> 4) & 0x0F0F0F0Fu) | (H & 0x30303030u);
                const uint32_t q3 = ((B >> 4) & 0x0F0F0F0Fu) | ((H >> 2) & 0x30303030u);
                const XUnit &xv = xu[ku];
                float2 s0 = __fmul2_rn(make_float2(two_plus<0>(q0), two_plus<1>(q0)), xv.x[0]);
                float2 s1 = __fmul2_rn(make_float2(two_plus<0>(q1), two_plus<1>(q1)), xv.x[2]);
                float2 s2 = __fmul2_rn(make_float2(two_plus<0>(q2), two_plus<1>(q2)), xv.x[4]);
                float2 s3 = __fmul2_rn(make_float2(two_plus<0>(q3), two_plus<1>(q3)), xv.x[6]);
                s0 = __ffma2_rn(make_float2(two_plus<2>(q0), two_plus<3>(q0)), xv.x[1], s0);
                s1 = __ffma2_rn(make_float2(two_plus<2>(q1), two_plus<3>(q1)), xv.x[3], s1);
                s2 = __ffma2_rn(make_float2(two_plus<2>(q2), two_plus<3>(q2)), xv.x[5], s2);
                s3 = __ffma2_rn(make_float2(two_plus<2>(q3), two_plus<3>(q3)), xv.x[7], s3);
                // sum x (code - 32) = 64 sum x v - 160 sum x, with v = 2 + code / 64
                float a = acc[j];
                a = fmaf(ds.x, fmaf(64.0f, s0.x + s0.y, xv.c[0]), a);
                a = fmaf(ds.y, fmaf(64.0f, s1.x + s1.y, xv.c[1]), a);
                a = fmaf(ds.z, fmaf(64.0f, s2.x + s2.y, xv.c[2]), a);
                a = fmaf(ds.w, fmaf(64.0f, s3.x + s3.y, xv.c[3]), a);
                acc[j] = a;
            }
        }
        __syncthreads();  // every read of this buffer is done
        if (grp + 2 * gridDim.x < ngrp) load_stage(g, qb, bufs[k & 1], grp + 2 * gridDim.x);
        // row sums: over the lanes of a warp that share a slot, then over the slot's warps in order
        const uint32_t wl = g.tpr < 32 ? g.tpr : 32;
#pragma unroll
        for (int j = 0; j < MAX_RPT; ++j) {
            if (j >= (int)g.rpt) break;
            float v = acc[j];
            for (uint32_t o = wl >> 1; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if ((lane & (wl - 1)) == 0) red[(slot + g.slots * j) * 32 + (lt / 32)] = v;
        }
        __syncthreads();
        if (t < nr) {
            const uint32_t nw = g.tpr >= 32 ? g.tpr / 32 : 1;
            float s = 0.0f;
            for (uint32_t w = 0; w < nw; ++w) s += red[t * 32 + w];
            y[r0 + t] = s;
        }
    }
    (void)warp;
}

uint32_t pow2_ceil(uint32_t v) {
    uint32_t p = 1;
    while (p < v) p <<= 1;
    return p;
}
uint32_t gcd(uint32_t a, uint32_t b) {
    while (b) {
        const uint32_t t = a % b;
        a = b;
        b = t;
    }
    return a;
}

// The stream kernel's geometry, or false where it does not apply (the lane kernel runs then).
bool plan(uint32_t rows, uint32_t cols, Geo &g) {
    if (cols % 256 || cols == 0 || cols > 256u * 16u * MAX_UPT) return false;
    g = {};
    g.rows = rows;
    g.cols = cols;
    g.nsb = cols / 256;
    g.rb = g.nsb * Q6K_BYTES;
    g.U = 16 * g.nsb;
    g.tpr = g.U >= (uint32_t)NTHR ? NTHR : pow2_ceil(g.U);
    g.slots = NTHR / g.tpr;
    g.upt = (g.U + g.tpr - 1) / g.tpr;
    const uint32_t G = 16 / gcd(g.rb, 16);  // rows whose bytes are a whole number of 16-byte vectors
    const uint32_t unit = G * g.slots / gcd(G, g.slots);
    uint32_t rs = 0;
    for (uint32_t m = 1;; ++m) {
        const uint32_t cand = unit * m;
        if (cand / g.slots > (uint32_t)MAX_RPT || cand > 32 * 8) break;
        const uint32_t alloc = (cand * g.rb + 16 + 127) & ~127u;
        if (2 * alloc + cand * 32 * 4 > SMEM_MAX) break;
        rs = cand;
        if (cand * g.rb >= 24 * 1024) break;  // enough bytes in flight per stage
    }
    if (rs == 0) return false;
    g.rs = rs;
    g.rpt = rs / g.slots;
    g.stage_alloc = (rs * g.rb + 16 + 127) & ~127u;
    g.red_off = 2 * g.stage_alloc;
    return true;
}

}  // namespace q6

int launch_q6k_dequant(const uint8_t *qb, float *w, uint64_t off, uint64_t n, cudaStream_t s) {
    if (n) k_q6k_dequant<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(qb, w, off, n);
    return (int)cudaGetLastError();
}
int launch_q6k_ordered(const uint8_t *qb, const float *x, float *y, uint32_t rows, uint32_t cols, cudaStream_t s) {
    if (rows) k_q6k_ordered<<<(rows + 127) / 128, 128, 0, s>>>(qb, x, y, rows, cols);
    return (int)cudaGetLastError();
}
int launch_q6k_part(const uint8_t *qb, const float *x, float *part, uint32_t rows, uint32_t cols, uint32_t parts,
                    cudaStream_t s) {
    const uint64_t n = (uint64_t)rows * parts;
    if (n) k_q6k_part<<<(unsigned)((n + 127) / 128), 128, 0, s>>>(qb, x, part, rows, cols, parts);
    return (int)cudaGetLastError();
}
int launch_q6k_matvec(const uint8_t *qb, const float *x, float *y, uint32_t rows, uint32_t cols, uint32_t ntok,
                      cudaStream_t s) {
    if (rows == 0 || ntok == 0) return 0;
    q6::Geo g;
    const bool stream = q6::plan(rows, cols, g) && (reinterpret_cast<uintptr_t>(qb) & 15) == 0 &&
                        (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (cols * 4) % 16 == 0;
    if (stream) {
        static unsigned long long set = 0;
        if (attr_pending(set)) {
            for (auto fn : {q6::k_q6k_stream<1>, q6::k_q6k_stream<2>, q6::k_q6k_stream<4>}) {
                const cudaError_t e =
                    cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, q6::SMEM_MAX);
                if (e != cudaSuccess) return (int)e;
            }
            attr_mark(set);
        }
        auto fn = g.upt == 1 ? q6::k_q6k_stream<1> : g.upt == 2 ? q6::k_q6k_stream<2> : q6::k_q6k_stream<4>;
        int dev = 0, nsm = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
        const uint32_t ngrp = (rows + g.rs - 1) / g.rs;
        const uint32_t per_sm = g.upt <= 2 ? 2u : 1u;
        const uint32_t grid = ngrp < per_sm * (uint32_t)nsm ? ngrp : per_sm * (uint32_t)nsm;
        const size_t smem = g.red_off + g.rs * 32 * 4;
        // token t: x + t * cols -> y + t * rows; the weights of a later token come from L2
        for (uint32_t t = 0; t < ntok; ++t)
            fn<<<grid, q6::NTHR, smem, s>>>(qb, x + (uint64_t)t * cols, y + (uint64_t)t * rows, g);
    } else {
        for (uint32_t t = 0; t < ntok; ++t)
            k_q6k_lane<<<(unsigned)(((uint64_t)rows * 32 + 255) / 256), 256, 0, s>>>(qb, x + (uint64_t)t * cols,
                                                                                   y + (uint64_t)t * rows, rows, cols);
    }
    return (int)cudaGetLastError();
}

}  // namespace ck
