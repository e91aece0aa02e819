// gemv_stream.cu -- HBM-streaming decode matvec for Q4_K and Q8_0 rows (cols % 256 == 0, cols <= 8192).
//
// y[r] = sum_j W[r, j] x[j], x and y fp32 (the fused form of form_q4k_matvec_f32, q4k-msl.fk:111-114,
// and form_q8_0_matvec_f32, q8-0-msl.fk:100-123).  Decode is bound by the weight stream, so the
// kernel is built to keep HBM busy rather than to keep registers busy:
//   * one producer lane per CTA copies groups of four weight rows into a shared-memory ring (four
//     stages, three CTAs per SM) with 1-D bulk copies (cp.async.bulk, completion counted on an
//     mbarrier), so the bytes in flight come from the ring depth, not from registers or occupancy;
//   * four consumer warps own fixed column slices -- a Q4_K 64-weight chunk, or two Q8_0 blocks,
//     per thread -- whose activations stay in registers for every row the CTA streams;
//   * codes become floats with one byte permute each and feed packed fp32 FMAs (__ffma2_rn): a
//     Q4_K nibble as 2 + q/64 (the constant folded into the sub-block's min term), a Q8_0 code as
//     2^23 + q + 128 less the offset; per sub-block or block the dot is factored as
//     scale * sum(q * x) (- min * sum(x) for Q4_K), the activation sums computed once.
// A row's warp partials are summed in warp order, one consumer barrier per group of four rows.
// Every wait is bounded (about one second); a CTA whose wait gives up writes NaN to its remaining
// rows.
#include "ck_common.cuh"
#include "ck_launch.h"

namespace ck {
namespace gv {

constexpr int NCONS = 4;                // consumer warps
constexpr int NTHR = (1 + NCONS) * 32;  // + the producer warp
constexpr uint32_t MAX_COLS = 8192;
#ifndef CK_GV_CTAS
#define CK_GV_CTAS 3  // CTAs per SM
#endif

CK_DEV void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
CK_DEV void consumer_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }


// Byte B of w over the float 2.0 in bits 16..23 (0x40 in the top byte): for a byte q < 128 the
// float is 2 * (1 + q / 128) = 2 + q / 64, exactly.
template <int B>
CK_DEV float two_plus(uint32_t w) { return __uint_as_float(__byte_perm(w, 0x40000000u, 0x7054u + (B << 8))); }
// Byte B of w over the float 2^23: 2^23 + byte, exactly.
template <int B>
CK_DEV float big_plus(uint32_t w) { return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540u + B)); }

// ------------------------------------------------------------------ Q4_K consumer: one chunk
struct Q4Slice {
    float2 xp[32];   // the chunk's 64 activations as 32 pairs
    float xs0, xs1;  // sums of the low-nibble (sub-block 2c) and high-nibble (2c+1) halves
};
CK_DEV void q4_load_x(Q4Slice &s, const float *x, uint32_t c, bool live) {
    float xs0 = 0.0f, xs1 = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const float4 v = live ? __ldg(reinterpret_cast<const float4 *>(x + (uint64_t)c * 64) + i) : make_float4(0, 0, 0, 0);
        s.xp[2 * i] = make_float2(v.x, v.y);
        s.xp[2 * i + 1] = make_float2(v.z, v.w);
        if (i < 8) xs0 += (v.x + v.y) + (v.z + v.w);
        else xs1 += (v.x + v.y) + (v.z + v.w);
    }
    s.xs0 = xs0;
    s.xs1 = xs1;
}
// The chunk's contribution from its 144-byte superblock in shared memory.  With v = 2 + q/64 per
// nibble, S = sum(v x) = 2 X + Q/64 (X = sum x, Q = sum q x), so the sub-block's
// (d sc) Q - (dmin m) X = 64 (d sc) S - (128 (d sc) + dmin m) X: one byte permute and one packed
// FMA per weight.  The cancellation costs a few fp32 roundings, far inside the matvec bound.
CK_DEV float q4_dot(const Q4Slice &s, const uint8_t *sblk, int cc) {
    const uint4 hdr = *reinterpret_cast<const uint4 *>(sblk);
    const uint4 qa = *reinterpret_cast<const uint4 *>(sblk + 16 + cc * 32);
    const uint4 qb = *reinterpret_cast<const uint4 *>(sblk + 32 + cc * 32);
    const uint32_t qw[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    float2 sl0 = make_float2(0.f, 0.f), sl1 = sl0, sh0 = sl0, sh1 = sl0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        // byte k of the chunk: low nibble = weight k (x pair k/2), high nibble = weight 32 + k
        const uint32_t lo = qw[j] & 0x0F0F0F0Fu, hi = (qw[j] >> 4) & 0x0F0F0F0Fu;
        sl0 = __ffma2_rn(make_float2(two_plus<0>(lo), two_plus<1>(lo)), s.xp[2 * j], sl0);
        sl1 = __ffma2_rn(make_float2(two_plus<2>(lo), two_plus<3>(lo)), s.xp[2 * j + 1], sl1);
        sh0 = __ffma2_rn(make_float2(two_plus<0>(hi), two_plus<1>(hi)), s.xp[16 + 2 * j], sh0);
        sh1 = __ffma2_rn(make_float2(two_plus<2>(hi), two_plus<3>(hi)), s.xp[16 + 2 * j + 1], sh1);
    }
    const float d = f16_bits_to_float(hdr.x & 0xFFFF), dmin = f16_bits_to_float(hdr.x >> 16);
    int sc0, m0, sc1, m1;
    q4k_scale_min(hdr.y, hdr.z, hdr.w, 2 * cc, sc0, m0);
    q4k_scale_min(hdr.y, hdr.z, hdr.w, 2 * cc + 1, sc1, m1);
    const float ds0 = d * (float)sc0, ds1 = d * (float)sc1;  // exact in fp32
    float a = (64.0f * ds0) * ((sl0.x + sl0.y) + (sl1.x + sl1.y));
    a = fmaf(-fmaf(128.0f, ds0, dmin * (float)m0), s.xs0, a);
    a = fmaf(64.0f * ds1, (sh0.x + sh0.y) + (sh1.x + sh1.y), a);
    return fmaf(-fmaf(128.0f, ds1, dmin * (float)m1), s.xs1, a);
}

// ------------------------------------------------------------------ Q8_0 consumer: one block
struct Q8Slice {
    float2 xp[16];  // the block's 32 activations as 16 pairs
};
CK_DEV void q8_load_x(Q8Slice &s, const float *x, uint32_t b, bool live) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 v = live ? __ldg(reinterpret_cast<const float4 *>(x + (uint64_t)b * 32) + i) : make_float4(0, 0, 0, 0);
        s.xp[2 * i] = make_float2(v.x, v.y);
        s.xp[2 * i + 1] = make_float2(v.z, v.w);
    }
}
// block b of the row in shared memory: 34 bytes at 34b, ODD = b & 1 (then the block starts 2 bytes
// into a word and its codes are word-aligned; an even block's codes straddle words).  Codes are
// biased to q + 128 (one XOR per word), become 2^23 + q + 128 exactly and lose the offset in one
// packed add.
template <int ODD>
CK_DEV float q8_dot(const Q8Slice &s, const uint8_t *row, uint32_t b) {
    const uint32_t *w = reinterpret_cast<const uint32_t *>(row + ((34 * b) & ~3u));
    uint32_t v[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) v[i] = w[i];
    const float d = f16_bits_to_float(ODD ? (v[0] >> 16) : (v[0] & 0xFFFF));
#pragma unroll
    for (int i = 0; i < 9; ++i) v[i] ^= 0x80808080u;
    const float2 off = make_float2(-8388736.0f, -8388736.0f);  // -(2^23 + 128)
    float2 s0 = make_float2(0.f, 0.f), s1 = s0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {  // codes 4j .. 4j+3
        float2 p01, p23;
        if (ODD) {  // codes at bytes 4 + 4j .. : word 1 + j
            p01 = make_float2(big_plus<0>(v[1 + j]), big_plus<1>(v[1 + j]));
            p23 = make_float2(big_plus<2>(v[1 + j]), big_plus<3>(v[1 + j]));
        } else {  // codes at bytes 2 + 4j .. : bytes 2,3 of word j and 0,1 of word j+1
            p01 = make_float2(big_plus<2>(v[j]), big_plus<3>(v[j]));
            p23 = make_float2(big_plus<0>(v[j + 1]), big_plus<1>(v[j + 1]));
        }
        s0 = __ffma2_rn(__fadd2_rn(p01, off), s.xp[2 * j], s0);
        s1 = __ffma2_rn(__fadd2_rn(p23, off), s.xp[2 * j + 1], s1);
    }
    return d * ((s0.x + s0.y) + (s1.x + s1.y));
}

// ------------------------------------------------------------------ the streaming kernel
// A ring stage holds a group of four consecutive rows (one bulk copy); CTA b streams the groups
// b, b + grid, ...  KIND 12: Q4_K (thread t owns chunk t % TPR); KIND 8: Q8_0 (blocks, see below).
template <int KIND>
__global__ void __launch_bounds__(NTHR, 3) k_gemv_stream(const uint8_t *__restrict__ qb, const float *__restrict__ x,
                                                      float *__restrict__ y, uint32_t rows, uint32_t cols,
                                                      uint32_t row_bytes, uint32_t stage_bytes, uint32_t lg_nst) {
    constexpr uint32_t GR = 4;  // rows per group (and per stage)
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~(uintptr_t)127);
    const uint32_t nst = 1u << lg_nst;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + nst * stage_bytes);
    uint64_t *empty = full + nst;
    float *red = reinterpret_cast<float *>(empty + nst);  // [2][NCONS][GR]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t ngr = (rows + GR - 1) / GR;
    const uint32_t nk = ngr > blockIdx.x ? (ngr - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < nst; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NCONS);
        }
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == 0) {
        if (lane == 0) {
            uint32_t k = 0;
            for (; k < nk; ++k) {
                const uint32_t s = k & (nst - 1);
                if (!mbar_wait_bounded(&empty[s], ((k >> lg_nst) & 1u) ^ 1u, nullptr, 0)) break;
                const uint32_t r0 = (blockIdx.x + k * gridDim.x) * GR;
                const uint32_t bytes = min(GR, rows - r0) * row_bytes;
                mbar_arrive_expect_tx(&full[s], bytes);
                bulk_g2s(smem + s * stage_bytes, qb + (uint64_t)r0 * row_bytes, bytes, &full[s]);
            }
            // the copies issued must land before the CTA exits
            for (uint32_t d = 0; d < nst && d < k; ++d) {
                const uint32_t j = k - 1 - d;
                mbar_wait_bounded(&full[j & (nst - 1)], (j >> lg_nst) & 1u, nullptr, 0);
            }
        }
        return;
    }

    // Consumers.  A row's units (Q4_K: 64-weight chunks; Q8_0: 32-weight blocks, two per thread
    // past 128) go to TPR threads; when TPR is a multiple of 32, RP = 128 / TPR rows of the group
    // share a pass (thread t reads row sub-index t / TPR), so each thread folds G = 4 / RP rows.
    const int t = threadIdx.x - 32, cw = warp - 1;
    const uint32_t units = KIND == 12 ? cols / 64 : cols / 32;
    const uint32_t upt = units > 128 ? 2 : 1, tpr = units / upt;
    const uint32_t rp = (tpr % 32 == 0 && tpr < 128) ? 128 / tpr : 1;
    const uint32_t rsub = (uint32_t)t / tpr, tu = (uint32_t)t % tpr;
    const bool live = rsub < rp;
    Q4Slice s4;
    Q8Slice s8a, s8b;
    uint32_t b8 = 0;
    if constexpr (KIND == 12) {
        q4_load_x(s4, x, tu, live);
    } else {
        // tpr in {64, 128}: a warp's blocks share their parity (no divergence between the odd and
        // even block layouts); otherwise block = unit
        b8 = (tpr % 64 == 0) ? 2 * (tu % (tpr / 2)) + tu / (tpr / 2) : tu;
        q8_load_x(s8a, x, b8, live);
        q8_load_x(s8b, x, b8 + 128, live && upt == 2);
    }
    const uint32_t G = GR / rp;
    const uint32_t wpr = rp == 1 ? (uint32_t)NCONS : tpr / 32;  // warps that hold one row's partials
    // Every consumer walks every group and every barrier: a warp whose wait gives up stops waiting
    // (its later reads are garbage) but keeps the barrier count, and its rows are written as NaN.
    bool ok = true;
    for (uint32_t k = 0; k < nk; ++k) {
        const uint32_t s = k & (nst - 1);
        const uint32_t r0 = (blockIdx.x + k * gridDim.x) * GR, nr = min(GR, rows - r0);
        if (ok && !mbar_wait_bounded(&full[s], (k >> lg_nst) & 1u, nullptr, 0)) ok = false;
        const uint8_t *stage = smem + s * stage_bytes;
        float part[GR];
#pragma unroll
        for (uint32_t g = 0; g < GR; ++g) {
            part[g] = 0.0f;
            const uint32_t j = g * rp + rsub;  // row of the group
            if (g < G && live && j < nr) {
                const uint8_t *row = stage + j * row_bytes;
                if constexpr (KIND == 12) {
                    part[g] = q4_dot(s4, row + (tu >> 2) * Q4K_BYTES, tu & 3);
                } else if (b8 & 1) {
                    part[g] = q8_dot<1>(s8a, row, b8);
                    if (upt == 2) part[g] += q8_dot<1>(s8b, row, b8 + 128);
                } else {
                    part[g] = q8_dot<0>(s8a, row, b8);
                    if (upt == 2) part[g] += q8_dot<0>(s8b, row, b8 + 128);
                }
            }
        }
        // this thread's shared-memory reads of the stage are done: order them before the bulk copy
        // that refills it, then release the stage once per warp
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        float *rb = red + (k & 1) * NCONS * GR;
#pragma unroll
        for (uint32_t g = 0; g < GR; ++g) {
            float v = part[g];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0 && g < G) rb[cw * GR + g] = v;
        }
        consumer_sync();
        if ((uint32_t)t < nr) {
            const uint32_t g = (uint32_t)t / rp, r = (uint32_t)t % rp;  // row t = g*rp + r
            float v = 0.0f;
            for (uint32_t w = r * wpr; w < (r + 1) * wpr; ++w) v += rb[w * GR + g];
            y[r0 + t] = ok ? v : __int_as_float(0x7FC00000);
        }
    }
}

}  // namespace gv

bool gemv_stream_ok(const void *qb, uint32_t cols) {
    return cols % 256 == 0 && cols <= gv::MAX_COLS && (reinterpret_cast<uintptr_t>(qb) & 15) == 0;
}

int launch_gemv_stream(int kind, const uint8_t *qb, const float *x, float *y, uint32_t rows, uint32_t cols,
                       cudaStream_t s) {
    if (!gemv_stream_ok(qb, cols)) return CK_ERR_SHAPE;
    if (rows == 0) return 0;
    const uint32_t row_bytes = kind == 12 ? cols / 256 * Q4K_BYTES : cols / 32 * Q80_BYTES;
    const uint32_t stage_bytes = (4 * row_bytes + 127) & ~127u;  // a group of four rows
    // ring: four stages within 72 KB (three CTAs per SM), else two
    const uint32_t lg_nst = 4 * stage_bytes <= 72 * 1024 ? 2 : 1;
    if ((stage_bytes << lg_nst) > 72 * 1024) return CK_ERR_SHAPE;
    const size_t smem = 128 + ((size_t)stage_bytes << lg_nst) + 2 * (8u << lg_nst) + 2 * gv::NCONS * 4 * 4;
    int dev = 0, nsm = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    const uint32_t ngr = (rows + 3) / 4;
    const unsigned grid = (unsigned)(ngr < (uint32_t)(CK_GV_CTAS * nsm) ? ngr : (uint32_t)(CK_GV_CTAS * nsm));
    if (kind == 12) {
        static bool attr = false;
        if (!attr) {
            cudaFuncSetAttribute(gv::k_gemv_stream<12>, cudaFuncAttributeMaxDynamicSharedMemorySize, 75 * 1024);
            attr = true;
        }
        gv::k_gemv_stream<12><<<grid, gv::NTHR, smem, s>>>(qb, x, y, rows, cols, row_bytes, stage_bytes, lg_nst);
    } else {
        static bool attr = false;
        if (!attr) {
            cudaFuncSetAttribute(gv::k_gemv_stream<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, 75 * 1024);
            attr = true;
        }
        gv::k_gemv_stream<8><<<grid, gv::NTHR, smem, s>>>(qb, x, y, rows, cols, row_bytes, stage_bytes, lg_nst);
    }
    return (int)cudaGetLastError();
}

}  // namespace ck
