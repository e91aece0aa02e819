// gemv_stream.cu -- HBM-streaming decode matvec for Q4_K and Q8_0 rows (cols % 256 == 0, cols <= 8192).
//
// y[r] = sum_j W[r, j] x[j], x and y fp32 (the fused form of form_q4k_matvec_f32, q4k-msl.fk:111-114,
// and form_q8_0_matvec_f32, q8-0-msl.fk:100-123).  Decode is bound by the weight stream, so the
// kernel is built to keep HBM busy rather than to keep registers busy:
//   * one CTA per SM holds three row groups; each group's producer lane copies stages of rows into
//     the group's shared-memory sub-ring with 1-D bulk copies (cp.async.bulk, completion counted
//     on an mbarrier), so the bytes in flight come from the ring depth, not from occupancy;
//   * x is read once per CTA with coalesced loads into a padded shared-memory copy (16 bytes of pad
//     per 1 KB for Q4_K, per 256 bytes for Q8_0) so that the lanes of a warp, which own units 1 KB
//     or 256 bytes apart, fetch their slices without bank conflicts;
//   * every consumer thread owns one fixed 64-weight column unit -- a Q4_K chunk (a quarter of a
//     superblock: sub-blocks 2c and 2c+1) or a pair of Q8_0 blocks -- whose activations stay in
//     registers for every row the group streams, and folds four (Q4_K) or two (Q8_0) rows of each
//     stage at once;
//   * for Q4_K the four consumer warps of a group are the four chunk positions c (warp-uniform
//     scale unpack) and lanes index superblocks; one code path serves all four (a copy of the
//     unrolled row loop per chunk position overflows the instruction cache and runs 1.7x slower);
//   * codes become floats with one byte permute each and feed packed fp32 FMAs (__ffma2_rn): a
//     Q4_K nibble as 2 + q/64 (the constant folded into the sub-block's min term), a Q8_0 code as
//     2^23 + q + 128 less the offset; per sub-block or block the dot is factored as
//     scale * sum(q * x) (- min * sum(x) for Q4_K), the activation sums computed once;
//   * a thread's row partials are summed across the lanes of its row slot by a transposed
//     butterfly (each exchange halves the rows a lane carries), then across warps in shared
//     memory in warp order -- a fixed order, so results are deterministic.
// Launched with programmatic stream serialization: the next kernel in the stream may be scheduled
// while this one drains, and every thread waits for the previous kernel (griddepcontrol.wait)
// before it reads x or writes y, so stream order is kept; only the producers' first stages of
// packed weights, which no kernel of this library writes, are copied before that wait.
// Every wait is bounded (about one second); a row group whose wait gives up writes NaN to its
// remaining rows.
#include "ck_common.cuh"
#include "ck_launch.h"

namespace ck {
namespace gv {

constexpr int NCONS = 4;  // consumer warps per row group
constexpr int NRG = 3;    // row groups per CTA
constexpr int NTHR = NRG * (1 + NCONS) * 32;
constexpr uint32_t MAX_COLS = 8192;
constexpr uint32_t SMEM_MAX = 224 * 1024;  // dynamic shared memory of the one CTA per SM

CK_DEV void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
CK_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
CK_DEV void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Byte B of w over the float 2.0 in bits 16..23 (0x40 in the top byte): for a byte q < 128 the
// float is 2 * (1 + q / 128) = 2 + q / 64, exactly.
template <int B>
CK_DEV float two_plus(uint32_t w) { return __uint_as_float(__byte_perm(w, 0x40000000u, 0x7054u + (B << 8))); }
// Byte B of w over the float 2^23: 2^23 + byte, exactly.
template <int B>
CK_DEV float big_plus(uint32_t w) { return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540u + B)); }
// A 6-bit field as a float: 2^23 + v less 2^23, exact.
CK_DEV float small_int_float(uint32_t v) { return __uint_as_float(v | 0x4B000000u) - 8388608.0f; }

// The 64 activations of a thread's unit as 32 pairs, and the sums of its two 32-wide halves, read
// from the CTA's padded shared-memory copy of x (pad: 4 floats after every 2^lgp floats).
struct XSlice {
    float2 xp[32];
    float xlo, xhi;
};
CK_DEV void load_x(XSlice &s, const float *xs_smem, uint32_t unit, uint32_t lgp, bool live) {
    float a = 0.0f, b = 0.0f;
    const uint32_t e = unit * 64;
    const float4 *src = reinterpret_cast<const float4 *>(xs_smem + e + ((e >> lgp) << 2));
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const float4 v = live ? src[i] : make_float4(0, 0, 0, 0);
        s.xp[2 * i] = make_float2(v.x, v.y);
        s.xp[2 * i + 1] = make_float2(v.z, v.w);
        if (i < 8) a += (v.x + v.y) + (v.z + v.w);
        else b += (v.x + v.y) + (v.z + v.w);
    }
    s.xlo = a;
    s.xhi = b;
}

// ------------------------------------------------------------------ Q4_K: chunk c of a superblock
// Scales and mins of sub-blocks 2c and 2c+1 (get_scale_min_k4) from the three little-endian scale
// words Y = bytes 0..3, Z = 4..7, W = 8..11; c is uniform across a warp, so the branch is too.
CK_DEV void q4_scales(uint32_t Y, uint32_t Z, uint32_t W, uint32_t c, float &sc0, float &m0, float &sc1, float &m1) {
    uint32_t a0, b0, a1, b1;
    if (c < 2) {  // j < 4: scales[j] & 63, scales[j + 4] & 63
        const uint32_t s0 = 16 * c, s1 = s0 + 8;
        a0 = (Y >> s0) & 63u;
        b0 = (Z >> s0) & 63u;
        a1 = (Y >> s1) & 63u;
        b1 = (Z >> s1) & 63u;
    } else {  // j >= 4: low / high nibble of scales[j + 4], top bits of scales[j - 4] / scales[j]
        const uint32_t s0 = 16 * (c - 2), s1 = s0 + 8;
        a0 = ((W >> s0) & 0xFu) | ((Y >> (s0 + 2)) & 0x30u);
        b0 = ((W >> (s0 + 4)) & 0xFu) | ((Z >> (s0 + 2)) & 0x30u);
        a1 = ((W >> s1) & 0xFu) | ((Y >> (s1 + 2)) & 0x30u);
        b1 = ((W >> (s1 + 4)) & 0xFu) | ((Z >> (s1 + 2)) & 0x30u);
    }
    sc0 = small_int_float(a0);
    m0 = small_int_float(b0);
    sc1 = small_int_float(a1);
    m1 = small_int_float(b1);
}
// The chunk's contribution from its superblock in shared memory.  With v = 2 + q/64 per nibble,
// S = sum(v x) = 2 X + Q/64 (X = sum x, Q = sum q x), so Q = 64 S - 128 X and the two sub-blocks
// give d (sc0 Q0 + sc1 Q1) - dmin (m0 X0 + m1 X1): one byte permute and half a packed FMA per
// weight.  The cancellation costs a few fp32 roundings, far inside the matvec bound.
CK_DEV float q4_dot(const XSlice &s, const uint8_t *sblk, uint32_t c) {
    const uint4 hdr = *reinterpret_cast<const uint4 *>(sblk);
    const uint4 qa = *reinterpret_cast<const uint4 *>(sblk + 16 + c * 32);
    const uint4 qb = *reinterpret_cast<const uint4 *>(sblk + 32 + c * 32);
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
    float sc0, m0, sc1, m1;
    q4_scales(hdr.y, hdr.z, hdr.w, c, sc0, m0, sc1, m1);
    const float d = f16_bits_to_float(hdr.x & 0xFFFF), dmin = f16_bits_to_float(hdr.x >> 16);
    const float q0 = fmaf(64.0f, (sl0.x + sl0.y) + (sl1.x + sl1.y), -128.0f * s.xlo);
    const float q1 = fmaf(64.0f, (sh0.x + sh0.y) + (sh1.x + sh1.y), -128.0f * s.xhi);
    const float qs = fmaf(sc1, q1, sc0 * q0), mx = fmaf(m1, s.xhi, m0 * s.xlo);
    return fmaf(d, qs, -dmin * mx);
}

// ------------------------------------------------------------------ Q8_0: a pair of blocks
// The pair is 68 bytes at 68 p (word aligned): the even block's d in bytes 0..1 and codes in
// 2..33 (straddling words), the odd block's d in 34..35 and codes in 36..67 (word aligned).
// Codes are biased to q + 128 (one XOR per word), become 2^23 + q + 128 exactly and lose the
// offset in one packed add.
CK_DEV float q8_pair(const XSlice &s, const uint8_t *pair) {
    const uint32_t *w = reinterpret_cast<const uint32_t *>(pair);
    uint32_t v[17];
#pragma unroll
    for (int i = 0; i < 17; ++i) v[i] = w[i];
    const float de = f16_bits_to_float(v[0] & 0xFFFF), dodd = f16_bits_to_float(v[8] >> 16);
    v[0] ^= 0x80800000u;
    v[8] ^= 0x00008080u;
#pragma unroll
    for (int i = 1; i < 17; ++i)
        if (i != 8) v[i] ^= 0x80808080u;
    const float2 off = make_float2(-8388736.0f, -8388736.0f);  // -(2^23 + 128)
    float2 e0 = make_float2(0.f, 0.f), e1 = e0, o0 = e0, o1 = e0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        // even codes 4j .. 4j+3: bytes 2, 3 of word j and 0, 1 of word j+1
        const float2 a = make_float2(big_plus<2>(v[j]), big_plus<3>(v[j]));
        const float2 b = make_float2(big_plus<0>(v[j + 1]), big_plus<1>(v[j + 1]));
        e0 = __ffma2_rn(__fadd2_rn(a, off), s.xp[2 * j], e0);
        e1 = __ffma2_rn(__fadd2_rn(b, off), s.xp[2 * j + 1], e1);
        // odd codes 4j .. 4j+3: word 9 + j
        const float2 c = make_float2(big_plus<0>(v[9 + j]), big_plus<1>(v[9 + j]));
        const float2 e = make_float2(big_plus<2>(v[9 + j]), big_plus<3>(v[9 + j]));
        o0 = __ffma2_rn(__fadd2_rn(c, off), s.xp[16 + 2 * j], o0);
        o1 = __ffma2_rn(__fadd2_rn(e, off), s.xp[16 + 2 * j + 1], o1);
    }
    return fmaf(de, (e0.x + e0.y) + (e1.x + e1.y), dodd * ((o0.x + o0.y) + (o1.x + o1.y)));
}

// ------------------------------------------------------------------ the streaming kernel
// One CTA per SM: NRG row groups, each a producer warp (one lane issues its bulk copies) and four
// consumer warps with a private sub-ring of nsub stages, so the groups stream independently.  A
// stage holds GR = rpt * slots consecutive rows (one bulk copy); the CTA's k-th stage holds row
// group blockIdx.x + k * gridDim.x and goes to row group k % NRG.  A consumer thread serves row
// slot `slot` and folds rows i * slots + slot, i < rpt, of each stage.
//   Q4_K (rpt 4): warp c of the group holds chunk c of superblock `lane % lg` (lg = superblocks
//         per row rounded up to a power of two), slot = lane / lg; a row's partials come from all
//         four warps.
//   Q8_0 (rpt 2): group thread t holds block pair t % tps (tps = pairs per row rounded up to a
//         power of two), slot = t / tps; a row's partials come from max(1, tps / 32) warps.
struct Geo {
    uint32_t rows, cols, row_bytes, stage_bytes, nsub;
    uint32_t lg;     // lanes of one row slot within a warp (power of two, <= 32)
    uint32_t slots;  // row slots per stage
    uint32_t tps;    // Q8_0: threads per row slot
    uint32_t lgp;    // x padding period: 4 floats of pad after every 2^lgp floats
    uint32_t ring_off, bar_off, red_off;  // shared-memory layout: x at 0, then ring, barriers, partials
};

// Sum v[0..R) over the lg (>= R) lanes of a slot by a transposed butterfly.  On return the lane
// holds the sum for row `row` of the slot, and `writer` marks one lane per (slot, row).
template <int R>
CK_DEV float slot_reduce(const float (&v)[R], uint32_t lane, uint32_t lg, uint32_t &row, bool &writer) {
    const uint32_t o1 = lg >> 1;
    const bool b1 = (lane & o1) != 0;
    if constexpr (R == 4) {
        const uint32_t o2 = lg >> 2;
        const bool b2 = (lane & o2) != 0;
        // keep rows {2,3} or {0,1}; send the other two
        float k0 = b1 ? v[2] : v[0], k1 = b1 ? v[3] : v[1];
        const float s0 = b1 ? v[0] : v[2], s1 = b1 ? v[1] : v[3];
        k0 += __shfl_xor_sync(0xffffffffu, s0, o1);
        k1 += __shfl_xor_sync(0xffffffffu, s1, o1);
        float k = b2 ? k1 : k0;
        k += __shfl_xor_sync(0xffffffffu, b2 ? k0 : k1, o2);
        for (uint32_t o = lg >> 3; o > 0; o >>= 1) k += __shfl_xor_sync(0xffffffffu, k, o);
        row = (b1 ? 2u : 0u) + (b2 ? 1u : 0u);
        writer = (lane & (o2 - 1)) == 0;
        return k;
    } else {
        float k = b1 ? v[1] : v[0];
        k += __shfl_xor_sync(0xffffffffu, b1 ? v[0] : v[1], o1);
        for (uint32_t o = lg >> 2; o > 0; o >>= 1) k += __shfl_xor_sync(0xffffffffu, k, o);
        row = b1 ? 1u : 0u;
        writer = (lane & (o1 - 1)) == 0;
        return k;
    }
}

template <int KIND>
CK_DEV void consume(const Geo &g, const float *__restrict__ x, float *__restrict__ y, uint8_t *smem, uint32_t rg,
                    uint32_t nkg) {
    constexpr int R = KIND == 12 ? 4 : 2;
    const uint32_t lane = threadIdx.x & 31, c = ((threadIdx.x >> 5) - NRG) & 3, tg = c * 32 + lane;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + g.bar_off) + rg * g.nsub;
    uint64_t *empty = full + NRG * g.nsub;
    float *red = reinterpret_cast<float *>(smem + g.red_off) + rg * 2 * NCONS * 128;
    const uint8_t *ring = smem + g.ring_off + rg * g.nsub * g.stage_bytes;
    float *xs_smem = reinterpret_cast<float *>(smem);
    uint32_t slot, unit, uoff;
    bool live;
    if constexpr (KIND == 12) {
        const uint32_t nsb = g.cols / 256, sb = lane % g.lg;
        slot = lane / g.lg;
        live = sb < nsb;
        unit = (live ? sb : 0) * 4 + c;
        uoff = (live ? sb : 0) * Q4K_BYTES;
    } else {
        const uint32_t np = g.cols / 64, p = tg % g.tps;
        slot = tg / g.tps;
        live = p < np;
        unit = live ? p : 0;
        uoff = unit * 68;
    }
    // x into the padded shared copy: coalesced 16-byte loads by all consumer threads
    pdl_wait();
    for (uint32_t i = threadIdx.x - NRG * 32; i < g.cols / 4; i += NRG * NCONS * 32) {
        const float4 v = __ldg(reinterpret_cast<const float4 *>(x) + i);
        const uint32_t e = 4 * i;
        *reinterpret_cast<float4 *>(xs_smem + e + ((e >> g.lgp) << 2)) = v;
    }
    asm volatile("bar.sync %0, %1;" ::"r"(1 + NRG), "r"(NRG * NCONS * 32) : "memory");
    XSlice xs;
    load_x(xs, xs_smem, unit, g.lgp, live);
    const uint32_t GR = R * g.slots, lg = g.lg;
    bool ok = true;
    for (uint32_t kk = 0; kk < nkg; ++kk) {
        const uint32_t st = kk % g.nsub, ph = (kk / g.nsub) & 1u;
        const uint32_t r0 = (blockIdx.x + (kk * NRG + rg) * gridDim.x) * GR, nr = min(GR, g.rows - r0);
        if (ok && !mbar_wait_bounded(&full[st], ph, nullptr, 0)) ok = false;
        const uint8_t *stage = ring + st * g.stage_bytes;
        float part[R];
#pragma unroll
        for (int i = 0; i < R; ++i) {
            const uint32_t j = min(i * g.slots + slot, nr - 1);  // rows past the stage's end re-read its last
            const uint8_t *src = stage + j * g.row_bytes + uoff;
            if constexpr (KIND == 12) part[i] = q4_dot(xs, src, c);
            else part[i] = q8_pair(xs, src);
            part[i] = live ? part[i] : 0.0f;
        }
        // this thread's shared-memory reads of the stage are done: order them before the bulk copy
        // that refills it, then release the stage once per warp
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
        float *rb = red + (kk & 1) * NCONS * 128;
        if (lg >= (uint32_t)R) {
            uint32_t row;
            bool writer;
            const float v = slot_reduce<R>(part, lane, lg, row, writer);
            if (writer) rb[c * 128 + row * g.slots + slot] = v;
        } else {  // fewer lanes per slot than rows: each writer lane stores all its rows
#pragma unroll
            for (int i = 0; i < R; ++i) {
                float u = part[i];
                if (lg == 2) u += __shfl_xor_sync(0xffffffffu, u, 1);
                if ((lane & (lg - 1)) == 0) rb[c * 128 + i * g.slots + slot] = u;
            }
        }
        asm volatile("bar.sync %0, 128;" ::"r"(1 + rg) : "memory");
        if (tg < nr) {
            float acc;
            if constexpr (KIND == 12) {
                acc = ((rb[tg] + rb[128 + tg]) + rb[256 + tg]) + rb[384 + tg];
            } else {
                const uint32_t sl = tg % g.slots;
                const uint32_t w0 = sl * g.tps / 32, nw = g.tps >= 32 ? g.tps / 32 : 1;
                acc = 0.0f;
                for (uint32_t w = w0; w < w0 + nw; ++w) acc += rb[w * 128 + tg];
            }
            y[r0 + tg] = ok ? acc : __int_as_float(0x7FC00000);
        }
    }
}

template <int KIND>
__global__ void __launch_bounds__(NTHR, 1) k_gemv_stream(const uint8_t *__restrict__ qb, const float *__restrict__ x,
                                                       float *__restrict__ y, Geo g) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + g.bar_off);  // full[NRG][nsub], empty[NRG][nsub]
    const uint32_t nst = NRG * g.nsub;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t GR = (KIND == 12 ? 4 : 2) * g.slots;
    const uint32_t ngr = (g.rows + GR - 1) / GR;
    const uint32_t nk = ngr > blockIdx.x ? (ngr - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < nst; ++s) {
            mbar_init(&bars[s], 1);
            mbar_init(&bars[nst + s], NCONS);
        }
        fence_barrier_init();
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp < NRG) {  // producer of row group `warp`
        if (lane == 0) {
            const uint32_t rg = warp, nkg = nk > rg ? (nk - rg + NRG - 1) / NRG : 0;
            uint64_t *full = bars + rg * g.nsub, *empty = bars + nst + rg * g.nsub;
            uint8_t *ring = smem + g.ring_off + rg * g.nsub * g.stage_bytes;
            // the weights are never written by the kernel before this one (no kernel of this library
            // writes packed weights): the sub-ring's first stages are filled before the wait on it,
            // overlapping its tail
            uint32_t kk = 0;
            for (; kk < nkg; ++kk) {
                if (kk == g.nsub) pdl_wait();
                const uint32_t st = kk % g.nsub, ph = (kk / g.nsub) & 1u;
                if (!mbar_wait_bounded(&empty[st], ph ^ 1u, nullptr, 0)) break;
                const uint32_t r0 = (blockIdx.x + (kk * NRG + rg) * gridDim.x) * GR;
                const uint32_t bytes = min(GR, g.rows - r0) * g.row_bytes;
                mbar_arrive_expect_tx(&full[st], bytes);
                bulk_g2s(ring + st * g.stage_bytes, qb + (uint64_t)r0 * g.row_bytes, bytes, &full[st]);
            }
            if (kk <= g.nsub) pdl_wait();
            // the copies issued must land before the CTA exits: wait for the last min(nsub, kk)
            for (uint32_t d = 0; d < g.nsub && d < kk; ++d) {
                const uint32_t j = kk - 1 - d;
                mbar_wait_bounded(&full[j % g.nsub], (j / g.nsub) & 1u, nullptr, 0);
            }
        }
        return;
    }
    const uint32_t rg = (uint32_t)(warp - NRG) >> 2, nkg = nk > rg ? (nk - rg + NRG - 1) / NRG : 0;
    consume<KIND>(g, x, y, smem, rg, nkg);
}

uint32_t pow2_ceil(uint32_t v) {
    uint32_t p = 1;
    while (p < v) p <<= 1;
    return p;
}

template <int KIND>
cudaError_t launch_kind(const cudaLaunchConfig_t &cfg, const uint8_t *qb, const float *x, float *y, const Geo &g) {
    static unsigned long long set = 0;
    if (attr_pending(set)) {
        const cudaError_t e =
            cudaFuncSetAttribute(k_gemv_stream<KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_MAX);
        if (e != cudaSuccess) return e;
        attr_mark(set);
    }
    return cudaLaunchKernelEx(&cfg, k_gemv_stream<KIND>, qb, x, y, g);
}

}  // namespace gv

bool gemv_stream_ok(const void *qb, const float *x, uint32_t cols) {
    return cols % 256 == 0 && cols > 0 && cols <= gv::MAX_COLS && (reinterpret_cast<uintptr_t>(qb) & 15) == 0 &&
           (reinterpret_cast<uintptr_t>(x) & 15) == 0;
}

int launch_gemv_stream(int kind, const uint8_t *qb, const float *x, float *y, uint32_t rows, uint32_t cols,
                       cudaStream_t s) {
    if (!gemv_stream_ok(qb, x, cols)) return CK_ERR_SHAPE;
    if (rows == 0) return 0;
    gv::Geo g = {};
    g.rows = rows;
    g.cols = cols;
    uint32_t rpt;
    if (kind == 12) {
        rpt = 4;
        g.row_bytes = cols / 256 * Q4K_BYTES;
        g.lg = gv::pow2_ceil(cols / 256);
        g.slots = 32 / g.lg;
        g.tps = 0;
        g.lgp = 8;  // lanes own units 1 KB apart
    } else {
        rpt = 2;
        g.row_bytes = cols / 32 * Q80_BYTES;
        g.tps = gv::pow2_ceil(cols / 64);  // cols % 256 == 0: 4 .. 128
        g.lg = g.tps < 32 ? g.tps : 32;
        g.slots = 128 / g.tps;
        g.lgp = 6;  // lanes own units 256 bytes apart
    }
    // padded x, then NRG sub-rings of as many stages (2 .. 4) as fit, the barriers and the partials
    g.stage_bytes = (rpt * g.slots * g.row_bytes + 127) & ~127u;
    g.ring_off = (cols * 4 + ((cols >> g.lgp) << 4) + 127) & ~127u;
    const uint32_t tail = 2 * gv::NRG * 4 * 8 + 128 + gv::NRG * 2 * gv::NCONS * 128 * 4;
    g.nsub = (gv::SMEM_MAX - g.ring_off - tail) / (gv::NRG * g.stage_bytes);
    if (g.nsub > 4) g.nsub = 4;
    if (g.nsub < 2) return CK_ERR_SHAPE;
    g.bar_off = g.ring_off + gv::NRG * g.nsub * g.stage_bytes;
    g.red_off = g.bar_off + ((2 * gv::NRG * g.nsub * 8 + 127) & ~127u);
    const size_t smem = g.red_off + gv::NRG * 2 * gv::NCONS * 128 * 4;
    int dev = 0, nsm = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    const uint32_t GR = rpt * g.slots, ngr = (rows + GR - 1) / GR;
    const unsigned grid = (unsigned)(ngr < (uint32_t)nsm ? ngr : (uint32_t)nsm);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(gv::NTHR);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = kind == 12 ? gv::launch_kind<12>(cfg, qb, x, y, g) : gv::launch_kind<8>(cfg, qb, x, y, g);
    return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

}  // namespace ck
