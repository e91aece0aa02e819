// tc_i8.cuh -- helpers shared by the integer tensor-core matvec kernels (gemv_tc.cu, moe_gemv.cu):
// kind::i8 MMA issue from an elected lane, TMA loads, tensor-memory loads, programmatic dependent
// launch, and the fixed-point digits of an activation sub-block.
//
// The activation scheme: 32 consecutive x (one Q4_K sub-block) are held as X = rint(x 2^(22-e)),
// e the sub-block's power-of-two bound on |x| (|x| < 2^e), and X is split into three balanced
// base-256 digits X = 65536 l0 + 256 l1 + l2, each in [-128, 127], that an s8 MMA operand takes
// exactly.  Against u8 weight codes the MMA's int32 sums are exact; the epilogue weighs the three
// digit sums by 65536, 256, 1 and the sub-block's 2^(e-22).
#pragma once
#include "ck_common.cuh"

namespace ck {
namespace tci8 {

// one lane of a converged warp: a tcgen05.mma issued by a lone diverged thread issues several
// times slower than a narrow tile takes to compute
CK_DEV bool elect_one() {
    uint32_t pred = 0;
    asm volatile("{\n .reg .b32 %%rx;\n .reg .pred %%px;\n elect.sync %%rx|%%px, %1;\n selp.u32 %0, 1, 0, %%px;\n}"
                 : "=r"(pred)
                 : "r"(0xffffffffu));
    return pred != 0;
}
// kind::i8 instruction descriptor: D s32, A u8, B s8, both K-major, M x N
__host__ __device__ constexpr uint32_t idesc_u8s8(int M, int N) {
    return (2u << 4) | (0u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
// D[tmem] (+)= A[tmem] * B[smem desc]^T, u8 x s8 -> s32
CK_DEV void umma_i8_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
CK_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
CK_DEV void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
CK_DEV void tma_load_3d(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
        "[%2];" ::"r"(smem_u32(dst)),
        "l"((uint64_t)map), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
        : "memory");
}
CK_DEV void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}
CK_DEV void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
// 16-byte asynchronous global -> shared copies (completion per commit group)
CK_DEV void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
CK_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
CK_DEV void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
// bytes 0 of a, b, c, d packed low to high
CK_DEV uint32_t pack_b0(int a, int b, int c, int d) {
    return __byte_perm(__byte_perm((uint32_t)a, (uint32_t)b, 0x0040), __byte_perm((uint32_t)c, (uint32_t)d, 0x0040),
                       0x5410);
}
// byte offset of (row n, K kk) in a [rows x 128] s8 tile with the 128-byte swizzle
CK_DEV uint32_t b_off(int n, int kk) {
    return (uint32_t)((n >> 3) * 1024 + (n & 7) * 128 + ((((kk >> 4) ^ (n & 7))) << 4) + (kk & 15));
}
// The sub-block exponent e (|x| < 2^e; 0 for an all-zero sub-block; kept in [-100, 129]) from the
// largest |x|, and the three digits of eight x of the sub-block, packed as two words per digit.
CK_DEV int subblock_exponent(float mx) {
    const int e = (int)((__float_as_uint(mx) >> 23) & 255u) - 126;
    return mx == 0.0f ? 0 : max(-100, e);
}
CK_DEV void digits8(const float (&xv)[8], int e, uint2 &w0, uint2 &w1, uint2 &w2) {
    const float up = __uint_as_float((uint32_t)(127 + 22 - e) << 23);  // 2^(22-e)
    int d0[8], d1[8], d2[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int X = __float2int_rn(xv[i] * up);  // |X| <= 2^22
        const int X1 = (X + 128) >> 8, X0 = (X1 + 128) >> 8;
        d2[i] = X;  // low bytes: the balanced digits
        d1[i] = X1;
        d0[i] = X0;
    }
    w0 = make_uint2(pack_b0(d0[0], d0[1], d0[2], d0[3]), pack_b0(d0[4], d0[5], d0[6], d0[7]));
    w1 = make_uint2(pack_b0(d1[0], d1[1], d1[2], d1[3]), pack_b0(d1[4], d1[5], d1[6], d1[7]));
    w2 = make_uint2(pack_b0(d2[0], d2[1], d2[2], d2[3]), pack_b0(d2[4], d2[5], d2[6], d2[7]));
}
// 2^(e - 22 - extra): the weight of a digit sum of the sub-block (extra = 4 where the weight codes
// sit in the high nibble of their byte, i.e. hold 16 q)
CK_DEV float digit_scale(int e, int extra) { return __uint_as_float((uint32_t)(127 - 22 - extra + e) << 23); }
// the weighted sum of a sub-block's three exact digit sums (each below 2^24 in magnitude, so
// exact as floats; their combination can exceed int32)
CK_DEV float digit_sum(uint32_t d0, uint32_t d1, uint32_t d2) {
    return fmaf((float)(int)d0, 65536.0f, fmaf((float)(int)d1, 256.0f, (float)(int)d2));
}

}  // namespace tci8

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
// cuTensorMapEncodeTiled through the runtime's driver entry point (null if unavailable)
EncodeTiledFn tensor_map_encoder();

}  // namespace ck
