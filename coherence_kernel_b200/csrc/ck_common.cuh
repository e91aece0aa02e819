// ck_common.cuh -- shared device helpers for the sm_100a kernels of the quantized path:
// GGUF block field decoding, bf16 packing, and thin inline-PTX wrappers for mbarriers, TMA and
// the 5th-generation tensor core (tcgen05 / TMEM).
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define CK_DEV __device__ __forceinline__

namespace ck {

// Kernel attributes such as the dynamic shared-memory limit belong to a device, so a process that
// drives several GPUs sets them on each: one bit per device (up to 64) of a call site's `done` word.
inline bool attr_pending(unsigned long long done) {
    int dev = 0;
    cudaGetDevice(&dev);
    return !((done >> (dev & 63)) & 1ull);
}
inline void attr_mark(unsigned long long &done) {
    int dev = 0;
    cudaGetDevice(&dev);
    done |= 1ull << (dev & 63);
}


// ----------------------------------------------------------------------------- GGUF fields
// block_q8_0: f16 d @0, int8 qs[32] @2 (34 bytes); block_q4_K: f16 d @0, f16 dmin @2,
// scales[12] @4, qs[128] @16 (144 bytes).  The f16 decode is IEEE half -> float (exact).
constexpr int Q80_BYTES = 34;
constexpr int Q4K_BYTES = 144;

CK_DEV float f16_bits_to_float(uint32_t bits) {
    return __half2float(__ushort_as_half((unsigned short)(bits & 0xFFFFu)));
}

// get_scale_min_k4 over the 12 packed scale bytes held as three little-endian words.
// The three scale words are taken by value and picked apart with shifts: indexing an array of
// them with the run-time sub-block j would put it in local memory.
CK_DEV void q4k_scale_min(uint32_t s0, uint32_t s1, uint32_t s2, int j, int &sc, int &mn) {
    const int sh = (j & 3) * 8;
    const int b0 = (int)((s0 >> sh) & 0xFFu), b1 = (int)((s1 >> sh) & 0xFFu), b2 = (int)((s2 >> sh) & 0xFFu);
    if (j < 4) {
        sc = b0 & 63;  // scales[j]
        mn = b1 & 63;  // scales[j + 4]
    } else {
        sc = (b2 & 0xF) | ((b0 >> 6) << 4);  // scales[j + 4] low nibble, scales[j - 4] top bits
        mn = (b2 >> 4) | ((b1 >> 6) << 4);   // scales[j + 4] high nibble, scales[j] top bits
    }
}
CK_DEV void q4k_scale_min(const uint32_t s[3], int j, int &sc, int &mn) { q4k_scale_min(s[0], s[1], s[2], j, sc, mn); }

CK_DEV uint32_t pack_bf16x2(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}

CK_DEV float bf16_bits_to_float(uint16_t b) { return __uint_as_float(((uint32_t)b) << 16); }

CK_DEV uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

// ----------------------------------------------------------------------------- mbarrier
CK_DEV void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
CK_DEV void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
CK_DEV void mbar_arrive(uint64_t *bar) {
    asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.shared::cta.b64 st, [%0];\n}" ::"r"(smem_u32(bar)) : "memory");
}
CK_DEV void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n}" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}
CK_DEV bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Non-blocking probe of a phase: far cheaper than try_wait when the phase has already completed.
CK_DEV bool mbar_test_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
CK_DEV uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
// Bounded wait: gives up after `limit_ns` (about one second in every pipeline), records `code` in
// the error word and returns false, so a broken pipeline ends the kernel with a status the host
// reads instead of hanging.
CK_DEV bool mbar_wait_bounded_ns(uint64_t *bar, uint32_t parity, int *err, int code, uint64_t limit_ns) {
    if (mbar_test_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 1023u) == 0) {
            if (err && *(volatile int *)err) return false;  // another role already gave up
            if (globaltimer_ns() - t0 > limit_ns) break;
        }
    }
    if (err) atomicCAS(err, 0, code);
    return false;
}
CK_DEV bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, int *err, int code) {
    return mbar_wait_bounded_ns(bar, parity, err, code, 1000000000ull);
}

// ----------------------------------------------------------------------------- TMA
CK_DEV void tma_load_2d(void *smem_dst, const CUtensorMap *map, uint64_t *bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(smem_dst)),
        "l"((uint64_t)map), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}
CK_DEV void prefetch_tmap(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)map) : "memory");
}
CK_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ----------------------------------------------------------------------------- dependent launch
// Kernels launched with programmatic stream serialization (launch_pdl) may start while the kernel
// before them finishes: each calls grid_dep_trigger (let the next one be scheduled) and then
// grid_dep_wait (the previous kernel has completed and its writes are visible) before its first
// global-memory access.  Both are no-ops for a kernel launched without the attribute.
CK_DEV void grid_dep_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
// An early trigger only from a grid that fits on the GPU at once (one CTA per SM of a B200 at
// most): the next kernel's CTAs then wait on otherwise idle SMs.  From a larger grid they would take
// SM room from the CTAs still running, so such a grid triggers implicitly as its CTAs exit.
CK_DEV void grid_dep_trigger_small() {
    if (gridDim.x * gridDim.y * gridDim.z <= 148u) grid_dep_trigger();
}
CK_DEV void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args &&...args) {
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// ----------------------------------------------------------------------------- tcgen05
CK_DEV void tmem_alloc(uint32_t *smem_slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_slot)),
                 "r"(ncols)
                 : "memory");
}
CK_DEV void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
CK_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
CK_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
CK_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, bf16 inputs, fp32 accumulate, one elected thread.
CK_DEV void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]^T with the A tile in tensor memory: row i of A in lane i,
// K packed two bf16 per 32-bit column in K order (the lower K in the low half), 8 columns per
// K = 16 step.
CK_DEV void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive on an mbarrier once every tcgen05 op issued so far by this thread has completed.
CK_DEV void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
// 32 lanes x 32 consecutive fp32 columns (this warp's TMEM sub-partition).
CK_DEV void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
CK_DEV void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// 32 lanes x 32 consecutive 32-bit columns from registers (this warp's TMEM sub-partition).
CK_DEV void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
        "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
        "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
CK_DEV void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row core groups 1024 bytes apart
// (the layout TMA SWIZZLE_128B writes for 128-byte rows); the tile base must be 1024-aligned.
CK_DEV uint64_t sdesc_k_sw128(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);
    d |= (uint64_t)1 << 16;               // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;     // stride byte offset
    d |= (uint64_t)1 << 46;               // descriptor version (sm_100)
    d |= (uint64_t)2 << 61;               // SWIZZLE_128B
    return d;
}
// Instruction descriptor: bf16 x bf16 -> fp32, both operands K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
    return (1u << 4)                 // D = f32
           | (1u << 7)               // A = bf16
           | (1u << 10)              // B = bf16
           | ((uint32_t)(N >> 3) << 17)
           | ((uint32_t)(M >> 4) << 24);
}

}  // namespace ck
