// gemm_tc.cu -- grouped Q4_K x bf16 GEMM on the 5th-generation tensor core (tcgen05 / TMEM).
//
// Computes, for every token tile of every group (an expert, a shared expert, or the single matrix
// of a prefill GEMM):
//     dual = 0 :  out[o + t, n] = sum_k X[x + t, k] * W_g[n, k]
//     dual = 1 :  out[o + t, n] = silu(sum_k X W0_g) * (sum_k X W1_g) * row_w[o + t]
// with W_g the GGUF Q4_K tensor of group g (flat index, rows may straddle superblocks at 64-weight
// chunk boundaries, as q4k-msl.fk:73-86 reads it).  Output is bf16, accumulation fp32.
//
// A third form, dense = 1, reads a bf16 A operand through TMA instead of dequantizing and writes
// fp32: the router logits, with the fp32 router split into three bf16 terms along K.
//
// One persistent CTA per SM, warp-specialised:
//   warp 0      TMA producer: the token tile (BN x 64 bf16, 128-byte swizzle) per K step
//   warp 1      TMEM allocator and the single MMA-issuing thread (tcgen05.mma kind::f16, M=128)
//   warps 2-9   dequant producers: two threads per weight row of the 128-row tile; each loads the
//               packed superblock fields with 16-byte loads (one stage ahead), unpacks nibbles and
//               6-bit scales in registers and writes bf16 into the swizzled shared-memory A tile
//   warps 10-13 epilogue: tcgen05.ld the fp32 accumulators, SwiGLU + route weight, stores
// Every wait is bounded (about one second); on a timeout the kernel records a code in *err and
// every role leaves its loop, waits for its own copies and MMAs, and frees TMEM.
#include "ck_common.cuh"
#include "ck_launch.h"

#include <mutex>

namespace ck {

namespace gemm {
constexpr int BM = 128;
constexpr int BK = 64;
constexpr int BN = 256;
constexpr int NDQ = 8;   // dequant warps (two threads per weight row)
constexpr int NEPI = 4;  // epilogue warps
constexpr int NTHREADS = (2 + NDQ + NEPI) * 32;
constexpr int A_BYTES = BM * BK * 2;
constexpr int B_BYTES = BN * BK * 2;

template <int DUAL>
struct Cfg {
    static constexpr int NMAT = DUAL ? 2 : 1;
    static constexpr int STAGE_BYTES = NMAT * A_BYTES + B_BYTES;
    static constexpr int STAGES = DUAL ? 3 : 4;
    static constexpr int ACC_COLS = NMAT * BN;
    static constexpr int ACC_BUFS = 512 / ACC_COLS;
    // the dense form splits its K loop over DENSE_ACC accumulators of DENSE_TILE columns (token
    // tiles of at most DENSE_TILE) and sums them in fp32 in the epilogue: each tensor-core
    // accumulation chain is an eighth as long, and so is its rounding error
    static constexpr int DENSE_ACC = 8;
    static constexpr int DENSE_TILE = 64;
    static constexpr int DENSE_B_BYTES = DENSE_TILE * BK * 2;
    static constexpr int BAR_BYTES = 256;
    static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + BAR_BYTES;
};

struct Tile {
    int g, xrow, orow, ntok;
};
CK_DEV Tile load_tile(const int4 *tiles, int i) {
    int4 v = tiles[i];
    return Tile{v.x, v.y, v.z, v.w};
}

// The packed fields one thread needs for one K step of one matrix: the superblock header
// (d, dmin, scales[12]) and the 32 qs bytes of the 64-weight chunk.
struct Packed {
    uint4 hdr, q0, q1;
    int c;
};
CK_DEV void load_packed(Packed &p, const uint8_t *base, uint64_t flat) {
    const uint8_t *blk = base + (flat >> 8) * Q4K_BYTES;
    p.c = (int)((flat >> 6) & 3);
    p.hdr = __ldg(reinterpret_cast<const uint4 *>(blk));
    p.q0 = __ldg(reinterpret_cast<const uint4 *>(blk + 16 + p.c * 32));
    p.q1 = __ldg(reinterpret_cast<const uint4 *>(blk + 32 + p.c * 32));
}

// Two adjacent weights (k, k+1) as bf16x2 from the nibbles of two qs bytes spread to the low byte
// of each 16-bit half (pp = byte_k | byte_k+1 << 16).  OR-ing a nibble q into the mantissa of
// bf16 128.0 (0x4300) gives exactly 128 + q; subtracting 128 is exact; then one bf16x2 FMA
// q * (d*sc) - dmin*m rounds the weight once.
CK_DEV uint32_t deq_pair(uint32_t pp, int hi, __nv_bfloat162 ds2, __nv_bfloat162 ndm2) {
    const uint32_t v = ((hi ? (pp >> 4) : pp) & 0x000F000Fu) | 0x43004300u;
    const __nv_bfloat162 q = __hsub2(*reinterpret_cast<const __nv_bfloat162 *>(&v), __floats2bfloat162_rn(128.f, 128.f));
    const __nv_bfloat162 w = __hfma2(q, ds2, ndm2);
    return *reinterpret_cast<const uint32_t *>(&w);
}

// Dequantize one 32-weight half of the 64-weight chunk into the 128-byte swizzled smem row `r` of
// tile `a`: half 0 = sub-block 2c (low nibbles, k = 0..31), half 1 = sub-block 2c+1 (high
// nibbles, k = 32..63).  16-byte chunk cc of the row holds k = 8cc .. 8cc+7 and sits at position
// cc ^ (r & 7) (the 128-byte swizzle the MMA descriptor names).
CK_DEV void dequant_half(const Packed &p, uint8_t *a, int r, int half) {
    const float d = f16_bits_to_float(p.hdr.x & 0xFFFF), dmin = f16_bits_to_float(p.hdr.x >> 16);
    uint32_t s[3] = {p.hdr.y, p.hdr.z, p.hdr.w};
    int sc, mn;
    q4k_scale_min(s, 2 * p.c + half, sc, mn);
    const float ds = d * (float)sc, dm = dmin * (float)mn;  // both exact in fp32
    const __nv_bfloat162 ds2 = __floats2bfloat162_rn(ds, ds), ndm2 = __floats2bfloat162_rn(-dm, -dm);
    const uint32_t qw[8] = {p.q0.x, p.q0.y, p.q0.z, p.q0.w, p.q1.x, p.q1.y, p.q1.z, p.q1.w};
    uint8_t *row = a + r * 128;
    const int sw = r & 7;
#pragma unroll
    for (int c4 = 0; c4 < 4; ++c4) {
        const uint32_t w0 = qw[2 * c4], w1 = qw[2 * c4 + 1];
        uint4 o;
        o.x = deq_pair(__byte_perm(w0, 0u, 0x4140), half, ds2, ndm2);
        o.y = deq_pair(__byte_perm(w0, 0u, 0x4342), half, ds2, ndm2);
        o.z = deq_pair(__byte_perm(w1, 0u, 0x4140), half, ds2, ndm2);
        o.w = deq_pair(__byte_perm(w1, 0u, 0x4342), half, ds2, ndm2);
        *reinterpret_cast<uint4 *>(row + (((c4 + 4 * half) ^ sw) << 4)) = o;
    }
}

template <int DUAL, int DENSE>
__global__ void __launch_bounds__(NTHREADS, 1) k_gemm_q4k(const __grid_constant__ CUtensorMap tmap_x,
                                                          const __grid_constant__ CUtensorMap tmap_a, GemmParams p) {
    using C = Cfg<DUAL>;
    static_assert(!(DUAL && DENSE), "the dense form has one accumulator");
    constexpr int NBUF = DENSE ? 1 : C::ACC_BUFS;  // accumulator buffers in flight
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::STAGES * C::STAGE_BYTES);
    uint64_t *full_a = bars;
    uint64_t *full_b = bars + C::STAGES;
    uint64_t *empty = bars + 2 * C::STAGES;
    uint64_t *acc_full = bars + 3 * C::STAGES;
    uint64_t *acc_empty = acc_full + C::ACC_BUFS;
    uint64_t *done_bar = acc_empty + C::ACC_BUFS;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done_bar + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntiles = min(*p.ntiles, (int)p.max_tiles);
    const int nrt = (int)((p.N + BM - 1) / BM);
    const int nunits = ntiles * nrt;
    const int nk = (int)(p.K / BK);
    // the x operand's own K steps: the dense form walks x once per bf16 term of the split A
    const int nkx = DENSE && p.kx ? (int)(p.kx / BK) : nk;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(&full_a[s], NDQ * 32);
            mbar_init(&full_b[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < C::ACC_BUFS; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], NEPI * 32);
        }
        mbar_init(done_bar, 1);
        fence_barrier_init();
        prefetch_tmap(&tmap_x);
        if (DENSE) prefetch_tmap(&tmap_a);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            int it = 0;
            for (int u = blockIdx.x; u < nunits; u += gridDim.x) {
                const Tile t = load_tile(p.tiles, u / nrt);
                bool ok = true;
                for (int kb = 0; kb < nk; ++kb, ++it) {
                    const int s = it % C::STAGES;
                    const uint32_t ph = (uint32_t)(it / C::STAGES) & 1u;
                    if (!mbar_wait_bounded(&empty[s], ph ^ 1u, p.err, 1)) { ok = false; break; }
                    uint8_t *b_tile = smem + s * C::STAGE_BYTES + C::NMAT * A_BYTES;
                    mbar_arrive_expect_tx(&full_b[s], DENSE ? C::DENSE_B_BYTES + A_BYTES : B_BYTES);
                    tma_load_2d(b_tile, &tmap_x, &full_b[s], (kb % nkx) * BK, p.xrow_is_orow ? t.orow : t.xrow);
                    if (DENSE) tma_load_2d(smem + s * C::STAGE_BYTES, &tmap_a, &full_b[s], kb * BK, (u % nrt) * BM);
                }
                if (!ok) break;
            }
            // drain: the copies this thread issued must land before the CTA can exit
            for (int d = 0; d < C::STAGES && it - 1 - d >= 0; ++d) {
                const int j = it - 1 - d;
                mbar_wait_bounded(&full_b[j % C::STAGES], (uint32_t)(j / C::STAGES) & 1u, nullptr, 0);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            int it = 0, ut = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < nunits && ok; u += gridDim.x, ++ut) {
                const Tile t = load_tile(p.tiles, u / nrt);
                int nmma = ((t.ntok + 15) / 16) * 16;
                const int nmax = DENSE ? C::DENSE_TILE : BN;
                nmma = nmma < 16 ? 16 : (nmma > nmax ? nmax : nmma);
                const uint32_t idesc = idesc_bf16(BM, nmma);
                const int ab = ut % NBUF;
                const uint32_t aph = (uint32_t)(ut / NBUF) & 1u;
                if (!mbar_wait_bounded(&acc_empty[ab], aph ^ 1u, p.err, 2)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d0 = tmem_base + (uint32_t)(ab * C::ACC_COLS);
                const int chunk = (nk + C::DENSE_ACC - 1) / C::DENSE_ACC;
                for (int kb = 0; kb < nk; ++kb, ++it) {
                    const int s = it % C::STAGES;
                    const uint32_t ph = (uint32_t)(it / C::STAGES) & 1u;
                    if ((!DENSE && !mbar_wait_bounded(&full_a[s], ph, p.err, 3)) ||
                        !mbar_wait_bounded(&full_b[s], ph, p.err, 4)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(smem + s * C::STAGE_BYTES);
                    const uint32_t b0 = smem_u32(smem + s * C::STAGE_BYTES + C::NMAT * A_BYTES);
                    // dense form: K chunk kb / chunk accumulates into its own 128-column accumulator
                    const uint32_t dd = DENSE ? d0 + (uint32_t)((kb / chunk) * C::DENSE_TILE) : d0;
                    const int kfirst = DENSE ? kb % chunk : kb;
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k) {
                        const uint64_t bd = sdesc_k_sw128(b0 + k * 32);
                        const uint32_t acc = (kfirst | k) != 0;
                        umma_bf16(dd, sdesc_k_sw128(a0 + k * 32), bd, idesc, acc);
                        if (DUAL) umma_bf16(d0 + BN, sdesc_k_sw128(a0 + A_BYTES + k * 32), bd, idesc, acc);
                    }
                    umma_commit(&empty[s]);
                }
                if (!ok) break;
                umma_commit(&acc_full[ab]);
            }
            // every MMA this thread issued completes before TMEM is released
            umma_commit(done_bar);
            mbar_wait_bounded(done_bar, 0, nullptr, 0);
        }
    } else if (warp < 2 + NDQ && !DENSE) {  // in the dense form the A operand arrives by TMA
        // ------------------------------------------------------------ dequant producers
        // 256 threads: thread i owns row (i & 127) of the tile; part = i >> 7 selects the matrix
        // (dual: gate or up, both halves of the 64-weight chunk) or the nibble half (single).
        const int di = threadIdx.x - 64;
        const int r = di & (BM - 1);
        const int part = di >> 7;
        int it = 0;
        // software pipeline: the packed fields of step it+1 are in flight while step it is unpacked
        Packed cur, nxt;
        int u = blockIdx.x, kb = 0;
        auto base_of = [&](int uu, uint64_t &rowflat) -> const uint8_t * {
            const Tile t = load_tile(p.tiles, uu / nrt);
            const int n0 = (uu % nrt) * BM;
            const uint32_t row = min((uint32_t)(n0 + r), p.N - 1);
            const bool shared = (uint32_t)t.g >= p.n_routed;
            const uint64_t g = shared ? (uint64_t)(t.g - p.n_routed) : (uint64_t)t.g;
            const uint8_t *b = (DUAL && part) ? (shared ? p.s1 : p.w1) : (shared ? p.s0 : p.w0);
            rowflat = (uint64_t)row * p.K;
            return b + g * p.w_stride;
        };
        const uint8_t *b = nullptr;
        uint64_t rowflat = 0;
        if (u < nunits) {
            b = base_of(u, rowflat);
            load_packed(nxt, b, rowflat);
        }
        while (u < nunits) {
            cur = nxt;
            // advance to the next (unit, k step) and issue its loads
            int nu = u, nkb = kb + 1;
            if (nkb == nk) { nkb = 0; nu = u + gridDim.x; }
            if (nu < nunits) {
                if (nu != u) b = base_of(nu, rowflat);
                load_packed(nxt, b, rowflat + (uint64_t)nkb * BK);
            }
            const int s = it % C::STAGES;
            const uint32_t ph = (uint32_t)(it / C::STAGES) & 1u;
            if (!mbar_wait_bounded(&empty[s], ph ^ 1u, p.err, 5)) break;
            uint8_t *a = smem + s * C::STAGE_BYTES;
            if (DUAL) {
                dequant_half(cur, a + part * A_BYTES, r, 0);
                dequant_half(cur, a + part * A_BYTES, r, 1);
            } else {
                dequant_half(cur, a, r, part);
            }
            fence_proxy_async_smem();
            mbar_arrive(&full_a[s]);
            ++it;
            u = nu;
            kb = nkb;
        }
    } else if (warp >= 2 + NDQ) {
        // ------------------------------------------------------------ epilogue
        const int sp = warp & 3;  // TMEM sub-partition this warp may read
        int ut = 0;
        __nv_bfloat16 *out = reinterpret_cast<__nv_bfloat16 *>(p.out);
        for (int u = blockIdx.x; u < nunits; u += gridDim.x, ++ut) {
            const Tile t = load_tile(p.tiles, u / nrt);
            const int n0 = (u % nrt) * BM;
            const int ab = ut % NBUF;
            const uint32_t aph = (uint32_t)(ut / NBUF) & 1u;
            if (!mbar_wait_bounded(&acc_full[ab], aph, p.err, 6)) break;
            tc_fence_after();
            const uint32_t row = (uint32_t)(n0 + 32 * sp + lane);
            const uint32_t tbase = tmem_base + ((uint32_t)(32 * sp) << 16) + (uint32_t)(ab * C::ACC_COLS);
            for (int cb = 0; cb * 32 < t.ntok; ++cb) {
                uint32_t g[32], v[32];
                tmem_ld32(tbase + cb * 32, g);
                if (DUAL) tmem_ld32(tbase + BN + cb * 32, v);
                tmem_ld_wait();
                if (DENSE) {
                    // sum the K-chunk accumulators in fp32, in chunk order
#pragma unroll 1
                    for (int a = 1; a < C::DENSE_ACC; ++a) {
                        tmem_ld32(tbase + a * C::DENSE_TILE + cb * 32, v);
                        tmem_ld_wait();
#pragma unroll
                        for (int j = 0; j < 32; ++j) g[j] = __float_as_uint(__uint_as_float(g[j]) + __uint_as_float(v[j]));
                    }
                }
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int tok = cb * 32 + j;
                    if (tok < t.ntok && row < p.N) {
                        float val = __uint_as_float(g[j]);
                        if (DUAL) {
                            const float up = __uint_as_float(v[j]);
                            const float rw = p.row_w ? p.row_w[t.orow + tok] : 1.0f;
                            val = (val / (1.0f + __expf(-val))) * up * rw;
                        }
                        if (DENSE)
                            p.out_f32[(uint64_t)(t.orow + tok) * p.N + row] = val;
                        else
                            out[(uint64_t)(t.orow + tok) * p.N + row] = __float2bfloat16_rn(val);
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&acc_empty[ab]);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, 512);
    }
}

// ----------------------------------------------------------------------------- host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(f);
    });
    return fn;
}

// bf16 [rows, K] row-major, box = box_rows x 64 columns, 128-byte swizzle.
static int make_map(CUtensorMap *m, const void *x, uint32_t rows, uint32_t K, uint32_t box_rows) {
    EncodeTiledFn enc = get_encode();
    if (!enc) return CK_ERR_NODEV;
    cuuint64_t dims[2] = {K, rows};
    cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    cuuint32_t box[2] = {BK, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(x), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : CK_ERR_ARG;
}

template <int DUAL, int DENSE>
static int launch_t(const GemmParams &p, cudaStream_t s) {
    using C = Cfg<DUAL>;
    static bool attr = false;
    if (!attr) {
        cudaError_t e =
            cudaFuncSetAttribute(k_gemm_q4k<DUAL, DENSE>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        if (e != cudaSuccess) return (int)e;
        attr = true;
    }
    CUtensorMap mx, ma;
    int rc = make_map(&mx, p.x, p.x_rows, DENSE && p.kx ? p.kx : p.K, DENSE ? C::DENSE_TILE : BN);
    if (rc) return rc;
    if (DENSE) {
        rc = make_map(&ma, p.a_dense, p.N, p.K, BM);
        if (rc) return rc;
    } else {
        ma = mx;
    }
    int dev = 0, nsm = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    const long long units = (long long)p.max_tiles * ((p.N + BM - 1) / BM);
    const int grid = (int)(units < nsm ? units : nsm);
    if (grid <= 0) return 0;
    k_gemm_q4k<DUAL, DENSE><<<grid, NTHREADS, C::SMEM, s>>>(mx, ma, p);
    return (int)cudaGetLastError();
}
}  // namespace gemm

int launch_gemm_q4k(const GemmParams &p, cudaStream_t s) {
    if (!p.w0 || !p.x || !p.out || !p.tiles || !p.ntiles || !p.err) return CK_ERR_ARG;
    if (p.K % gemm::BK != 0 || p.N == 0 || p.K == 0 || ((uint64_t)p.N * p.K) % 256 != 0) return CK_ERR_SHAPE;
    if (p.dual && !p.w1) return CK_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(p.x) & 15) || (reinterpret_cast<uintptr_t>(p.w0) & 15)) return CK_ERR_ARG;
    return p.dual ? gemm::launch_t<1, 0>(p, s) : gemm::launch_t<0, 0>(p, s);
}

int launch_gemm_dense(const GemmParams &p, cudaStream_t s) {
    if (!p.a_dense || !p.x || !p.out_f32 || !p.tiles || !p.ntiles || !p.err) return CK_ERR_ARG;
    if (p.K % gemm::BK != 0 || p.K == 0 || p.N == 0 || (p.kx && (p.kx % gemm::BK || p.K % p.kx))) return CK_ERR_SHAPE;
    if ((reinterpret_cast<uintptr_t>(p.x) & 15) || (reinterpret_cast<uintptr_t>(p.a_dense) & 15)) return CK_ERR_ARG;
    return gemm::launch_t<0, 1>(p, s);
}

}  // namespace ck
