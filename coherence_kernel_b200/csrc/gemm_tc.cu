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
// One persistent CTA per SM, warp-specialised.  The dequantized weights never touch shared
// memory: the dequant threads write them straight into tensor memory (tcgen05.st) and the MMA
// reads its A operand from there, so shared-memory bandwidth goes to the token tiles and the packed
// weights only.  Tensor memory (512 columns) holds the fp32 accumulators (token tiles of at most
// BN = 192 columns; gate and up in the dual form, two buffers in the single form) and the A
// stages (32 columns per matrix per 64-wide K step).  Shared-memory rings:
//   P ring  packed Q4_K bytes of the 128-row weight tile per K step -- each row's superblock
//           header (16 B) and the 32 qs bytes of its 64-weight chunk -- brought in by TMA (3D maps
//           over [expert, row, byte]) several steps ahead, when every row starts on a superblock
//           (K % 256 == 0); otherwise the dequant threads load the bytes themselves.
//   B ring  the bf16 token tile (up to 192 x 64, 128-byte swizzle) by TMA in boxes of 64 tokens,
//           only as many boxes as the tile has tokens (the MMA's B operand)
// Warps:
//   0       TMA producer of the B ring (and of the A operand in the dense form)
//   1       TMEM allocator and the single MMA-issuing thread (tcgen05.mma kind::f16, M = 128)
//   2-9     dequant: warps 2-5 and 6-9 take alternate K steps; thread `lane` of warp w owns row
//           32 (w % 4) + lane (the TMEM lanes its warp may write); prmt + magic-exponent nibble
//           decode, one exact bf16x2 subtract and one bf16x2 FMA per weight pair, 32 columns per
//           matrix stored with tcgen05.st
//   10-13   epilogue: tcgen05.ld of the fp32 accumulators, SwiGLU x route weight, stores
//   14      TMA producer of the P ring
// Every wait is bounded (about one second); on a timeout the kernel records a code in *err and
// every role leaves its loop, waits for its own copies and MMAs, and frees TMEM.
#include "ck_common.cuh"
#include "ck_launch.h"

#include <cstring>
#include <mutex>

namespace ck {

namespace gemm {
constexpr int BM = 128;
constexpr int BK = 64;
constexpr int BN = (int)GEMM_TILE_TOKENS;  // largest token tile (accumulator columns)
constexpr int B_BOX = 64;                   // token rows per TMA box of the B ring
constexpr int NDQ = 8;   // dequant warps (two groups of one thread per weight row)
constexpr int NEPI = 4;  // epilogue warps
constexpr int NTHREADS = (2 + NDQ + NEPI + 1) * 32;
constexpr int A_BYTES = BM * BK * 2;
constexpr int B_BYTES = BN * BK * 2;
constexpr int P_HDR = BM * 16;  // superblock headers of the tile's rows
constexpr int P_QS = BM * 32;   // the qs bytes of the K step's chunk
constexpr int W_EPI0 = 2 + NDQ, W_PTMA = 2 + NDQ + NEPI;
// shared-memory ring depths (B: token tiles, P: packed weights) for the dual (gate/up) and single
// forms; the defaults fill the shared memory of one CTA per SM
#ifndef CK_DUAL_BST
#define CK_DUAL_BST 5
#endif
#ifndef CK_DUAL_PST
#define CK_DUAL_PST 6
#endif
#ifndef CK_SINGLE_BST
#define CK_SINGLE_BST 6
#endif
#ifndef CK_SINGLE_PST
#define CK_SINGLE_PST 8
#endif

template <int DUAL, int DENSE, int PT>
struct Cfg {
    static constexpr int NMAT = DUAL ? 2 : 1;
    // the dense form splits its K loop over DENSE_ACC accumulators of DENSE_TILE columns (token
    // tiles of at most DENSE_TILE) and sums them in fp32 in the epilogue: each tensor-core
    // accumulation chain is an eighth as long, and so is its rounding error
    static constexpr int DENSE_ACC = 8;
    static constexpr int DENSE_TILE = 64;
    static constexpr int DENSE_B_BYTES = DENSE_TILE * BK * 2;
    // tensor memory: accumulators first, then the A stages
    static constexpr int ACC_COLS = DENSE ? 512 : NMAT * BN;
    static constexpr int NBUF = (DENSE || DUAL) ? 1 : 2;
    static constexpr int A_TCOLS = 32 * NMAT;  // one 64-wide K step of every matrix, bf16x2 per column
    static constexpr int A_TOFF = NBUF * ACC_COLS;
    static constexpr int A_ST = DENSE ? 0 : (512 - A_TOFF) / A_TCOLS;
    static_assert(DENSE || (A_ST >= 2 && A_ST <= 4), "tensor-memory A stages");
    static constexpr int B_ST = DENSE ? 6 : (DUAL ? CK_DUAL_BST : CK_SINGLE_BST);
    static constexpr int B_STAGE = DENSE ? A_BYTES + DENSE_B_BYTES : B_BYTES;
    static constexpr int P_ST = (DENSE || !PT) ? 0 : (DUAL ? CK_DUAL_PST : CK_SINGLE_PST);
    static constexpr int P_STAGE = NMAT * (P_HDR + P_QS);
    // per epilogue warp, one 32-token x 32-row bf16 chunk of the output, token-major
    static constexpr int EPI_STAGE = 32 * 32 * 2;
    static constexpr int B_OFF = 0;
    static constexpr int P_OFF = B_OFF + B_ST * B_STAGE;
    static constexpr int EPI_OFF = P_OFF + P_ST * P_STAGE;
    static constexpr int BAR_OFF = EPI_OFF + (DENSE ? 0 : NEPI * EPI_STAGE);
    static constexpr int SMEM = BAR_OFF + 512 + 1024;
    static_assert(B_ST <= 8 && P_ST <= 8, "barrier arrays");
    static_assert(SMEM <= 227 * 1024, "shared memory");
};

struct Tile {
    int g, xrow, orow, ntok;
};
// one lane of a converged warp issues the MMAs: a tcgen05.mma from a lone diverged thread issues
// several times slower
CK_DEV bool elect_lane() {
    uint32_t pred = 0;
    asm volatile("{\n .reg .b32 %%rx;\n .reg .pred %%px;\n elect.sync %%rx|%%px, %1;\n selp.u32 %0, 1, 0, %%px;\n}"
                 : "=r"(pred)
                 : "r"(0xffffffffu));
    return pred != 0;
}
// A tile longer than the largest token tile is cut to BN tokens by every role alike (the MMA
// thread also records the error); the tile builders never make one.
CK_DEV Tile load_tile(const int4 *tiles, int i) {
    int4 v = tiles[i];
    return Tile{v.x, v.y, v.z, min(v.w, BN)};
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

// Dequantize one 32-weight half of the 64-weight chunk into 16 bf16x2 words in K order: half 0 =
// sub-block 2c (low nibbles, k = 0..31), half 1 = sub-block 2c+1 (high nibbles, k = 32..63).
CK_DEV void dequant_words(const Packed &p, int half, uint32_t *w) {
    const float d = f16_bits_to_float(p.hdr.x & 0xFFFF), dmin = f16_bits_to_float(p.hdr.x >> 16);
    int sc, mn;
    q4k_scale_min(p.hdr.y, p.hdr.z, p.hdr.w, 2 * p.c + half, sc, mn);
    const float ds = d * (float)sc, dm = dmin * (float)mn;  // both exact in fp32
    const __nv_bfloat162 ds2 = __floats2bfloat162_rn(ds, ds), ndm2 = __floats2bfloat162_rn(-dm, -dm);
    const uint32_t qw[8] = {p.q0.x, p.q0.y, p.q0.z, p.q0.w, p.q1.x, p.q1.y, p.q1.z, p.q1.w};
#pragma unroll
    for (int c4 = 0; c4 < 4; ++c4) {
        const uint32_t w0 = qw[2 * c4], w1 = qw[2 * c4 + 1];
        w[4 * c4 + 0] = deq_pair(__byte_perm(w0, 0u, 0x4140), half, ds2, ndm2);
        w[4 * c4 + 1] = deq_pair(__byte_perm(w0, 0u, 0x4342), half, ds2, ndm2);
        w[4 * c4 + 2] = deq_pair(__byte_perm(w1, 0u, 0x4140), half, ds2, ndm2);
        w[4 * c4 + 3] = deq_pair(__byte_perm(w1, 0u, 0x4342), half, ds2, ndm2);
    }
}

CK_DEV void tma_load_3d(void *smem_dst, const CUtensorMap *map, uint64_t *bar, int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
            smem_u32(smem_dst)),
        "l"((uint64_t)map), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
        : "memory");
}

// the eight packed-weight maps: header and qs boxes of w0, w1 (routed) and s0, s1 (shared)
struct PMaps {
    CUtensorMap hdr[4];
    CUtensorMap qs[4];
};

template <int DUAL, int DENSE, int PT>
__global__ void __launch_bounds__(NTHREADS, 1)
    k_gemm_q4k(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_a,
               const __grid_constant__ PMaps pm, GemmParams p) {
    using C = Cfg<DUAL, DENSE, PT>;
    static_assert(!(DUAL && DENSE), "the dense form has one accumulator");
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::BAR_OFF);
    uint64_t *p_full = bars, *p_empty = bars + 8;
    uint64_t *a_full = bars + 16, *a_empty = bars + 20;
    uint64_t *b_full = bars + 24, *b_empty = bars + 32;
    uint64_t *acc_full = bars + 40, *acc_empty = bars + 42;
    uint64_t *done_bar = bars + 44;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 45);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntiles = min(*p.ntiles, (int)p.max_tiles);
    const int nrt = (int)((p.N + BM - 1) / BM);
    const int nk = (int)(p.K / BK);
    // The dense form may give each of its K-chunk accumulators a unit of its own (p.ksplit > 1):
    // unit u is then (tile, row block) u / ks and K chunk u % ks, and writes that chunk's sums to
    // plane u % ks of the output for the caller to add in chunk order.
    const int kchunk = (nk + C::DENSE_ACC - 1) / C::DENSE_ACC;
    const int ks = DENSE && p.ksplit > 1 ? (nk + kchunk - 1) / kchunk : 1;
    const int nunits = ntiles * nrt * ks;
    auto krange = [&](int u, int &kb0, int &kb1) {
        kb0 = ks > 1 ? (u % ks) * kchunk : 0;
        kb1 = ks > 1 ? min(nk, kb0 + kchunk) : nk;
    };
    // the x operand's own K steps: the dense form walks x once per bf16 term of the split A
    const int nkx = DENSE && p.kx ? (int)(p.kx / BK) : nk;

    if (threadIdx.x == 0) {
        for (int s = 0; s < 8; ++s) {
            mbar_init(&p_full[s], 1);
            mbar_init(&p_empty[s], DUAL ? NDQ * 32 : NDQ * 16);  // dequant threads per stage
            mbar_init(&b_full[s], 1);
            mbar_init(&b_empty[s], 1);
        }
        for (int s = 0; s < 4; ++s) {
            mbar_init(&a_full[s], DUAL ? NDQ * 32 : NDQ * 16);
            mbar_init(&a_empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
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
        // ------------------------------------------------------------ B ring producer (TMA)
        if (lane == 0) {
            int it = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < nunits && ok; u += gridDim.x) {
                const Tile t = load_tile(p.tiles, u / ks / nrt);
                int kb0, kb1;
                krange(u, kb0, kb1);
                for (int kb = kb0; kb < kb1; ++kb, ++it) {
                    const int s = it % C::B_ST;
                    const uint32_t ph = (uint32_t)(it / C::B_ST) & 1u;
                    if (!mbar_wait_bounded(&b_empty[s], ph ^ 1u, p.err, 1)) { ok = false; break; }
                    uint8_t *st = smem + C::B_OFF + s * C::B_STAGE;
                    if (DENSE) {
                        mbar_arrive_expect_tx(&b_full[s], C::B_STAGE);
                        tma_load_2d(st, &tmap_a, &b_full[s], kb * BK, (u / ks % nrt) * BM);
                        tma_load_2d(st + A_BYTES, &tmap_x, &b_full[s], (kb % nkx) * BK, t.xrow);
                    } else {
                        // only the boxes that hold the tile's tokens (the MMA reads round16(ntok))
                        const int nbox = max(1, (min(t.ntok, BN) + B_BOX - 1) / B_BOX);
                        const int row0 = p.xrow_is_orow ? t.orow : t.xrow;
                        mbar_arrive_expect_tx(&b_full[s], (uint32_t)(nbox * B_BOX * BK * 2));
                        for (int i = 0; i < nbox; ++i)
                            tma_load_2d(st + i * B_BOX * BK * 2, &tmap_x, &b_full[s], kb * BK, row0 + i * B_BOX);
                    }
                }
            }
            // drain: the copies this thread issued must land before the CTA can exit
            for (int d = 0; d < C::B_ST && it - 1 - d >= 0; ++d) {
                const int j = it - 1 - d;
                mbar_wait_bounded(&b_full[j % C::B_ST], (uint32_t)(j / C::B_ST) & 1u, nullptr, 0);
            }
        }
    } else if (warp == W_PTMA) {
        // ------------------------------------------------------------ P ring producer (TMA)
        if constexpr (PT && !DENSE) if (lane == 0) {
            int it = 0;
            bool ok = true;
            const uint32_t row_bytes = p.K / 256 * Q4K_BYTES;
            (void)row_bytes;
            for (int u = blockIdx.x; u < nunits && ok; u += gridDim.x) {
                const Tile t = load_tile(p.tiles, u / nrt);
                const int n0 = (u % nrt) * BM;
                const bool shared = (uint32_t)t.g >= p.n_routed;
                const int gg = shared ? t.g - (int)p.n_routed : t.g;
                for (int kb = 0; kb < nk; ++kb, ++it) {
                    const int s = it % C::P_ST;
                    const uint32_t ph = (uint32_t)(it / C::P_ST) & 1u;
                    if (!mbar_wait_bounded(&p_empty[s], ph ^ 1u, p.err, 7)) { ok = false; break; }
                    uint8_t *st = smem + C::P_OFF + s * C::P_STAGE;
                    mbar_arrive_expect_tx(&p_full[s], C::P_STAGE);
                    const int sb = kb >> 2, c = kb & 3;
#pragma unroll
                    for (int m = 0; m < C::NMAT; ++m) {
                        const int mi = (shared ? 2 : 0) + m;
                        tma_load_3d(st + m * (P_HDR + P_QS), &pm.hdr[mi], &p_full[s], sb * Q4K_BYTES, n0, gg);
                        tma_load_3d(st + m * (P_HDR + P_QS) + P_HDR, &pm.qs[mi], &p_full[s], sb * Q4K_BYTES + 16 + 32 * c,
                                    n0, gg);
                    }
                }
            }
            for (int d = 0; d < C::P_ST && it - 1 - d >= 0; ++d) {
                const int j = it - 1 - d;
                mbar_wait_bounded(&p_full[j % C::P_ST], (uint32_t)(j / C::P_ST) & 1u, nullptr, 0);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        // The whole warp runs the loop: lane 0 takes the (bounded) barrier waits and broadcasts
        // their outcome, and one elected lane of the converged warp issues the MMAs and commits.
        {
            // running ring positions and phases (no division in the loop); the B operand's
            // descriptor is the stage's base descriptor plus 2 per 16-wide K slice (32 bytes)
            int sb = 0, sa = 0, ut = 0;
            uint32_t phb = 0, pha = 0;
            bool ok = true;
            const int chunk = kchunk;
            const uint64_t bdesc0 = sdesc_k_sw128(smem_u32(smem + C::B_OFF) + (DENSE ? A_BYTES : 0));
            const uint64_t adesc0 = sdesc_k_sw128(smem_u32(smem + C::B_OFF));  // dense form's A
            const uint32_t atm0 = tmem_base + (uint32_t)C::A_TOFF;              // first A stage (TMEM)
            for (int u = blockIdx.x; u < nunits && ok; u += gridDim.x, ++ut) {
                const Tile t = load_tile(p.tiles, u / ks / nrt);
                if (lane == 0 && p.tiles[u / ks / nrt].w > BN) atomicCAS(p.err, 0, 9);
                int kb0, kb1;
                krange(u, kb0, kb1);
                int nmma = ((t.ntok + 15) / 16) * 16;
                const int nmax = DENSE ? C::DENSE_TILE : BN;
                nmma = nmma < 16 ? 16 : (nmma > nmax ? nmax : nmma);
                const uint32_t idesc = idesc_bf16(BM, nmma);
                const int ab = ut % C::NBUF;
                const uint32_t aph = (uint32_t)(ut / C::NBUF) & 1u;
                int w_ok = 1;
                if (lane == 0) w_ok = mbar_wait_bounded(&acc_empty[ab], aph ^ 1u, p.err, 2);
                if (!__shfl_sync(0xffffffffu, w_ok, 0)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d0 = tmem_base + (uint32_t)(ab * C::ACC_COLS);
                for (int kb = kb0; kb < kb1; ++kb) {
                    int k_ok = 1;
                    if (lane == 0)
                        k_ok = (DENSE || mbar_wait_bounded(&a_full[sa], pha, p.err, 3)) &&
                               mbar_wait_bounded(&b_full[sb], phb, p.err, 4);
                    if (!__shfl_sync(0xffffffffu, k_ok, 0)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t bd = bdesc0 + (uint64_t)(sb * (C::B_STAGE >> 4));
                    if (elect_lane()) {
                        if constexpr (DENSE) {
                            // K chunk kb / chunk accumulates into its own accumulator
                            const uint32_t dd = d0 + (uint32_t)((kb / chunk) * C::DENSE_TILE);
                            const int kfirst = kb % chunk;
                            const uint64_t ad = adesc0 + (uint64_t)(sb * (C::B_STAGE >> 4));
#pragma unroll
                            for (int k = 0; k < BK / 16; ++k)
                                umma_bf16(dd, ad + 2 * k, bd + 2 * k, idesc, (kfirst | k) != 0);
                        } else {
                            const uint32_t at = atm0 + (uint32_t)(sa * C::A_TCOLS);
#pragma unroll
                            for (int k = 0; k < BK / 16; ++k) {
                                const uint32_t acc = (kb | k) != 0;
                                umma_bf16_ts(d0, at + 8 * k, bd + 2 * k, idesc, acc);
                                if (DUAL) umma_bf16_ts(d0 + BN, at + 32 + 8 * k, bd + 2 * k, idesc, acc);
                            }
                            umma_commit(&a_empty[sa]);
                        }
                        umma_commit(&b_empty[sb]);
                    }
                    __syncwarp();
                    if constexpr (!DENSE) {
                        if (++sa == C::A_ST) { sa = 0; pha ^= 1u; }
                    }
                    if (++sb == C::B_ST) { sb = 0; phb ^= 1u; }
                }
                if (!ok) break;
                if (elect_lane()) umma_commit(&acc_full[ab]);
                __syncwarp();
            }
            // every MMA this warp issued completes before TMEM is released
            if (elect_lane()) umma_commit(done_bar);
            __syncwarp();
            if (lane == 0) mbar_wait_bounded(done_bar, 0, nullptr, 0);
            __syncwarp();
        }
    } else if (warp < W_EPI0 && !DENSE) {
        // ------------------------------------------------------------ dequant producers
        // Warps 2-5 form group 0 and warps 6-9 group 1.  Dual form: group g converts matrix g
        // (gate or up) of every K step, so a stage is ready one half-item after its slot frees --
        // the dual form has only two A stages.  Single form: the groups take alternate K steps
        // (items it with it % 2 == group) over its four stages, spreading each thread's waits and
        // fences over the whole 64-weight chunk.  A warp may write only the 32 TMEM lanes of its
        // sub-partition (warp % 4): thread `lane` owns weight row 32 (warp % 4) + lane and stores
        // its 64-weight chunk of matrix m as 32 bf16x2 columns at A_TOFF + stage * A_TCOLS + 32 m.
        if constexpr (!DENSE) {
            const int sub = warp & 3;
            const int r = 32 * sub + lane;
            const int grp = (warp - 2) >> 2;
            constexpr int ISTEP = DUAL ? 1 : 2;  // items between two of this thread's items
            const int m = DUAL ? grp : 0;         // the matrix this thread converts
            const uint32_t trow = tmem_base + ((uint32_t)(32 * sub) << 16) + (uint32_t)C::A_TOFF;
            auto convert_store = [&](const Packed &pk, int sa, int m) {
                uint32_t w[32];
                dequant_words(pk, 0, w);
                dequant_words(pk, 1, w + 16);
                tmem_st32(trow + (uint32_t)(sa * C::A_TCOLS + 32 * m), w);
            };
            if constexpr (PT) {
                int it = 0;
                bool ok = true;
                for (int u = blockIdx.x; u < nunits && ok; u += gridDim.x) {
                    for (int kb = 0; kb < nk; ++kb, ++it) {
                        if (!DUAL && (it & 1) != grp) continue;
                        const int sp = it % C::P_ST, sa = it % C::A_ST;
                        const uint32_t php = (uint32_t)(it / C::P_ST) & 1u, pha = (uint32_t)(it / C::A_ST) & 1u;
                        if (!mbar_wait_bounded(&p_full[sp], php, p.err, 8) ||
                            !mbar_wait_bounded(&a_empty[sa], pha ^ 1u, p.err, 5)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();  // after the MMAs that read this A stage
                        const uint8_t *pm_ = smem + C::P_OFF + sp * C::P_STAGE + m * (P_HDR + P_QS);
                        Packed pk;
                        pk.hdr = *reinterpret_cast<const uint4 *>(pm_ + r * 16);
                        pk.q0 = *reinterpret_cast<const uint4 *>(pm_ + P_HDR + r * 32);
                        pk.q1 = *reinterpret_cast<const uint4 *>(pm_ + P_HDR + r * 32 + 16);
                        pk.c = kb & 3;
                        convert_store(pk, sa, m);
                        tmem_st_wait();
                        // The proxy fence orders this thread's generic reads of the P stage before
                        // the TMA that refills it: without it the TMA write (async proxy) may land
                        // before the reads are done, even after the mbarrier release.
                        fence_proxy_async_smem();
                        tc_fence_before();
                        mbar_arrive(&p_empty[sp]);
                        mbar_arrive(&a_full[sa]);
                    }
                }
            } else {
                // rows that straddle superblocks: each thread loads the packed fields of its next
                // own item (two items ahead) while it converts the current one
                auto advance = [&](int &uu, int &kk) {
                    if (++kk == nk) {
                        kk = 0;
                        uu += gridDim.x;
                    }
                };
                auto load_item = [&](int uu, int kk, Packed &pk) {
                    const Tile t = load_tile(p.tiles, uu / nrt);
                    const int n0 = (uu % nrt) * BM;
                    const uint32_t row = min((uint32_t)(n0 + r), p.N - 1);
                    const bool shared = (uint32_t)t.g >= p.n_routed;
                    const uint64_t g = shared ? (uint64_t)(t.g - p.n_routed) : (uint64_t)t.g;
                    const uint8_t *b = m ? (shared ? p.s1 : p.w1) : (shared ? p.s0 : p.w0);
                    load_packed(pk, b + g * p.w_stride, (uint64_t)row * p.K + (uint64_t)kk * BK);
                };
                Packed cur, nxt;
                int u = blockIdx.x, kb = 0, it = DUAL ? 0 : grp;
                if (it) advance(u, kb);
                if (u < nunits) load_item(u, kb, nxt);
                while (u < nunits) {
                    cur = nxt;
                    int nu = u, nkb = kb;
                    for (int i = 0; i < ISTEP; ++i) advance(nu, nkb);
                    if (nu < nunits) load_item(nu, nkb, nxt);
                    const int sa = it % C::A_ST;
                    const uint32_t pha = (uint32_t)(it / C::A_ST) & 1u;
                    if (!mbar_wait_bounded(&a_empty[sa], pha ^ 1u, p.err, 5)) break;
                    tc_fence_after();
                    convert_store(cur, sa, m);
                    tmem_st_wait();
                    tc_fence_before();
                    mbar_arrive(&a_full[sa]);
                    it += ISTEP;
                    u = nu;
                    kb = nkb;
                }
            }
        }
    } else if (warp >= W_EPI0 && warp < W_PTMA) {
        // ------------------------------------------------------------ epilogue
        const int sp = warp & 3;  // TMEM sub-partition this warp may read
        int ut = 0;
        __nv_bfloat16 *out = reinterpret_cast<__nv_bfloat16 *>(p.out);
        uint8_t *epi_stage = smem + C::EPI_OFF + (warp - W_EPI0) * C::EPI_STAGE;
        const bool vec_out = !DENSE && p.N % 8 == 0 && (reinterpret_cast<uintptr_t>(p.out) & 15) == 0;
        // the bf16 row of output row o: out + o N, or the address row_dst[o] holds
        auto out_row = [&](uint32_t o) -> __nv_bfloat16 * {
            return p.row_dst ? reinterpret_cast<__nv_bfloat16 *>(p.row_dst[o]) : out + (uint64_t)o * p.N;
        };
        // lane j holds the route weight of token cb*32 + j of the current chunk (shuffled out
        // below); the next chunk's weight is loaded one chunk ahead, the first before the wait
        auto route_w = [&](const Tile &t, int cb) -> float {
            return (DUAL && p.row_w && cb * 32 + lane < t.ntok) ? p.row_w[t.orow + cb * 32 + lane] : 1.0f;
        };
        for (int u = blockIdx.x; u < nunits; u += gridDim.x, ++ut) {
            const Tile t = load_tile(p.tiles, u / ks / nrt);
            const int n0 = (u / ks % nrt) * BM;
            const int kc = u % ks;  // the dense form's K chunk when split over units
            const int ab = ut % C::NBUF;
            const uint32_t aph = (uint32_t)(ut / C::NBUF) & 1u;
            float rw_lane = route_w(t, 0);
            if (!mbar_wait_bounded(&acc_full[ab], aph, p.err, 6)) break;
            tc_fence_after();
            const uint32_t row = (uint32_t)(n0 + 32 * sp + lane);
            // this warp's 32 rows are all inside N and every 8-row group starts 16-byte aligned
            const bool vec_rows = vec_out && (uint32_t)(n0 + 32 * sp + 32) <= p.N;
            const uint32_t tbase = tmem_base + ((uint32_t)(32 * sp) << 16) + (uint32_t)(ab * C::ACC_COLS);
            for (int cb = 0; cb * 32 < t.ntok; ++cb) {
                uint32_t g[32], v[32];
                tmem_ld32(tbase + cb * 32, g);
                if (DUAL) tmem_ld32(tbase + BN + cb * 32, v);
                const float rw_next = route_w(t, cb + 1);
                tmem_ld_wait();
                if (DENSE && ks > 1 && kc > 0) {
                    // a split unit holds one K chunk, in accumulator kc
                    tmem_ld32(tbase + kc * C::DENSE_TILE + cb * 32, g);
                    tmem_ld_wait();
                } else if (DENSE && ks == 1) {
                    // sum the K-chunk accumulators in fp32, in chunk order; with fewer than
                    // DENSE_ACC K steps per chunk only the first ceil(nk / chunk) were written
                    const int nacc = (nk + kchunk - 1) / kchunk;
#pragma unroll 1
                    for (int a = 1; a < nacc; ++a) {
                        tmem_ld32(tbase + a * C::DENSE_TILE + cb * 32, v);
                        tmem_ld_wait();
#pragma unroll
                        for (int j = 0; j < 32; ++j) g[j] = __float_as_uint(__uint_as_float(g[j]) + __uint_as_float(v[j]));
                    }
                }
                if (!DENSE && vec_rows) {
                    // the chunk goes through shared memory, token-major (64 bytes per token), and
                    // leaves as 16-byte stores: lane l writes rows 8(l%4).. of token 8q + l/4
                    __nv_bfloat16 *st = reinterpret_cast<__nv_bfloat16 *>(epi_stage);
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        float val = __uint_as_float(g[j]);
                        if (DUAL) {
                            // silu(g) = g / (1 + e^-g); where e^-g overflows the quotient is
                            // the limit 0, which __fdividef returns for divisors past 2^126
                            const float rw = __shfl_sync(0xffffffffu, rw_lane, j);
                            val = __fdividef(val, 1.0f + __expf(-val)) * __uint_as_float(v[j]) * rw;
                        }
                        st[j * 32 + lane] = __float2bfloat16_rn(val);
                    }
                    __syncwarp();
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const int tl = q * 8 + (lane >> 2), seg = lane & 3;
                        const uint4 o = *reinterpret_cast<const uint4 *>(epi_stage + q * 512 + lane * 16);
                        if (cb * 32 + tl < t.ntok)
                            *reinterpret_cast<uint4 *>(out_row((uint32_t)(t.orow + cb * 32 + tl)) + n0 + 32 * sp + 8 * seg) = o;
                    }
                    __syncwarp();
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const int tok = cb * 32 + j;
                        const float rw = __shfl_sync(0xffffffffu, rw_lane, j);
                        if (tok < t.ntok && row < p.N) {
                            float val = __uint_as_float(g[j]);
                            if (DUAL) {
                                const float up = __uint_as_float(v[j]);
                                val = __fdividef(val, 1.0f + __expf(-val)) * up * rw;
                            }
                            if (DENSE)
                                (kc == 0 ? p.out_f32 : p.out_planes + (uint64_t)(kc - 1) * p.out_rows * p.N)
                                    [(uint64_t)(t.orow + tok) * p.N + row] = val;
                            else
                                out_row((uint32_t)(t.orow + tok))[row] = __float2bfloat16_rn(val);
                        }
                    }
                }
                rw_lane = rw_next;
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

// packed Q4_K weights of `count` experts viewed as bytes [count, N, K/256*144]; box = box_bytes x
// 128 rows x 1 expert, no swizzle (rows land 16 or 32 bytes apart in shared memory).
static int make_packed_map(CUtensorMap *m, const void *base, uint32_t count, uint32_t N, uint32_t K,
                           uint32_t box_bytes) {
    EncodeTiledFn enc = get_encode();
    if (!enc) return CK_ERR_NODEV;
    const cuuint64_t row_bytes = (cuuint64_t)K / 256 * Q4K_BYTES;
    cuuint64_t dims[3] = {row_bytes, N, count ? count : 1};
    cuuint64_t strides[2] = {row_bytes, row_bytes * N};
    cuuint32_t box[3] = {box_bytes, BM, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : CK_ERR_ARG;
}

template <int DUAL, int DENSE, int PT>
static int launch_t(const GemmParams &p, cudaStream_t s) {
    using C = Cfg<DUAL, DENSE, PT>;
    static unsigned long long attr = 0;
    if (attr_pending(attr)) {
        cudaError_t e =
            cudaFuncSetAttribute(k_gemm_q4k<DUAL, DENSE, PT>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        if (e != cudaSuccess) return (int)e;
        attr_mark(attr);
    }
    CUtensorMap mx, ma;
    int rc = make_map(&mx, p.x, p.x_rows, DENSE && p.kx ? p.kx : p.K, DENSE ? C::DENSE_TILE : B_BOX);
    if (rc) return rc;
    if (DENSE) {
        rc = make_map(&ma, p.a_dense, p.N, p.K, BM);
        if (rc) return rc;
    } else {
        ma = mx;
    }
    PMaps pm;
    memset(&pm, 0, sizeof(pm));
    if (PT) {
        const uint8_t *bases[4] = {p.w0, DUAL ? p.w1 : p.w0, p.s0 ? p.s0 : p.w0,
                                   DUAL ? (p.s1 ? p.s1 : p.w1) : (p.s0 ? p.s0 : p.w0)};
        const uint32_t counts[4] = {p.n_routed, p.n_routed, p.s0 ? p.n_shared : p.n_routed,
                                    p.s0 ? p.n_shared : p.n_routed};
        for (int i = 0; i < 4; ++i) {
            rc = make_packed_map(&pm.hdr[i], bases[i], counts[i], p.N, p.K, 16);
            if (!rc) rc = make_packed_map(&pm.qs[i], bases[i], counts[i], p.N, p.K, 32);
            if (rc) return rc;
        }
    }
    int dev = 0, nsm = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    long long units = (long long)p.max_tiles * ((p.N + BM - 1) / BM);
    if (DENSE && p.ksplit > 1) units *= C::DENSE_ACC;
    const int grid = (int)(units < nsm ? units : nsm);
    if (grid <= 0) return 0;
    k_gemm_q4k<DUAL, DENSE, PT><<<grid, NTHREADS, C::SMEM, s>>>(mx, ma, pm, p);
    return (int)cudaGetLastError();
}
}  // namespace gemm

int launch_gemm_q4k(const GemmParams &p, cudaStream_t s) {
    if (!p.w0 || !p.x || !(p.out || p.row_dst) || !p.tiles || !p.ntiles || !p.err) return CK_ERR_ARG;
    if (p.row_dst && (p.dual || p.N % 8 || p.max_tile_tok)) return CK_ERR_ARG;
    if (p.K % gemm::BK != 0 || p.N == 0 || p.K == 0 || ((uint64_t)p.N * p.K) % 256 != 0) return CK_ERR_SHAPE;
    if (p.dual && !p.w1) return CK_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(p.x) & 15) || (reinterpret_cast<uintptr_t>(p.w0) & 15)) return CK_ERR_ARG;
    // tiles of at most eight tokens (a decode-sized batch): the weight-streaming grouped matvec
    if (p.max_tile_tok && gemv_moe_ok(p)) return launch_gemv_moe(p, s);
    // TMA-staged packed weights when every row starts on a superblock and the tile is full height
    const bool pt = p.K % 256 == 0 && p.N >= (uint32_t)gemm::BM && !(reinterpret_cast<uintptr_t>(p.w0) & 15) &&
                    !(p.w1 && (reinterpret_cast<uintptr_t>(p.w1) & 15)) &&
                    !(p.s0 && (reinterpret_cast<uintptr_t>(p.s0) & 15)) &&
                    !(p.s1 && (reinterpret_cast<uintptr_t>(p.s1) & 15));
    if (p.dual) return pt ? gemm::launch_t<1, 0, 1>(p, s) : gemm::launch_t<1, 0, 0>(p, s);
    return pt ? gemm::launch_t<0, 0, 1>(p, s) : gemm::launch_t<0, 0, 0>(p, s);
}

int launch_gemm_dense(const GemmParams &p, cudaStream_t s) {
    if (!p.a_dense || !p.x || !p.out_f32 || !p.tiles || !p.ntiles || !p.err || (p.ksplit > 1 && !p.out_planes))
        return CK_ERR_ARG;
    if (p.K % gemm::BK != 0 || p.K == 0 || p.N == 0 || (p.kx && (p.kx % gemm::BK || p.K % p.kx))) return CK_ERR_SHAPE;
    if ((reinterpret_cast<uintptr_t>(p.x) & 15) || (reinterpret_cast<uintptr_t>(p.a_dense) & 15)) return CK_ERR_ARG;
    return gemm::launch_t<0, 1, 0>(p, s);
}

}  // namespace ck
