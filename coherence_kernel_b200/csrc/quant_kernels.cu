// quant_kernels.cu -- GGUF Q8_0 / Q4_K dequant and decode matvec on sm_100a.
//
// Every kernel reads the packed GGUF blocks exactly as they lie in memory (flat index, rows may
// straddle blocks: form/form-stdlib/q4k-msl.fk:73-86, q8-0-msl.fk:53-70).  Two families:
//   *_ordered : one thread per row, j counting down, acc = p + acc with no fused multiply-add --
//               the attestant order of the reference's emitted kernels (q8-0-msl.fk:100-103,
//               q4k-msl.fk:111-114), kept for callers that want that association.
//   *_fast    : bandwidth-bound decode matvecs: coalesced vector loads of the packed blocks, the
//               nibble / scale unpack in registers, warp-shuffle reductions.
#include "ck_common.cuh"
#include "ck_launch.h"

namespace ck {

// ------------------------------------------------------------------ scalar weight decode
CK_DEV float q80_weight(const uint8_t *__restrict__ qb, uint64_t idx) {
    uint64_t b = (idx >> 5) * Q80_BYTES;
    uint32_t i = (uint32_t)(idx & 31);
    float d = f16_bits_to_float((uint32_t)qb[b] | ((uint32_t)qb[b + 1] << 8));
    return d * (float)(int8_t)qb[b + 2 + i];
}

CK_DEV float q4k_weight(const uint8_t *__restrict__ qb, uint64_t idx) {
    const uint8_t *b = qb + (idx >> 8) * Q4K_BYTES;
    int i = (int)(idx & 255);
    int c = i >> 6, hf = (i >> 5) & 1, l = i & 31, j = 2 * c + hf;
    uint32_t s[3];
    for (int k = 0; k < 3; ++k)
        s[k] = (uint32_t)b[4 + 4 * k] | ((uint32_t)b[5 + 4 * k] << 8) | ((uint32_t)b[6 + 4 * k] << 16) |
               ((uint32_t)b[7 + 4 * k] << 24);
    int sc, mn;
    q4k_scale_min(s, j, sc, mn);
    int qbyte = b[16 + c * 32 + l];
    int nib = hf ? (qbyte >> 4) : (qbyte & 15);
    float d = f16_bits_to_float((uint32_t)b[0] | ((uint32_t)b[1] << 8));
    float dmin = f16_bits_to_float((uint32_t)b[2] | ((uint32_t)b[3] << 8));
    // (d*sc)*nib - dmin*m: d*sc and dmin*m are exact in fp32; one rounding for the product with
    // nib, one for the difference -- the operation order of q4k-msl.fk's q4k_w.
    return __fsub_rn(__fmul_rn(d * (float)sc, (float)nib), dmin * (float)mn);
}

__global__ void k_q80_dequant(const uint8_t *__restrict__ qb, float *__restrict__ w, uint64_t off, uint64_t n) {
    uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) w[i] = q80_weight(qb, off + i);
}
__global__ void k_q4k_dequant(const uint8_t *__restrict__ qb, float *__restrict__ w, uint64_t off, uint64_t n) {
    uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) w[i] = q4k_weight(qb, off + i);
}

// Dequant to bf16 (used to build dense references and by callers that want bf16 weights).
__global__ void k_q4k_dequant_bf16(const uint8_t *__restrict__ qb, __nv_bfloat16 *__restrict__ w, uint64_t off,
                                   uint64_t n) {
    uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) w[i] = __float2bfloat16_rn(q4k_weight(qb, off + i));
}

// ------------------------------------------------------------------ attestant-order matvecs
template <int KIND>
__global__ void k_matvec_ordered(const uint8_t *__restrict__ qb, const float *__restrict__ x, float *__restrict__ y,
                                 uint32_t rows, uint32_t cols) {
    uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    float acc = 0.0f;
    uint32_t j = cols;
    while (j > 0) {
        j -= 1;
        uint64_t idx = (uint64_t)r * cols + j;
        float w = KIND == 8 ? q80_weight(qb, idx) : q4k_weight(qb, idx);
        float p = __fmul_rn(w, x[j]);
        acc = __fadd_rn(p, acc);
    }
    y[r] = acc;
}

// ------------------------------------------------------------------ Q4_K decode matvec (fast)
// One warp per row.  The row is walked in 64-weight chunks (cols % 64 == 0, so every row starts
// on a chunk boundary even when it straddles superblocks).  A group of 8 lanes owns one chunk:
// lane q of the group loads 4 bytes of the chunk's 32 qs bytes (weights 4q..4q+3 of sub-block 2c
// in the low nibbles, of sub-block 2c+1 in the high nibbles) plus the superblock's 16-byte header
// (one broadcast load); four groups cover one 144-byte superblock's qs in one coalesced 128-byte
// load.  Per sub-block the dot is factored as d*sc*sum(q*x) - dmin*m*sum(x).
// xc[t] points at token t's 64 activations for this chunk.
template <int NT>
CK_DEV void q4k_chunk_dot(const uint8_t *__restrict__ qb, uint64_t chunk, int q, const float *const *xc,
                          float (&acc)[NT]) {
    const uint64_t sb = chunk >> 2;
    const int c = (int)(chunk & 3);
    const uint8_t *blk = qb + sb * Q4K_BYTES;
    const uint4 hdr = __ldg(reinterpret_cast<const uint4 *>(blk));
    const uint32_t qw = __ldg(reinterpret_cast<const uint32_t *>(blk + 16 + c * 32 + q * 4));
    const float d = f16_bits_to_float(hdr.x & 0xFFFF), dmin = f16_bits_to_float(hdr.x >> 16);
    uint32_t s[3] = {hdr.y, hdr.z, hdr.w};
    int sc0, m0, sc1, m1;
    q4k_scale_min(s, 2 * c, sc0, m0);
    q4k_scale_min(s, 2 * c + 1, sc1, m1);
    const float ds0 = d * (float)sc0, dm0 = dmin * (float)m0, ds1 = d * (float)sc1, dm1 = dmin * (float)m1;
    const float q0 = (float)(qw & 15), q1 = (float)((qw >> 8) & 15), q2 = (float)((qw >> 16) & 15),
                q3 = (float)((qw >> 24) & 15);
    const float h0 = (float)((qw >> 4) & 15), h1 = (float)((qw >> 12) & 15), h2 = (float)((qw >> 20) & 15),
                h3 = (float)((qw >> 28) & 15);
#pragma unroll
    for (int t = 0; t < NT; ++t) {
        const float4 xl = __ldg(reinterpret_cast<const float4 *>(xc[t] + q * 4));
        const float4 xh = __ldg(reinterpret_cast<const float4 *>(xc[t] + 32 + q * 4));
        float sl = q0 * xl.x;
        sl = fmaf(q1, xl.y, sl);
        sl = fmaf(q2, xl.z, sl);
        sl = fmaf(q3, xl.w, sl);
        float sh = h0 * xh.x;
        sh = fmaf(h1, xh.y, sh);
        sh = fmaf(h2, xh.z, sh);
        sh = fmaf(h3, xh.w, sh);
        const float xsl = (xl.x + xl.y) + (xl.z + xl.w);
        const float xsh = (xh.x + xh.y) + (xh.z + xh.w);
        acc[t] = fmaf(ds0, sl, acc[t]);
        acc[t] = fmaf(-dm0, xsl, acc[t]);
        acc[t] = fmaf(ds1, sh, acc[t]);
        acc[t] = fmaf(-dm1, xsh, acc[t]);
    }
}

// y[t*rows + r] = sum_j W[r, j] * x[t*cols + j] for NT tokens at once (NT = 1: decode matvec).
template <int NT>
__global__ void __launch_bounds__(256) k_q4k_matvec_fast(const uint8_t *__restrict__ qb, const float *__restrict__ x,
                                                         float *__restrict__ y, uint32_t rows, uint32_t cols,
                                                         uint32_t ntok) {
    const int lane = threadIdx.x & 31;
    const uint32_t r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r >= rows) return;
    const uint32_t t0 = blockIdx.y * NT;
    const int g = lane >> 3, q = lane & 7;
    const float *xs[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) xs[t] = x + (uint64_t)min(t0 + t, ntok - 1) * cols;
    float acc[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[t] = 0.0f;
    const uint32_t nchunk = cols >> 6;
    const uint64_t chunk0 = ((uint64_t)r * cols) >> 6;
    uint32_t k = g;
#pragma unroll 1
    for (; k + 12 < nchunk; k += 16) {
        // four chunks per lane group in flight
        const float *xk[NT];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
#pragma unroll
            for (int t = 0; t < NT; ++t) xk[t] = xs[t] + (uint64_t)(k + 4 * u) * 64;
            q4k_chunk_dot<NT>(qb, chunk0 + k + 4 * u, q, xk, acc);
        }
    }
    for (; k < nchunk; k += 4) {
        const float *xk[NT];
#pragma unroll
        for (int t = 0; t < NT; ++t) xk[t] = xs[t] + (uint64_t)k * 64;
        q4k_chunk_dot<NT>(qb, chunk0 + k, q, xk, acc);
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) {
        float v = acc[t];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0 && t0 + t < ntok) y[(uint64_t)(t0 + t) * rows + r] = v;
    }
}

// ------------------------------------------------------------------ Q8_0 decode matvec (fast)
// One warp per row, cols % 256 == 0 so each row's 34*cols/32 bytes start 16-byte aligned.  The
// warp copies its row into shared memory with 16-byte coalesced loads, then lane q of an 8-lane
// group takes 4 codes of one block (4 blocks per warp step), reading x as float4.
__global__ void __launch_bounds__(256) k_q80_matvec_fast(const uint8_t *__restrict__ qb, const float *__restrict__ x,
                                                         float *__restrict__ y, uint32_t rows, uint32_t cols) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const uint32_t r = blockIdx.x * (blockDim.x >> 5) + w;
    const uint32_t row_bytes = cols / 32 * Q80_BYTES;
    uint8_t *rowbuf = smem + (size_t)w * row_bytes;
    if (r >= rows) return;
    const uint4 *src = reinterpret_cast<const uint4 *>(qb + (uint64_t)r * row_bytes);
    uint4 *dst = reinterpret_cast<uint4 *>(rowbuf);
    const uint32_t nvec = row_bytes / 16;
    for (uint32_t v = lane; v < nvec; v += 32) dst[v] = __ldg(src + v);
    __syncwarp();
    const int g = lane >> 3, q = lane & 7;
    float acc = 0.0f;
    const uint32_t nblk = cols / 32;
    for (uint32_t b = g; b < nblk; b += 4) {
        const uint8_t *blk = rowbuf + b * Q80_BYTES;
        const float d = f16_bits_to_float((uint32_t)blk[0] | ((uint32_t)blk[1] << 8));
        const uint16_t lo = *reinterpret_cast<const uint16_t *>(blk + 2 + 4 * q);
        const uint16_t hi = *reinterpret_cast<const uint16_t *>(blk + 4 + 4 * q);
        const float4 xv = __ldg(reinterpret_cast<const float4 *>(x + b * 32 + 4 * q));
        float s = (float)(int8_t)(lo & 0xFF) * xv.x;
        s = fmaf((float)(int8_t)(lo >> 8), xv.y, s);
        s = fmaf((float)(int8_t)(hi & 0xFF), xv.z, s);
        s = fmaf((float)(int8_t)(hi >> 8), xv.w, s);
        acc = fmaf(d, s, acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) y[r] = acc;
}

// Q8_0 matvec for any cols % 32 == 0: one warp per row, lane = code index inside each block.
__global__ void k_q80_matvec_lane(const uint8_t *__restrict__ qb, const float *__restrict__ x, float *__restrict__ y,
                                  uint32_t rows, uint32_t cols) {
    const int lane = threadIdx.x & 31;
    const uint32_t r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r >= rows) return;
    float acc = 0.0f;
    const uint64_t b0 = (uint64_t)r * (cols / 32);
    for (uint32_t b = 0; b < cols / 32; ++b) {
        const uint8_t *blk = qb + (b0 + b) * Q80_BYTES;
        const float d = f16_bits_to_float((uint32_t)blk[0] | ((uint32_t)blk[1] << 8));
        acc = fmaf(d * (float)(int8_t)blk[2 + lane], x[b * 32 + lane], acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) y[r] = acc;
}

// ------------------------------------------------------------------ F16 matvec (router gate)
// y[r] = sum_j f16(W[r*cols + j]) * x[j] (moe-msl.fk:123-126), one warp per row.
__global__ void k_f16_matvec(const uint16_t *__restrict__ w, const float *__restrict__ x, float *__restrict__ y,
                             uint32_t rows, uint32_t cols) {
    const int lane = threadIdx.x & 31;
    const uint32_t r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r >= rows) return;
    float acc = 0.0f;
    const uint16_t *row = w + (uint64_t)r * cols;
    for (uint32_t j = lane; j < cols; j += 32) acc = fmaf(f16_bits_to_float(row[j]), x[j], acc);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) y[r] = acc;
}

// ------------------------------------------------------------------ elementwise
// form_scale_f32 / form_axpy_f32 (moe-msl.fk:129-140): y = a*x ; y = y + a*x (no contraction).
__global__ void k_scale(const float *__restrict__ x, float *__restrict__ y, float a, uint32_t n) {
    uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = __fmul_rn(a, x[i]);
}
__global__ void k_axpy(const float *__restrict__ x, float *__restrict__ y, float a, uint32_t n) {
    uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = __fadd_rn(y[i], __fmul_rn(a, x[i]));
}
// form_dsv4_swiglu_f32 (dsv4-moe-msl.fk:87-88): (silu(clamp_hi g) * clamp(u)) * w, clamp off when
// lim <= 1e-6.  silu(g) = g / (1 + exp(-g)).
__global__ void k_swiglu(const float *__restrict__ g, const float *__restrict__ u, float *__restrict__ out, uint32_t n,
                         float w, float lim) {
    uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float gv = g[i], uv = u[i];
    if (lim > 1e-6f) {
        gv = gv > lim ? lim : gv;
        uv = uv > lim ? lim : uv;
        uv = uv < -lim ? -lim : uv;
    }
    float s = gv / (1.0f + expf(-gv));
    out[i] = __fmul_rn(__fmul_rn(s, uv), w);
}

// ------------------------------------------------------------------ launchers
static inline unsigned nblk(uint64_t n, unsigned t) { return (unsigned)((n + t - 1) / t); }

int launch_q80_dequant(const uint8_t *qb, float *w, uint64_t off, uint64_t n, cudaStream_t s) {
    if (n == 0) return 0;
    k_q80_dequant<<<nblk(n, 256), 256, 0, s>>>(qb, w, off, n);
    return (int)cudaGetLastError();
}
int launch_q4k_dequant(const uint8_t *qb, float *w, uint64_t off, uint64_t n, cudaStream_t s) {
    if (n == 0) return 0;
    k_q4k_dequant<<<nblk(n, 256), 256, 0, s>>>(qb, w, off, n);
    return (int)cudaGetLastError();
}
int launch_q4k_dequant_bf16(const uint8_t *qb, void *w, uint64_t off, uint64_t n, cudaStream_t s) {
    if (n == 0) return 0;
    k_q4k_dequant_bf16<<<nblk(n, 256), 256, 0, s>>>(qb, (__nv_bfloat16 *)w, off, n);
    return (int)cudaGetLastError();
}
int launch_matvec_ordered(int kind, const uint8_t *qb, const float *x, float *y, uint32_t rows, uint32_t cols,
                          cudaStream_t s) {
    if (kind == 8)
        k_matvec_ordered<8><<<nblk(rows, 128), 128, 0, s>>>(qb, x, y, rows, cols);
    else
        k_matvec_ordered<12><<<nblk(rows, 128), 128, 0, s>>>(qb, x, y, rows, cols);
    return (int)cudaGetLastError();
}
// ng matrices of one shape against the same x: one tensor-core launch where a single one would take
// the tensor-core matvec (each y bit-identical to its single launch), else one launch each
int launch_q4k_matvec_group(uint32_t ng, const uint8_t *const *qb, const float *x, float *const *y, uint32_t rows,
                            uint32_t cols, uint32_t ntok, cudaStream_t s) {
    bool tc = ntok == 1 && ng >= 1 && ng <= 4 && cols % 64 == 0;
    for (uint32_t g = 0; tc && g < ng; ++g)
        tc = gemv_tc_ok(qb[g], x, rows, cols) &&
             (!gemv_stream_ok(qb[g], x, cols) || (uint64_t)rows * (cols / 256) * Q4K_BYTES >= (12ull << 20));
    if (tc) return launch_gemv_tc_group(ng, qb, x, y, rows, cols, s);
    for (uint32_t g = 0; g < ng; ++g) {
        const int rc = launch_q4k_matvec(qb[g], x, y[g], rows, cols, ntok, s);
        if (rc) return rc;
    }
    return 0;
}

int launch_q4k_matvec(const uint8_t *qb, const float *x, float *y, uint32_t rows, uint32_t cols, uint32_t ntok,
                      cudaStream_t s) {
    if (cols % 64 != 0) return CK_ERR_SHAPE;
    // one token: the tensor-core matvec from about 12 MB of weights up (and wherever the streaming
    // kernel's x does not fit its shared memory), the streaming one below that, where its shorter
    // fixed cost per launch wins
    const bool stream_ok = gemv_stream_ok(qb, x, cols);
    if (ntok == 1 && gemv_tc_ok(qb, x, rows, cols) &&
        (!stream_ok || (uint64_t)rows * (cols / 256) * Q4K_BYTES >= (12ull << 20))) {
        return launch_gemv_tc(qb, x, y, rows, cols, s);
    } else if (ntok == 1 && stream_ok) {
        return launch_gemv_stream(12, qb, x, y, rows, cols, s);
    } else if (ntok == 1) {
        k_q4k_matvec_fast<1><<<dim3(nblk(rows, 8), 1), 256, 0, s>>>(qb, x, y, rows, cols, 1);
    } else {
        k_q4k_matvec_fast<8><<<dim3(nblk(rows, 8), nblk(ntok, 8)), 256, 0, s>>>(qb, x, y, rows, cols, ntok);
    }
    return (int)cudaGetLastError();
}
int launch_q80_matvec(const uint8_t *qb, const float *x, float *y, uint32_t rows, uint32_t cols, cudaStream_t s) {
    if (cols % 32 != 0) return CK_ERR_SHAPE;
    if (gemv_stream_ok(qb, x, cols)) {
        return launch_gemv_stream(8, qb, x, y, rows, cols, s);
    } else if (cols % 256 == 0 && (size_t)cols / 32 * Q80_BYTES * 8 <= 200 * 1024) {
        size_t smem = (size_t)cols / 32 * Q80_BYTES * 8;
        static unsigned long long attr_set = 0;
        if (attr_pending(attr_set)) {
            const cudaError_t e =
                cudaFuncSetAttribute(k_q80_matvec_fast, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
            if (e != cudaSuccess) return (int)e;
            attr_mark(attr_set);
        }
        k_q80_matvec_fast<<<nblk(rows, 8), 256, smem, s>>>(qb, x, y, rows, cols);
    } else {
        k_q80_matvec_lane<<<nblk(rows, 8), 256, 0, s>>>(qb, x, y, rows, cols);
    }
    return (int)cudaGetLastError();
}
int launch_f16_matvec(const uint16_t *w, const float *x, float *y, uint32_t rows, uint32_t cols, cudaStream_t s) {
    k_f16_matvec<<<nblk(rows, 8), 256, 0, s>>>(w, x, y, rows, cols);
    return (int)cudaGetLastError();
}
int launch_scale(const float *x, float *y, float a, uint32_t n, cudaStream_t s) {
    if (n) k_scale<<<nblk(n, 256), 256, 0, s>>>(x, y, a, n);
    return (int)cudaGetLastError();
}
int launch_axpy(const float *x, float *y, float a, uint32_t n, cudaStream_t s) {
    if (n) k_axpy<<<nblk(n, 256), 256, 0, s>>>(x, y, a, n);
    return (int)cudaGetLastError();
}
int launch_swiglu(const float *g, const float *u, float *out, uint32_t n, float w, float lim, cudaStream_t s) {
    if (n) k_swiglu<<<nblk(n, 256), 256, 0, s>>>(g, u, out, n, w, lim);
    return (int)cudaGetLastError();
}

}  // namespace ck
