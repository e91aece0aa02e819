// form_kernels.cu -- the small elementwise / partial kernels the reference's Form cells dispatch
// by name through the handle door, with their emitted argument layouts:
//   form_q4k_matvec_part_f32 / form_part_combine_f32   qk-matvec-split.fk:114-127
//   form_swiglu_f32                                     llama-decode-msl.fk:163-166
//   form_dsv4_matvec_f32                                dsv4-moe-msl.fk:82-83
//   form_dsv4_swiglu_experts / form_dsv4_moe_reduce     ds4-order-match.fk:261-264
// Each keeps the reference kernel's association (a right fold where the reference folds right).
#include "ck_common.cuh"
#include "ck_launch.h"
#include "form_kernels.h"

namespace ck {

CK_DEV float q4k_weight_f(const uint8_t *__restrict__ qb, uint64_t idx) {
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
    return __fsub_rn(__fmul_rn(d * (float)sc, (float)nib), dmin * (float)mn);
}

__global__ void k_q4k_part(const uint8_t *__restrict__ qb, const float *__restrict__ x, float *__restrict__ part,
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
        acc = __fadd_rn(__fmul_rn(q4k_weight_f(qb, (uint64_t)r * cols + j), x[j]), acc);
    }
    part[gid] = acc;
}
__global__ void k_part_combine(const float *__restrict__ part, float *__restrict__ y, uint32_t rows, uint32_t parts) {
    const uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    float acc = 0.0f;
    for (uint32_t p = parts; p > 0;) {
        --p;
        acc = __fadd_rn(part[(uint64_t)r * parts + p], acc);
    }
    y[r] = acc;
}
__global__ void k_swiglu_plain(const float *__restrict__ g, const float *__restrict__ u, float *__restrict__ y, uint32_t n) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float gv = g[i];
    const float sig = 1.0f / (1.0f + expf(-gv));
    y[i] = __fmul_rn(__fmul_rn(gv, sig), u[i]);
}
__global__ void k_f32_matvec(const float *__restrict__ W, const float *__restrict__ x, float *__restrict__ y, uint32_t rows,
                             uint32_t cols) {
    const uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    float acc = 0.0f;
    for (int c = (int)cols - 1; c >= 0; --c) acc = __fadd_rn(__fmul_rn(W[(uint64_t)r * cols + c], x[c]), acc);
    y[r] = acc;
}
__global__ void k_swiglu_experts(const float *__restrict__ g, const float *__restrict__ u, float *__restrict__ out,
                                 const float *__restrict__ wts, uint32_t n, uint32_t nexp, float lim) {
    const uint64_t gid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= (uint64_t)n * nexp) return;
    const uint32_t slot = (uint32_t)(gid / n);
    float gv = g[gid], uv = u[gid];
    if (lim > 1e-6f) {
        gv = gv > lim ? lim : gv;
        uv = uv > lim ? lim : uv;
        uv = uv < -lim ? -lim : uv;
    }
    const float s = gv / (1.0f + expf(-gv));
    out[gid] = __fmul_rn(__fmul_rn(s, uv), wts[slot]);
}
__global__ void k_moe_reduce(const float *__restrict__ parts, float *__restrict__ out, uint32_t n, uint32_t nexp) {
    const uint32_t d = blockIdx.x * blockDim.x + threadIdx.x;
    if (d >= n) return;
    float s = 0.0f;
    for (uint32_t slot = 0; slot < nexp; ++slot) s = __fadd_rn(s, parts[(uint64_t)slot * n + d]);
    out[d] = s;
}

static inline unsigned nb(uint64_t n, unsigned t) { return (unsigned)((n + t - 1) / t); }

int launch_q4k_part(const uint8_t *qb, const float *x, float *part, uint32_t rows, uint32_t cols, uint32_t parts,
                    cudaStream_t s) {
    if (parts == 0) return CK_ERR_ARG;
    const uint64_t n = (uint64_t)rows * parts;
    if (n) k_q4k_part<<<nb(n, 128), 128, 0, s>>>(qb, x, part, rows, cols, parts);
    return (int)cudaGetLastError();
}
int launch_part_combine(const float *part, float *y, uint32_t rows, uint32_t parts, cudaStream_t s) {
    if (rows) k_part_combine<<<nb(rows, 128), 128, 0, s>>>(part, y, rows, parts);
    return (int)cudaGetLastError();
}
int launch_swiglu_plain(const float *g, const float *u, float *y, uint32_t n, cudaStream_t s) {
    if (n) k_swiglu_plain<<<nb(n, 256), 256, 0, s>>>(g, u, y, n);
    return (int)cudaGetLastError();
}
int launch_f32_matvec(const float *W, const float *x, float *y, uint32_t rows, uint32_t cols, cudaStream_t s) {
    if (rows) k_f32_matvec<<<nb(rows, 128), 128, 0, s>>>(W, x, y, rows, cols);
    return (int)cudaGetLastError();
}
int launch_swiglu_experts(const float *g, const float *u, float *out, const float *wts, uint32_t n, uint32_t nexp,
                          float lim, cudaStream_t s) {
    const uint64_t t = (uint64_t)n * nexp;
    if (t) k_swiglu_experts<<<nb(t, 256), 256, 0, s>>>(g, u, out, wts, n, nexp, lim);
    return (int)cudaGetLastError();
}
int launch_moe_reduce(const float *parts, float *out, uint32_t n, uint32_t nexp, cudaStream_t s) {
    if (n) k_moe_reduce<<<nb(n, 256), 256, 0, s>>>(parts, out, n, nexp);
    return (int)cudaGetLastError();
}

}  // namespace ck
