// form_kernels.h -- launchers for the small Form-dispatched kernels (form_kernels.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace ck {
int launch_q4k_part(const uint8_t *qb, const float *x, float *part, uint32_t rows, uint32_t cols, uint32_t parts,
                    cudaStream_t s);
int launch_part_combine(const float *part, float *y, uint32_t rows, uint32_t parts, cudaStream_t s);
int launch_swiglu_plain(const float *g, const float *u, float *y, uint32_t n, cudaStream_t s);
int launch_f32_matvec(const float *W, const float *x, float *y, uint32_t rows, uint32_t cols, cudaStream_t s);
int launch_swiglu_experts(const float *g, const float *u, float *out, const float *wts, uint32_t n, uint32_t nexp,
                          float lim, cudaStream_t s);
int launch_moe_reduce(const float *parts, float *out, uint32_t n, uint32_t nexp, cudaStream_t s);
}  // namespace ck
