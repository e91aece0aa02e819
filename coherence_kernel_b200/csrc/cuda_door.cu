// cuda_door.cu -- the reference runtime's CUDA matvec doors (tag 232, the fixture witness, and tag
// 233, `(cuda_matvec_f32 W x)`), served on Linux by this library.
//
// In the reference (runtime/fkwu-uni.c:4753-5050) both doors are Windows-only and static: they
// load nvcuda.dll, JIT the Form-emitted PTX `form_matvec_f32` at -O0 (so mul.f32 and add.f32 stay
// unfused), run y = W.x with one thread per row on host-resident W and x, tear the context down,
// and compare every row BIT-EXACT with the CPU's downward right fold of two roundings.  Elsewhere
// the ops answer nil.  The seam here is fk_cuda_go_external, the same contract as the reference's
// fk_cuda_go (W [rows*cols], x [cols] and y [rows] in host memory; the device name into gname;
// 0 or the negative step code of the first refusal), on the sm_100a kernel k_f32_matvec: one thread
// per row, j counting down, acc = (w*x) + acc with __fmul_rn / __fadd_rn -- the same two roundings
// per term, so the rows agree bit for bit.  fk_cuda_matvec_f32_external adds the door's own CPU
// recomputation and answers the agreement count; fk_cuda_matvec_fixture_external is tag 232.
#include "../../include/fk_cuda_carrier.h"
#include "ck_launch.h"
#include "form_kernels.h"

#include <cuda_runtime.h>
#include <stdio.h>
#include <string.h>

namespace {
// the reference's refusal codes (fk_cuda_say): -3 the driver did not initialize, -4 no device,
// -9 the launch failed; -10 a device allocation or copy failed
long long go(const float *W, const float *x, float *y, unsigned rows, unsigned cols, char *gname, long long gcap) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return -3;
    }
    if (n == 0) return -4;
    int dev = 0;
    cudaGetDevice(&dev);
    if (gname && gcap > 0) {
        cudaDeviceProp p;
        gname[0] = 0;
        if (cudaGetDeviceProperties(&p, dev) == cudaSuccess) {
            strncpy(gname, p.name, (size_t)gcap - 1);
            gname[gcap - 1] = 0;
        }
    }
    const size_t wb = (size_t)rows * cols * 4, xb = (size_t)cols * 4, yb = (size_t)rows * 4;
    float *dW = nullptr, *dX = nullptr, *dY = nullptr;
    long long rc = 0;
    if (cudaMalloc(&dW, wb ? wb : 4) != cudaSuccess || cudaMalloc(&dX, xb ? xb : 4) != cudaSuccess ||
        cudaMalloc(&dY, yb ? yb : 4) != cudaSuccess)
        rc = -10;
    if (rc == 0 && (cudaMemcpy(dW, W, wb, cudaMemcpyHostToDevice) != cudaSuccess ||
                    cudaMemcpy(dX, x, xb, cudaMemcpyHostToDevice) != cudaSuccess))
        rc = -10;
    if (rc == 0 && (ck::launch_f32_matvec(dW, dX, dY, rows, cols, 0) != 0 || cudaDeviceSynchronize() != cudaSuccess))
        rc = -9;
    if (rc == 0 && cudaMemcpy(y, dY, yb, cudaMemcpyDeviceToHost) != cudaSuccess) rc = -10;
    if (rc != 0) cudaGetLastError();
    cudaFree(dW);
    cudaFree(dX);
    cudaFree(dY);
    return rc;
}

// the CPU side of the door: the downward right fold, two roundings per term (volatile keeps the
// compiler from contracting the multiply and the add)
long long agree_rows(const float *W, const float *x, const float *y, unsigned rows, unsigned cols) {
    long long agree = 0;
    for (unsigned i = 0; i < rows; ++i) {
        volatile float acc = 0.0f;
        for (long long j = (long long)cols - 1; j >= 0; --j) {
            volatile float prod = W[(size_t)i * cols + j] * x[j];
            acc = prod + acc;
        }
        const float cpu = acc;
        unsigned a, b;
        memcpy(&a, &cpu, 4);
        memcpy(&b, &y[i], 4);
        agree += a == b;
    }
    return agree;
}
}  // namespace

extern "C" {

long long fk_cuda_go_external(const float *W, const float *x, float *y, unsigned rows, unsigned cols, char *gname,
                              long long gcap) {
    if (!W || !x || !y || rows == 0 || cols == 0) return -9;
    return go(W, x, y, rows, cols, gname, gcap);
}

long long fk_cuda_matvec_f32_external(const float *W, const float *x, float *y, unsigned rows, unsigned cols) {
    // the door's own limits: at least one column, at most 4194304 weights
    if (!W || !x || !y || cols == 0 || rows == 0 || (unsigned long long)rows * cols > 4194304ull) return -1;
    char gname[256];
    const long long rc = go(W, x, y, rows, cols, gname, sizeof(gname));
    if (rc < 0) return rc;
    const long long agree = agree_rows(W, x, y, rows, cols);
    printf("GPU: %s  cuda_matvec_f32 rows=%u cols=%u  BIT-EXACT %lld/%u\n", gname, rows, cols, agree, rows);
    return agree;
}

long long fk_cuda_matvec_fixture_external(void) {
    const unsigned rows = 3, cols = 4;
    const float W[12] = {0.1f, 0.2f, 0.3f, 0.7f, 0.11f, 0.13f, 0.17f, 0.19f, 0.9f, 0.8f, 0.123456f, 0.654321f};
    const float X[4] = {0.5f, 0.25f, 0.125f, 0.333333f};
    float Y[3] = {0.0f, 0.0f, 0.0f};
    char gname[256];
    const long long rc = go(W, X, Y, rows, cols, gname, sizeof(gname));
    if (rc < 0) return rc;
    const long long agree = agree_rows(W, X, Y, rows, cols);
    printf("GPU: %s  sm_100a form_matvec_f32 (one thread per row, downward right fold, 2 roundings)\n", gname);
    printf("AGREEMENT: %lld/%u  ALL-BIT-EXACT=%s\n", agree, rows, agree == (long long)rows ? "true" : "false");
    return agree;
}

}  // extern "C"
