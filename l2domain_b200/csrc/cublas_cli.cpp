// gemv_cublas_benchmark -- the cuBLAS comparator column, same contract as the reference's
// applications/gemv/src/gemv_cublas_benchmark.cu:42-110:
//   argv  M K runs warmups flush_l2 [dtype]   ->   "cublas_ms <ms> ms <GFLOP/s> GFLOP/s"
// fp32 uses cublasSgemv(OP_T) on the row-major M x K matrix; fp16/bf16 use cublasGemmEx with fp32
// compute.  This binary is a comparator only: no product path calls cuBLAS.
#include "l2d.h"

#include <cublas_v2.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#define CB_CHECK(cond, what)                                   \
    do {                                                       \
        if (!(cond)) {                                         \
            std::fprintf(stderr, "%s failed\n", what);         \
            std::exit(1);                                      \
        }                                                      \
    } while (0)

int main(int argc, char **argv) {
    int M = argc > 1 ? std::atoi(argv[1]) : 65536;
    int K = argc > 2 ? std::atoi(argv[2]) : 1024;
    int runs = argc > 3 ? std::atoi(argv[3]) : 20;
    int warmups = argc > 4 ? std::atoi(argv[4]) : 5;
    int flush_l2 = argc > 5 ? std::atoi(argv[5]) : 0;
    const char *dts = argc > 6 ? argv[6] : "fp32";
    int dtype = !std::strcmp(dts, "fp16") ? L2D_F16 : !std::strcmp(dts, "bf16") ? L2D_BF16 : L2D_F32;
    M = std::max(M, 1);
    K = std::max(K, 1);
    runs = std::max(runs, 1);
    warmups = std::max(warmups, 0);
    flush_l2 = std::max(0, std::min(flush_l2, 1));
    const int eb = dtype == L2D_F32 ? 4 : 2;
    int device = 0;
    CB_CHECK(cudaGetDevice(&device) == cudaSuccess, "cudaGetDevice");
    char name[256];
    CB_CHECK(l2d_device_info(device, nullptr, nullptr, nullptr, nullptr, name, sizeof name) == L2D_OK, "device_info");
    void *A = nullptr, *x = nullptr, *y = nullptr;
    CB_CHECK(cudaMalloc(&A, static_cast<size_t>(M) * K * eb) == cudaSuccess, "cudaMalloc A");
    CB_CHECK(cudaMalloc(&x, static_cast<size_t>(K) * eb) == cudaSuccess, "cudaMalloc x");
    CB_CHECK(cudaMalloc(&y, static_cast<size_t>(M) * eb) == cudaSuccess, "cudaMalloc y");
    CB_CHECK(l2d_fill_ref(A, dtype, 0, static_cast<uint64_t>(M) * K, 4242, 0, 0, nullptr) == L2D_OK, "fill A");
    CB_CHECK(l2d_fill_ref(x, dtype, 0, static_cast<uint64_t>(K), 4242, 1, 0, nullptr) == L2D_OK, "fill x");
    cublasHandle_t h;
    CB_CHECK(cublasCreate(&h) == CUBLAS_STATUS_SUCCESS, "cublasCreate");
    const float alpha = 1.0f, beta = 0.0f;
    cudaDataType_t t = dtype == L2D_F32 ? CUDA_R_32F : dtype == L2D_F16 ? CUDA_R_16F : CUDA_R_16BF;
    auto call = [&]() {
        cublasStatus_t s;
        if (dtype == L2D_F32)
            s = cublasSgemv(h, CUBLAS_OP_T, K, M, &alpha, static_cast<const float *>(A), K,
                            static_cast<const float *>(x), 1, &beta, static_cast<float *>(y), 1);
        else
            s = cublasGemmEx(h, CUBLAS_OP_T, CUBLAS_OP_N, M, 1, K, &alpha, A, t, K, x, t, K, &beta, y, t, M,
                             CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
        CB_CHECK(s == CUBLAS_STATUS_SUCCESS, "cuBLAS call");
    };
    for (int i = 0; i < warmups; ++i) call();
    CB_CHECK(cudaDeviceSynchronize() == cudaSuccess, "sync");
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    double total = 0;
    for (int r = 0; r < runs; ++r) {
        if (flush_l2) {
            CB_CHECK(l2d_l2_flush(device, nullptr) == L2D_OK, "flush");
            cudaDeviceSynchronize();
        }
        cudaEventRecord(e0);
        call();
        cudaEventRecord(e1);
        cudaEventSynchronize(e1);
        float ms = 0;
        cudaEventElapsedTime(&ms, e0, e1);
        total += ms;
    }
    double avg = total / runs;
    std::printf("=== cuBLAS %s ===\n", dtype == L2D_F32 ? "SGEMV" : "GemmEx GEMV");
    std::printf("gpu=%s M=%d K=%d runs=%d flush_l2=%d matrix=%.1f MiB\n", name, M, K, runs, flush_l2,
                static_cast<double>(M) * K * eb / (1024.0 * 1024.0));
    std::printf("cublas_ms %.6f ms %.2f GFLOP/s\n", avg, 2.0 * M * K / (avg * 1e6));
    cublasDestroy(h);
    cudaFree(A);
    cudaFree(x);
    cudaFree(y);
    return 0;
}
