// Mirror of the reference's test harness (nirw4nna/hipgemm test.cpp:49-95), calling the
// B200 kernel through the C ABI.  Same flow: pinned host + device buffers, seeded
// inputs (utils.hpp:27-33), H2D copies, CPU GEMM (the oracle restating test.cpp:19-30),
// one launch, D2H copy, full-matrix validation, "Test passed: %i".  Differences: the
// exit code reflects the result (the reference always returns 0), the validator uses
// |ref| (test.cpp:39 compares against a signed threshold) and counts every mismatch.
//
//   ./test_gemm                      compile-time MDIM x NDIM x KDIM (default 4096^3),
//                                    the reference's own inputs: seed 0 for A and B,
//                                    N(-1, 1) cast straight to e4m3, no scale, launched
//                                    through fp8_gemm_4wave_256x256x128<M, N, K>(...)
//   ./test_gemm M N K scaled         runtime shape, benchmark-config inputs: A seed 0, B seed 1,
//                                    N(0, 1), per-tensor amax/448 scales (hgemm_fp8_tn)
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>

#include "hipgemm_b200.h"
#include "oracle.h"

#ifndef MDIM
#define MDIM 4096
#endif
#ifndef NDIM
#define NDIM 4096
#endif
#ifndef KDIM
#define KDIM 4096
#endif

#define CHECK_CUDA(expr)                                                                           \
    do {                                                                                           \
        cudaError_t e_ = (expr);                                                                   \
        if (e_ != cudaSuccess) {                                                                   \
            fprintf(stderr, "CUDA error: '%s'(%d) at %s:%d\n", cudaGetErrorString(e_), int(e_),   \
                    __FILE__, __LINE__);                                                           \
            exit(EXIT_FAILURE);                                                                    \
        }                                                                                          \
    } while (0)

static void* cuda_malloc_host(size_t n) {
    void* p = nullptr;
    CHECK_CUDA(cudaMallocHost(&p, n ? n : 1));
    return p;
}

static void* cuda_malloc_device(size_t n) {
    void* p = nullptr;
    CHECK_CUDA(cudaMalloc(&p, n ? n : 1));
    return p;
}

int main(int argc, char** argv) {
    const bool runtime_shape = argc >= 4;
    const int M = runtime_shape ? std::atoi(argv[1]) : MDIM;
    const int N = runtime_shape ? std::atoi(argv[2]) : NDIM;
    const int K = runtime_shape ? std::atoi(argv[3]) : KDIM;
    const bool scaled = argc >= 5 && std::string(argv[4]) == "scaled";

    const size_t a_bytes = size_t(M) * K, b_bytes = size_t(N) * K, c_bytes = size_t(M) * N * 2;
    uint8_t* A_host = static_cast<uint8_t*>(cuda_malloc_host(a_bytes));
    uint8_t* B_host = static_cast<uint8_t*>(cuda_malloc_host(b_bytes));
    uint16_t* C_host = static_cast<uint16_t*>(cuda_malloc_host(c_bytes));
    uint16_t* C_ref = static_cast<uint16_t*>(cuda_malloc_host(c_bytes));
    void* A_dev = cuda_malloc_device(a_bytes);
    void* B_dev = cuda_malloc_device(b_bytes);
    void* C_dev = cuda_malloc_device(c_bytes);
    float* scales_dev = static_cast<float*>(cuda_malloc_device(2 * sizeof(float)));

    float sa = 1.0f, sb = 1.0f;
    if (scaled) {
        sa = oracle_make_quantized(A_host, a_bytes, 0, 0.0f, 1.0f);
        sb = oracle_make_quantized(B_host, b_bytes, 1, 0.0f, 1.0f);
    } else {
        oracle_init_random_fp8(A_host, a_bytes, 0, -1.0f, 1.0f);  // test.cpp:70
        oracle_init_random_fp8(B_host, b_bytes, 0, -1.0f, 1.0f);  // test.cpp:71 (same seed)
    }
    const float scales[2] = {sa, sb};
    CHECK_CUDA(cudaMemcpy(A_dev, A_host, a_bytes, cudaMemcpyHostToDevice));
    CHECK_CUDA(cudaMemcpy(B_dev, B_host, b_bytes, cudaMemcpyHostToDevice));
    CHECK_CUDA(cudaMemcpy(scales_dev, scales, sizeof(scales), cudaMemcpyHostToDevice));

    oracle_gemm(A_host, B_host, C_ref, M, N, K, sa, sb, 0);

    int rc;
    if (runtime_shape) {
        rc = hgemm_fp8_tn(A_dev, B_dev, C_dev, M, N, K, scales_dev, scales_dev + 1, nullptr);
    } else {
        // The reference's launch line (test.cpp:79) minus the <<<grid, block>>>.
        rc = fp8_gemm_4wave_256x256x128<MDIM, NDIM, KDIM>(A_dev, B_dev, C_dev);
    }
    if (rc != HGEMM_OK) {
        fprintf(stderr, "hgemm error %d: %s\n", rc, hgemm_error_string(rc));
        return EXIT_FAILURE;
    }
    CHECK_CUDA(cudaMemcpy(C_host, C_dev, c_bytes, cudaMemcpyDeviceToHost));
    CHECK_CUDA(cudaGetLastError());
    uint32_t status = 0;
    if (hgemm_device_status(&status) != HGEMM_OK) {
        fprintf(stderr, "kernel status word %#x\n", status);
        return EXIT_FAILURE;
    }

    int64_t first_bad = -1;
    const int64_t bad = oracle_validate(C_host, C_ref, int64_t(M) * N, 1e-2f, 1e-3f, &first_bad);
    if (bad) {
        const int64_t r = first_bad / N, c = first_bad % N;
        fprintf(stderr, "%lld mismatches; first at (row=%lld, col=%lld): c = %f, c_ref = %f\n", (long long)bad,
                (long long)r, (long long)c, oracle_bf16_to_float(C_host[first_bad]),
                oracle_bf16_to_float(C_ref[first_bad]));
    }
    const bool success = bad == 0;
    printf("M=%d N=%d K=%d %s: %lld/%lld elements within |d| <= 1e-2*|ref| + 1e-3\n", M, N, K,
           scaled ? "scaled" : "reference-inputs", (long long)(int64_t(M) * N - bad), (long long)(int64_t(M) * N));
    if (!scaled) printf("reference validator (test.cpp:32-47): %s\n", oracle_validate_reference(C_host, C_ref, M, N) ? "pass" : "fail");
    printf("Test passed: %i\n", success);

    CHECK_CUDA(cudaFreeHost(A_host));
    CHECK_CUDA(cudaFreeHost(B_host));
    CHECK_CUDA(cudaFreeHost(C_host));
    CHECK_CUDA(cudaFreeHost(C_ref));
    CHECK_CUDA(cudaFree(A_dev));
    CHECK_CUDA(cudaFree(B_dev));
    CHECK_CUDA(cudaFree(C_dev));
    CHECK_CUDA(cudaFree(scales_dev));
    return success ? EXIT_SUCCESS : EXIT_FAILURE;
}
