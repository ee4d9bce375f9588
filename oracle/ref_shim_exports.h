// TEST INFRASTRUCTURE: the epilogue of oracle/_ref/libref_cpu.so (see ref_shim_types.h).
// C entry points over the reference's own functions, on raw e4m3 bytes and bf16 bits.

extern "C" {

// test.cpp:19-30, gemm_cpu: C (M x N, bf16) = A (M x K) . B^T (B: N x K), fp32 accumulator,
// k ascending, OpenMP over (row, col).  Unscaled, as the reference's test calls it.
void ref_gemm_cpu(const uint8_t* A, const uint8_t* B, uint16_t* C, int M, int N, int K) {
    gemm_cpu(reinterpret_cast<fp8*>(const_cast<uint8_t*>(A)), reinterpret_cast<fp8*>(const_cast<uint8_t*>(B)),
             reinterpret_cast<bf16*>(C), M, N, K);
}

// test.cpp:32-47, validate_matrix as written: 1 = passed.
int ref_validate_matrix(const uint16_t* C, const uint16_t* C_ref, int M, int N) {
    return validate_matrix(reinterpret_cast<bf16*>(const_cast<uint16_t*>(C)),
                           reinterpret_cast<bf16*>(const_cast<uint16_t*>(C_ref)), M, N) ? 1 : 0;
}

// utils.hpp:27-33, init_random: std::mt19937(seed) -> normal_distribution<float>(-1, 1) -> e4m3.
void ref_init_random(uint8_t* out, size_t n, size_t seed) {
    init_random(reinterpret_cast<fp8*>(out), n, seed);
}

int ref_max_threads(void) { return omp_get_max_threads(); }

// The thread count of the calling thread's next parallel regions (gemm_cpu's included): the
// process's OpenMP runtime may have read a launcher's OMP_NUM_THREADS=1 before this library
// was loaded.
void ref_set_num_threads(int n) { omp_set_num_threads(n); }

// The restated ROCm conversions alone (ref_shim_types.h), for checking them against the
// oracle's over whole ranges of inputs.
void ref_shim_e4m3_encode_array(const float* x, size_t n, uint8_t* out) {
    for (size_t i = 0; i < n; ++i) out[i] = fp8(x[i]).bits;
}

void ref_shim_bf16_array(const float* x, size_t n, uint16_t* out) {
    for (size_t i = 0; i < n; ++i) out[i] = bf16(x[i]).bits;
}

}  // extern "C"
