/*
 * CPU oracle for the FP8 e4m3 TN GEMM — TEST INFRASTRUCTURE ONLY.
 *
 * This library restates, on the host, the arithmetic of the reference's CPU GEMM
 * (nirw4nna/hipgemm test.cpp:19-30), its validator (test.cpp:32-47) and its input
 * generator (utils.hpp:27-33).  It is the checker for the CUDA path, and the timed
 * CPU baseline of bench.py.  Nothing in the product (hipgemm_b200/, include/) may
 * link or call it: only tests/, __graft_entry__.smoke() and bench.py's CPU legs.
 *
 * PINNED to the reference's own CPU code.  gemm_cpu, validate_matrix (test.cpp:19-47)
 * and init_random (utils.hpp:27-33) are compiled from the reference's files into
 * oracle/_ref/libref_cpu.so (`make -C oracle ref`), with only the ROCm element types
 * they use restated (ref_shim_types.h; the rest of those files is HIP code that g++
 * cannot compile).  This library reproduces that one bit for bit, the reference's own
 * test at its default 4096^3 included, and the fixtures it generated
 * (tests/golden/reference/) carry the comparison to machines without the reference's
 * sources (tests/test_oracle_reference.py).  The reference ships no golden vectors or
 * known-answer tests of its own.  Also pinned:
 *   - the fp8 e4m3 codec against the OCP FP8 spec's table values and, bit for bit
 *     over every float in a sweep, against CUDA's host-callable
 *     __nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3) (tests/test_oracle.py);
 *   - bf16 round-to-nearest-even against torch's float->bfloat16 cast;
 *   - std::mt19937 against the C++ standard's known answer (10000th draw of a
 *     default-seeded engine is 4123659995);
 *   - the GEMM loop against an independent numpy restatement on small shapes, and
 *     against the committed fixtures in tests/golden/.
 *
 * Conversion semantics follow the third-party headers the reference calls but does
 * not vendor (ROCm 7.2.2 amd_hip_fp8.h / amd_hip_bf16.h, pinned only by the image
 * tag in .devcontainer/devcontainer.json:3): OCP e4m3 ("fn": no infinities, max
 * 448), round-to-nearest-even, saturate finite overflow to +-448; bf16 by
 * round-to-nearest-even.
 */
#ifndef HIPGEMM_ORACLE_H
#define HIPGEMM_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* fp8 e4m3 (OCP, satfinite, RNE) encode of one float.  Call site in the reference:
 * utils.hpp:32 `fp8(dis(gen))`. */
uint8_t oracle_fp8_encode(float x);
/* Exact decode of one e4m3 byte.  Call site: test.cpp:25 `float(A[...])`. */
float oracle_fp8_decode(uint8_t b);
void oracle_fp8_encode_array(const float* x, size_t n, uint8_t* out);
void oracle_bf16_rne_array(const float* x, size_t n, uint16_t* out);
/* fp32 -> bf16 bits, round-to-nearest-even (NaN stays NaN).  Call site: test.cpp:27. */
uint16_t oracle_bf16_rne(float x);
float oracle_bf16_to_float(uint16_t b);

/* mt19937(seed) -> std::normal_distribution<float>(mean, stddev), n draws, as fp32.
 * utils.hpp:27-33 with the distribution's parameters made explicit. */
void oracle_normal_f32(float* out, size_t n, uint64_t seed, float mean, float stddev);
/* utils.hpp:27-33 exactly: the fp32 draws cast straight to e4m3 (no scale). */
void oracle_init_random_fp8(uint8_t* out, size_t n, uint64_t seed, float mean, float stddev);
/* Per-tensor quantiser of the benchmark configs: scale = amax/448 (fp32),
 * q = e4m3(x / scale).  Returns the scale; an all-zero tensor gets scale 1. */
float oracle_quantize_e4m3(const float* x, size_t n, uint8_t* q);
/* Delayed scaling: q = e4m3(x / scale) with the scale given; returns amax(|x|) (NaNs ignored). */
float oracle_quantize_e4m3_with_scale(const float* x, size_t n, float scale, uint8_t* q);
/* Draw + quantise in one pass: N(mean, stddev) from mt19937(seed), then
 * oracle_quantize_e4m3.  Returns the scale. */
float oracle_make_quantized(uint8_t* q, size_t n, uint64_t seed, float mean, float stddev);

/* The reference CPU GEMM (test.cpp:19-30) with the per-tensor scale factor added:
 *   C[row][col] = bf16_rne((scale_a*scale_b) * sum_k float(A[row][k]) * float(B[col][k]))
 * A is M x K row-major e4m3, B is N x K row-major e4m3 (the reference's B_T), C is
 * M x N row-major bf16 bits.  The k sum runs sequentially in fp32, as in the
 * reference.  Rows [row_begin, row_end) only, so a test can check a subset of rows.
 * nthreads <= 0 uses OpenMP's default. */
void oracle_gemm_rows(const uint8_t* A, const uint8_t* B, uint16_t* C, int M, int N, int K,
                      float scale_a, float scale_b, int row_begin, int row_end, int nthreads);
/* The reference's own loop nest (test.cpp:19-30): OpenMP collapse(2) over (row,
 * col), one scalar accumulator per element, rows [row_begin, row_end), written to
 * C_rows ((row_end - row_begin) x N).  Same bits as oracle_gemm_rows, slower; this is
 * what the CPU baseline times. */
void oracle_gemm_naive_rows(const uint8_t* A, const uint8_t* B, uint16_t* C_rows, int M, int N, int K,
                            float scale_a, float scale_b, int row_begin, int row_end, int nthreads);
/* The n-th (1-based) output of std::mt19937(seed); the C++ standard's known answer is
 * oracle_mt19937_nth(5489, 10000) == 4123659995. */
uint32_t oracle_mt19937_nth(uint32_t seed, uint64_t n);
/* Whole matrix. */
void oracle_gemm(const uint8_t* A, const uint8_t* B, uint16_t* C, int M, int N, int K,
                 float scale_a, float scale_b, int nthreads);
/* Chosen rows only: C_rows is len(rows) x N. */
void oracle_gemm_row_list(const uint8_t* A, const uint8_t* B, uint16_t* C_rows, int N, int K,
                          float scale_a, float scale_b, const int* rows, int nrows, int nthreads);

/* Validator (test.cpp:32-47) with the tolerance made symmetric:
 * mismatch when |c - ref| > rtol*|ref| + atol, or either value is NaN.
 * Unlike the reference it does not stop at the first mismatch: it returns the
 * number of mismatches and writes the first one's index to *first_bad (or -1). */
int64_t oracle_validate(const uint16_t* C, const uint16_t* C_ref, int64_t n, float rtol, float atol,
                        int64_t* first_bad);

/* The reference validator exactly as written (test.cpp:32-47): signed threshold
 * `diff > c_ref*0.01`, stops at the first mismatch.  Returns 1 when it passes. */
int oracle_validate_reference(const uint16_t* C, const uint16_t* C_ref, int M, int N);

/* OCP MX v1.0 e4m3 quantisation with an e8m0 scale per 32 elements of a row: X =
 * floor(log2(amax)) - 8 clamped to [-127, 127] (-127 for a zero block), scale byte X + 127,
 * q = e4m3(x * 2^-X).  x and q: rows x K (K % 32 == 0); sf: rows x K/32. */
void oracle_quantize_mx_e4m3(const float* x, int rows, int K, uint8_t* q, uint8_t* sf);
/* Block-scaled GEMM rows [row_begin, row_end) into C_rows, sequential fp32 accumulation of
 * A*2^(ea-127) * B*2^(eb-127), then bf16_rne((scale_a*scale_b) * acc); SFA, SFB row-major. */
void oracle_gemm_mx_rows(const uint8_t* A, const uint8_t* B, const uint8_t* SFA, const uint8_t* SFB, uint16_t* C_rows,
                         int N, int K, float scale_a, float scale_b, int row_begin, int row_end, int nthreads);

/* Threads OpenMP would use. */
int oracle_max_threads(void);

#ifdef __cplusplus
}
#endif
#endif
