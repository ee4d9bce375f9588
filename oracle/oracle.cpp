// CPU oracle for the FP8 e4m3 TN GEMM — TEST INFRASTRUCTURE ONLY (see oracle.h).
//
// Restates nirw4nna/hipgemm test.cpp:19-47 and utils.hpp:27-33 in portable C++.
// Pinned bit for bit to the reference's own gemm_cpu, validate_matrix and init_random,
// compiled from its sources (oracle/_ref, see oracle.h).  Build with -ffp-contract=off and without -ffast-math so
// the k-sum keeps the reference's sequential fp32 order.
#include "oracle.h"

#include <cmath>
#include <cstring>
#include <random>
#include <vector>
#include <algorithm>
#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

// ---- OCP FP8 E4M3 ("fn") ------------------------------------------------------------
// 1 sign bit, 4 exponent bits (bias 7), 3 mantissa bits.  No infinities; S.1111.111 is
// NaN; the largest finite value is S.1111.110 = 1.75 * 2^8 = 448.  Subnormals have
// exponent field 0 and value mantissa * 2^-9.

struct DecodeTable {
    float v[256];
    DecodeTable() {
        for (int b = 0; b < 256; ++b) {
            const int sign = b >> 7, e = (b >> 3) & 0xF, m = b & 7;
            float mag;
            if (e == 0xF && m == 7) {
                mag = NAN;
            } else if (e == 0) {
                mag = std::ldexp(float(m), -9);
            } else {
                mag = std::ldexp(1.0f + float(m) / 8.0f, e - 7);
            }
            v[b] = sign ? -mag : mag;
        }
    }
};
const DecodeTable kDecode;

inline uint8_t encode_e4m3(float x) {
    uint32_t bits;
    std::memcpy(&bits, &x, 4);
    const uint8_t sign = uint8_t((bits >> 24) & 0x80);
    if (std::isnan(x)) return uint8_t(sign | 0x7F);
    float a = std::fabs(x);
    // Saturate-to-finite: every magnitude that would round above 448 (including inf)
    // becomes 448.  Values in [448, 464] round to 448 under RNE anyway (464 is the tie
    // between 448 = mantissa 110 and the NaN slot 111; the tie goes to the even code).
    if (a >= 448.0f) return uint8_t(sign | 0x7E);
    if (a < std::ldexp(1.0f, -6)) {
        // Subnormal range: quantum 2^-9.  q in [0, 8]; q == 8 is the smallest normal,
        // whose code (exponent 1, mantissa 0) is also 8.
        const float q = std::nearbyint(std::ldexp(a, 9));  // exact scaling, RNE
        return uint8_t(sign | uint8_t(q));
    }
    int e;
    std::frexp(a, &e);  // a = f * 2^e, f in [0.5, 1)  =>  unbiased exponent e-1
    const int ue = e - 1;
    float q = std::nearbyint(std::ldexp(a, 3 - ue));  // in [8, 16]
    int ee = ue;
    if (q >= 16.0f) { q = 8.0f; ee += 1; }
    const int code = ((ee + 7) << 3) | (int(q) - 8);
    // ee + 7 <= 15 and code <= 0x7E here because a < 448.
    return uint8_t(sign | uint8_t(code));
}

inline uint16_t bf16_rne(float x) {
    uint32_t bits;
    std::memcpy(&bits, &x, 4);
    if (std::isnan(x)) return uint16_t(((bits >> 16) & 0x8000) | 0x7FC0);
    const uint32_t lsb = (bits >> 16) & 1u;
    bits += 0x7FFFu + lsb;
    return uint16_t(bits >> 16);
}

inline float bf16_to_f32(uint16_t b) {
    const uint32_t bits = uint32_t(b) << 16;
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

inline int resolve_threads(int nthreads) {
#ifdef _OPENMP
    return nthreads > 0 ? nthreads : omp_get_max_threads();
#else
    (void)nthreads;
    return 1;
#endif
}

// One output element exactly as test.cpp:22-27 computes it, plus the scale.
inline uint16_t dot_element(const uint8_t* a_row, const uint8_t* b_row, int K, float s) {
    float acc = 0.0f;
    for (int k = 0; k < K; ++k) acc += kDecode.v[a_row[k]] * kDecode.v[b_row[k]];
    return bf16_rne(s * acc);
}

constexpr int kColBlock = 32;

// Same per-element arithmetic as dot_element (one fp32 accumulator per element, k
// ascending, product then add), but kColBlock columns advance together so the
// compiler can keep independent accumulators in vector registers.  The products of
// two e4m3 values are exact in fp32, so each element's sum is bit-identical to the
// scalar loop.
void gemm_block(const uint8_t* A, const uint8_t* B, uint16_t* C, int ldc, int N, int K, float s,
                const int* rows, int nrows, int col0, std::vector<float>& bt, std::vector<float>& arow) {
    const int nc = std::min(kColBlock, N - col0);
    bt.assign(size_t(K) * kColBlock, 0.0f);
    for (int j = 0; j < nc; ++j) {
        const uint8_t* b = B + size_t(col0 + j) * K;
        for (int k = 0; k < K; ++k) bt[size_t(k) * kColBlock + j] = kDecode.v[b[k]];
    }
    arow.resize(K);
    for (int r = 0; r < nrows; ++r) {
        const uint8_t* a = A + size_t(rows[r]) * K;
        for (int k = 0; k < K; ++k) arow[k] = kDecode.v[a[k]];
        float acc[kColBlock];
        for (int j = 0; j < kColBlock; ++j) acc[j] = 0.0f;
        const float* btp = bt.data();
        for (int k = 0; k < K; ++k) {
            const float av = arow[k];
            const float* bk = btp + size_t(k) * kColBlock;
#pragma GCC ivdep
            for (int j = 0; j < kColBlock; ++j) acc[j] += av * bk[j];
        }
        uint16_t* c = C + size_t(r) * ldc + col0;
        for (int j = 0; j < nc; ++j) c[j] = bf16_rne(s * acc[j]);
    }
}

void gemm_rows_impl(const uint8_t* A, const uint8_t* B, uint16_t* C, int ldc, int N, int K, float s,
                    const int* rows, int nrows, int nthreads) {
    const int nblk = (N + kColBlock - 1) / kColBlock;
    const int nt = resolve_threads(nthreads);
    (void)nt;
#pragma omp parallel num_threads(nt)
    {
        std::vector<float> bt, arow;
#pragma omp for schedule(dynamic, 1)
        for (int cb = 0; cb < nblk; ++cb)
            gemm_block(A, B, C, ldc, N, K, s, rows, nrows, cb * kColBlock, bt, arow);
    }
}

}  // namespace

extern "C" {

uint8_t oracle_fp8_encode(float x) { return encode_e4m3(x); }
void oracle_fp8_encode_array(const float* x, size_t n, uint8_t* out) {
    for (size_t i = 0; i < n; ++i) out[i] = encode_e4m3(x[i]);
}
void oracle_bf16_rne_array(const float* x, size_t n, uint16_t* out) {
    for (size_t i = 0; i < n; ++i) out[i] = bf16_rne(x[i]);
}
float oracle_fp8_decode(uint8_t b) { return kDecode.v[b]; }
uint16_t oracle_bf16_rne(float x) { return bf16_rne(x); }
float oracle_bf16_to_float(uint16_t b) { return bf16_to_f32(b); }

void oracle_normal_f32(float* out, size_t n, uint64_t seed, float mean, float stddev) {
    std::mt19937 gen(static_cast<std::mt19937::result_type>(seed));
    std::normal_distribution<float> dis(mean, stddev);
    for (size_t i = 0; i < n; ++i) out[i] = dis(gen);
}

void oracle_init_random_fp8(uint8_t* out, size_t n, uint64_t seed, float mean, float stddev) {
    std::mt19937 gen(static_cast<std::mt19937::result_type>(seed));
    std::normal_distribution<float> dis(mean, stddev);
    for (size_t i = 0; i < n; ++i) out[i] = encode_e4m3(dis(gen));
}

float oracle_quantize_e4m3(const float* x, size_t n, uint8_t* q) {
    float amax = 0.0f;
    for (size_t i = 0; i < n; ++i) amax = std::max(amax, std::fabs(x[i]));
    const float scale = amax > 0.0f ? amax / 448.0f : 1.0f;
    for (size_t i = 0; i < n; ++i) q[i] = encode_e4m3(x[i] / scale);
    return scale;
}

float oracle_quantize_e4m3_with_scale(const float* x, size_t n, float scale, uint8_t* q) {
    float amax = 0.0f;
    for (size_t i = 0; i < n; ++i) {
        amax = std::max(amax, std::fabs(x[i]));
        q[i] = encode_e4m3(x[i] / scale);
    }
    return amax;
}

float oracle_make_quantized(uint8_t* q, size_t n, uint64_t seed, float mean, float stddev) {
    std::vector<float> x(n);
    oracle_normal_f32(x.data(), n, seed, mean, stddev);
    return oracle_quantize_e4m3(x.data(), n, q);
}

void oracle_gemm_rows(const uint8_t* A, const uint8_t* B, uint16_t* C, int M, int N, int K,
                      float scale_a, float scale_b, int row_begin, int row_end, int nthreads) {
    (void)M;
    if (row_end <= row_begin || N <= 0) return;
    const float s = scale_a * scale_b;
    std::vector<int> rows(row_end - row_begin);
    for (int i = 0; i < row_end - row_begin; ++i) rows[i] = row_begin + i;
    gemm_rows_impl(A, B, C + size_t(row_begin) * N, N, N, K, s, rows.data(), int(rows.size()), nthreads);
}

void oracle_gemm(const uint8_t* A, const uint8_t* B, uint16_t* C, int M, int N, int K,
                 float scale_a, float scale_b, int nthreads) {
    oracle_gemm_rows(A, B, C, M, N, K, scale_a, scale_b, 0, M, nthreads);
}

void oracle_gemm_row_list(const uint8_t* A, const uint8_t* B, uint16_t* C_rows, int N, int K,
                          float scale_a, float scale_b, const int* rows, int nrows, int nthreads) {
    if (nrows <= 0 || N <= 0) return;
    gemm_rows_impl(A, B, C_rows, N, N, K, scale_a * scale_b, rows, nrows, nthreads);
}

// The reference's loop nest itself (test.cpp:19-30): OpenMP collapse(2) over
// (row, col), one scalar fp32 accumulator per element.  This is the timed CPU
// baseline; oracle_gemm_rows computes the same bits faster for the tests.
void oracle_gemm_naive_rows(const uint8_t* A, const uint8_t* B, uint16_t* C, int M, int N, int K,
                            float scale_a, float scale_b, int row_begin, int row_end, int nthreads) {
    (void)M;
    const float s = scale_a * scale_b;
    const int nt = resolve_threads(nthreads);
    (void)nt;
#pragma omp parallel for collapse(2) num_threads(nt)
    for (int row = row_begin; row < row_end; ++row) {
        for (int col = 0; col < N; ++col) {
            C[size_t(row - row_begin) * N + col] = dot_element(A + size_t(row) * K, B + size_t(col) * K, K, s);
        }
    }
}

uint32_t oracle_mt19937_nth(uint32_t seed, uint64_t n) {
    std::mt19937 gen(seed);
    uint32_t v = 0;
    for (uint64_t i = 0; i < n; ++i) v = static_cast<uint32_t>(gen());
    return v;
}

int64_t oracle_validate(const uint16_t* C, const uint16_t* C_ref, int64_t n, float rtol, float atol,
                        int64_t* first_bad) {
    int64_t bad = 0, first = -1;
    for (int64_t i = 0; i < n; ++i) {
        const float c = bf16_to_f32(C[i]);
        const float r = bf16_to_f32(C_ref[i]);
        const float diff = std::fabs(c - r);
        if (std::isnan(c) || std::isnan(r) || diff > rtol * std::fabs(r) + atol) {
            if (first < 0) first = i;
            ++bad;
        }
    }
    if (first_bad) *first_bad = first;
    return bad;
}

int oracle_validate_reference(const uint16_t* C, const uint16_t* C_ref, int M, int N) {
    bool success = true;
    for (int row = 0; row < M && success; ++row) {
        for (int col = 0; col < N && success; ++col) {
            const float c_val = bf16_to_f32(C[size_t(row) * N + col]);
            const float c_ref_val = bf16_to_f32(C_ref[size_t(row) * N + col]);
            const float diff = std::fabs(c_val - c_ref_val);
            const float threshold = c_ref_val * 0.01f;
            if (diff > threshold || std::isnan(c_val) || std::isnan(c_ref_val)) success = false;
        }
    }
    return success ? 1 : 0;
}

int oracle_max_threads(void) { return resolve_threads(0); }

// ---- MX block scaling ---------------------------------------------------------------------

// OCP Microscaling Formats (MX) v1.0, e4m3 elements, e8m0 shared scale per 32 elements of a
// row: X = floor(log2(max |x|)) - 8 (8 is e4m3's largest exponent), clamped to [-127, 127],
// with X = -127 for an all-zero block; scale byte = X + 127; element = e4m3(x * 2^-X),
// round-to-nearest-even, saturating to +-448.
void oracle_quantize_mx_e4m3(const float* x, int rows, int K, uint8_t* q, uint8_t* sf) {
    const int groups = K / 32;
    for (int r = 0; r < rows; ++r) {
        for (int g = 0; g < groups; ++g) {
            const float* v = x + size_t(r) * K + size_t(g) * 32;
            float amax = 0.0f;
            for (int i = 0; i < 32; ++i) amax = std::max(amax, std::fabs(v[i]));
            int X = -127;
            if (amax > 0.0f && std::isfinite(amax)) {
                int e;
                std::frexp(amax, &e);  // amax = f * 2^e, f in [0.5, 1): floor(log2(amax)) = e - 1
                X = std::min(127, std::max(-127, (e - 1) - 8));
            }
            sf[size_t(r) * groups + g] = uint8_t(X + 127);
            for (int i = 0; i < 32; ++i) q[size_t(r) * K + size_t(g) * 32 + i] = encode_e4m3(std::ldexp(v[i], -X));
        }
    }
}

// The block-scaled product in the reference's loop order (test.cpp:19-30): per element one
// fp32 accumulator, k ascending, each term A*2^(ea-127) * B*2^(eb-127) (exact in fp32 for
// scales inside its range), then bf16_rne((scale_a*scale_b) * acc).  SFA / SFB row-major,
// K/32 bytes per row; a scale byte of 255 is NaN.
void oracle_gemm_mx_rows(const uint8_t* A, const uint8_t* B, const uint8_t* SFA, const uint8_t* SFB, uint16_t* C_rows,
                         int N, int K, float scale_a, float scale_b, int row_begin, int row_end, int nthreads) {
    const int groups = K / 32;
    const float s = scale_a * scale_b;
    const int nt = resolve_threads(nthreads);
    (void)nt;
    auto scaled = [](uint8_t v, uint8_t e) {
        return e == 255 ? NAN : std::ldexp(kDecode.v[v], int(e) - 127);
    };
#pragma omp parallel num_threads(nt)
    {
        std::vector<float> bt, arow(K);
#pragma omp for schedule(dynamic, 1)
        for (int cb = 0; cb < (N + kColBlock - 1) / kColBlock; ++cb) {
            const int col0 = cb * kColBlock, nc = std::min(kColBlock, N - col0);
            bt.assign(size_t(K) * kColBlock, 0.0f);
            for (int j = 0; j < nc; ++j) {
                const uint8_t* b = B + size_t(col0 + j) * K;
                const uint8_t* eb = SFB + size_t(col0 + j) * groups;
                for (int k = 0; k < K; ++k) bt[size_t(k) * kColBlock + j] = scaled(b[k], eb[k / 32]);
            }
            for (int r = row_begin; r < row_end; ++r) {
                const uint8_t* a = A + size_t(r) * K;
                const uint8_t* ea = SFA + size_t(r) * groups;
                for (int k = 0; k < K; ++k) arow[k] = scaled(a[k], ea[k / 32]);
                float acc[kColBlock];
                for (int j = 0; j < kColBlock; ++j) acc[j] = 0.0f;
                for (int k = 0; k < K; ++k) {
                    const float av = arow[k];
                    const float* bk = bt.data() + size_t(k) * kColBlock;
#pragma GCC ivdep
                    for (int j = 0; j < kColBlock; ++j) acc[j] += av * bk[j];
                }
                uint16_t* c = C_rows + size_t(r - row_begin) * N + col0;
                for (int j = 0; j < nc; ++j) c[j] = bf16_rne(s * acc[j]);
            }
        }
    }
}

}  // extern "C"
