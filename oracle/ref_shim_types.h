// TEST INFRASTRUCTURE: the prelude of oracle/_ref/libref_cpu.so, the reference's own CPU code
// compiled on the host without ROCm.
//
// The recipe (oracle/Makefile, target `ref`) feeds g++ this file, then the reference's
// gemm_cpu and validate_matrix (test.cpp:19-47) and init_random (utils.hpp:27-33) exactly as
// they stand in the reference's files, then ref_shim_exports.h.  Everything else in those
// two files is HIP host or device code that g++ cannot compile, and is left out.
//
// The reference takes its element types from ROCm (fp8_4wave.hpp:15-16):
//   fp8  = __hip_fp8_e4m3  (hip/hip_fp8.h)
//   bf16 = __hip_bfloat16  (hip/hip_bfloat16.h)
// ROCm is a dependency the reference does not vendor; .devcontainer/devcontainer.json:3 pins
// its image to ROCm 7.2.2.  The two types below restate the published behaviour of those
// types' host conversions, which are all that gemm_cpu, validate_matrix and init_random use:
//   * float -> e4m3: OCP FP8 E4M3 (bias 7, no infinities, S.1111.111 = NaN), round to
//     nearest even, saturating to +-448 (ROCm's default __HIP_SATFINITE); NaN -> NaN.
//   * e4m3 -> float: exact.
//   * float -> bf16: round to nearest even on the upper 16 bits; a NaN stays a NaN.
//   * bf16 -> float: exact (the bits shifted up by 16).
// They are written independently of liboracle.so (oracle.cpp), so that the comparison of the
// two libraries checks one restatement of the conversions against another, and the loop nests
// (the reference's own text here) against the oracle's.

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>

#include <omp.h>

namespace refshim {

inline uint32_t f32_bits(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    return u;
}

inline float f32_from_bits(uint32_t u) {
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

// OCP E4M3 value of code b: (-1)^s * 2^(e-7) * (1 + m/8) for e > 0, (-1)^s * 2^-6 * m/8 for e = 0.
inline float e4m3_to_float(uint8_t b) {
    const uint32_t e = (b >> 3) & 0xFu, m = b & 0x7u;
    const float sign = (b & 0x80u) ? -1.0f : 1.0f;
    if (e == 0xFu && m == 0x7u) return std::nanf("");
    if (e == 0) return sign * std::ldexp(static_cast<float>(m), -9);
    return sign * std::ldexp(static_cast<float>(8u + m), static_cast<int>(e) - 10);
}

// Nearest E4M3 code by search over the 127 non-negative finite codes, ties to the even code.
inline uint8_t float_to_e4m3(float x) {
    if (std::isnan(x)) return 0x7F;
    const uint8_t sign = std::signbit(x) ? 0x80 : 0x00;
    const double a = std::fabs(static_cast<double>(x));
    if (a >= 448.0) return static_cast<uint8_t>(sign | 0x7E);  // satfinite: +-448, infinities included
    // Codes 0x00..0x7E are ordered by value; find the pair around a.
    int lo = 0, hi = 0x7E;
    while (hi - lo > 1) {
        const int mid = (lo + hi) / 2;
        if (static_cast<double>(e4m3_to_float(static_cast<uint8_t>(mid))) <= a) lo = mid; else hi = mid;
    }
    const double vlo = e4m3_to_float(static_cast<uint8_t>(lo)), vhi = e4m3_to_float(static_cast<uint8_t>(hi));
    int pick;
    if (a - vlo < vhi - a) pick = lo;
    else if (a - vlo > vhi - a) pick = hi;
    else pick = (lo & 1) ? hi : lo;  // a tie: the code with an even mantissa
    return static_cast<uint8_t>(sign | pick);
}

inline uint16_t float_to_bf16(float f) {
    uint32_t u = f32_bits(f);
    if ((u & 0x7F800000u) != 0x7F800000u) {
        u += 0x7FFFu + ((u >> 16) & 1u);  // round to nearest, ties to even
    } else if (u & 0xFFFFu) {
        u |= 0x10000u;  // a NaN whose payload sits in the dropped bits stays a NaN
    }
    return static_cast<uint16_t>(u >> 16);
}

// The 256 decoded values, so that the reference's inner loop (two conversions per product)
// is timed at table-lookup speed rather than at the speed of the arithmetic above.
struct E4m3Table {
    float v[256];
    E4m3Table() {
        for (int b = 0; b < 256; ++b) v[b] = e4m3_to_float(static_cast<uint8_t>(b));
    }
};
inline const E4m3Table kE4m3Table;

}  // namespace refshim

struct fp8 {
    uint8_t bits;
    fp8() = default;
    explicit fp8(float x) : bits(refshim::float_to_e4m3(x)) {}
    explicit operator float() const { return refshim::kE4m3Table.v[bits]; }
};

struct bf16 {
    uint16_t bits;
    bf16() = default;
    explicit bf16(float x) : bits(refshim::float_to_bf16(x)) {}
    explicit operator float() const { return refshim::f32_from_bits(static_cast<uint32_t>(bits) << 16); }
};

static_assert(sizeof(fp8) == 1 && sizeof(bf16) == 2, "the element types are the raw bytes and bits");
