// Per-tensor FP8 e4m3 quantiser on the device: the step before the GEMM for real
// activations and weights.  scale = amax(|x|) / 448 (1 for an all-zero tensor) and
// q[i] = e4m3(x[i] / scale), with IEEE round-to-nearest division and CUDA's
// saturate-to-finite, round-to-nearest-even e4m3 conversion.  That is the benchmark
// configs' quantiser, which the reference applies on the host without a scale
// (utils.hpp:27-33 casts N(-1, 1) draws straight to fp8).
//
// HBM-bound: one pass reads x for the amax, a second reads x again and writes q
// (fp32: 9 bytes moved per element, bf16: 5).  Loads and stores are 16 bytes wide.
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "hipgemm_b200.h"

namespace hgq {

constexpr int kThreads = 256;

__device__ __forceinline__ float load_as_float(const float* x, size_t i) { return x[i]; }
__device__ __forceinline__ float load_as_float(const __nv_bfloat16* x, size_t i) { return __bfloat162float(x[i]); }

// 16 bytes of input as floats: 4 fp32 or 8 bf16.
template <typename T>
struct Vec;
template <>
struct Vec<float> {
    static constexpr int kElems = 4;
    __device__ static void load(const float* x, size_t v, float (&out)[4]) {
        const float4 f = __ldg(reinterpret_cast<const float4*>(x) + v);
        out[0] = f.x;
        out[1] = f.y;
        out[2] = f.z;
        out[3] = f.w;
    }
};
template <>
struct Vec<__nv_bfloat16> {
    static constexpr int kElems = 8;
    __device__ static void load(const __nv_bfloat16* x, size_t v, float (&out)[8]) {
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(x) + v);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            out[2 * i] = __uint_as_float(w[i] << 16);
            out[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
        }
    }
};

// amax(|x|) into *amax_bits (the float's bits; non-negative floats order like their
// bits, so an integer atomicMax is exact).  NaN elements are ignored, as std::max of
// the host restatement ignores them.
template <typename T>
__global__ void __launch_bounds__(kThreads) amax_kernel(const T* __restrict__ x, size_t n,
                                                        unsigned int* __restrict__ amax_bits) {
    constexpr int E = Vec<T>::kElems;
    const size_t nvec = n / E;
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    float m = 0.0f;
    for (size_t v = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < nvec; v += stride) {
        float f[E];
        Vec<T>::load(x, v, f);
#pragma unroll
        for (int i = 0; i < E; ++i) m = fmaxf(m, fabsf(f[i]));
    }
    for (size_t i = nvec * E + static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
        m = fmaxf(m, fabsf(load_as_float(x, i)));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    __shared__ float warp_max[kThreads / 32];
    if ((threadIdx.x & 31) == 0) warp_max[threadIdx.x / 32] = m;
    __syncthreads();
    if (threadIdx.x < 32) {
        m = threadIdx.x < kThreads / 32 ? warp_max[threadIdx.x] : 0.0f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (threadIdx.x == 0) atomicMax(amax_bits, __float_as_uint(m));
    }
}

__device__ __forceinline__ float scale_from_amax(unsigned int bits) {
    const float amax = __uint_as_float(bits);
    return amax > 0.0f ? __fdiv_rn(amax, 448.0f) : 1.0f;
}

__device__ __forceinline__ uint32_t e4m3x2(float lo, float hi) {
    return static_cast<uint32_t>(__nv_cvt_float2_to_fp8x2(make_float2(lo, hi), __NV_SATFINITE, __NV_E4M3));
}

// q = e4m3(x / scale): 16 elements (16 output bytes) per thread and step.  The sweep runs
// from the end of x to its start: the amax pass swept forwards, so the part of x it read
// last is still in L2 when this pass starts (measured on B200, both passes over one 8192 x 8192
// fp32 tensor, back to back: 105.5 us per call forwards, 98.6 us backwards; every element's
// result is the same either way).
template <typename T>
__global__ void __launch_bounds__(kThreads) quantize_kernel(const T* __restrict__ x, size_t n,
                                                             const unsigned int* __restrict__ amax_bits,
                                                             uint8_t* __restrict__ q) {
    constexpr int E = Vec<T>::kElems;
    constexpr int LOADS = 16 / E;
    const float s = scale_from_amax(*amax_bits);
    const size_t ngroups = n / 16;
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t g0 = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; g0 < ngroups; g0 += stride) {
        const size_t g = ngroups - 1 - g0;
        float f[16];
#pragma unroll
        for (int l = 0; l < LOADS; ++l) {
            float t[E];
            Vec<T>::load(x, g * LOADS + l, t);
#pragma unroll
            for (int i = 0; i < E; ++i) f[l * E + i] = __fdiv_rn(t[i], s);
        }
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) w[i] = e4m3x2(f[4 * i], f[4 * i + 1]) | (e4m3x2(f[4 * i + 2], f[4 * i + 3]) << 16);
        reinterpret_cast<uint4*>(q)[g] = make_uint4(w[0], w[1], w[2], w[3]);
    }
    for (size_t i = ngroups * 16 + static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
        q[i] = static_cast<uint8_t>(e4m3x2(__fdiv_rn(load_as_float(x, i), s), 0.0f) & 0xFFu);
    }
}

// Delayed scaling in one pass: q = e4m3(x / scale_in) with a scale the caller carries over
// (from the previous step's amax, as FP8 training and serving loops do), and amax(|x|) of
// this tensor accumulated into *amax_bits for the next step.  16 elements per thread and
// step, one atomicMax per block.
template <typename T>
__global__ void __launch_bounds__(kThreads) quantize_delayed_kernel(const T* __restrict__ x, size_t n,
                                                                     const float* __restrict__ scale_in,
                                                                     uint8_t* __restrict__ q,
                                                                     unsigned int* __restrict__ amax_bits) {
    constexpr int E = Vec<T>::kElems;
    constexpr int LOADS = 16 / E;
    // Groups of 16 in flight per thread (all loads issued before any use): 2 for fp32, 1 for
    // bf16 (measured at 8192 x 8192: fp32 60.8 -> 58.1 us with 2; bf16 49.3 -> 63.8 us).
    constexpr int U = sizeof(T) == 4 ? 2 : 1;
    const float s = *scale_in;
    const size_t ngroups = n / 16;
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    float m = 0.0f;
    for (size_t g0 = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; g0 < ngroups; g0 += U * stride) {
        float v[U][16];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const size_t g = g0 + u * stride;
            if (g < ngroups) {
#pragma unroll
                for (int l = 0; l < LOADS; ++l) Vec<T>::load(x, g * LOADS + l, *reinterpret_cast<float(*)[E]>(&v[u][l * E]));
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const size_t g = g0 + u * stride;
            if (g >= ngroups) break;
            uint32_t w[4];
#pragma unroll
            for (int i = 0; i < 16; ++i) m = fmaxf(m, fabsf(v[u][i]));
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                w[i] = e4m3x2(__fdiv_rn(v[u][4 * i], s), __fdiv_rn(v[u][4 * i + 1], s)) |
                       (e4m3x2(__fdiv_rn(v[u][4 * i + 2], s), __fdiv_rn(v[u][4 * i + 3], s)) << 16);
            }
            reinterpret_cast<uint4*>(q)[g] = make_uint4(w[0], w[1], w[2], w[3]);
        }
    }
    for (size_t i = ngroups * 16 + static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
        const float v = load_as_float(x, i);
        m = fmaxf(m, fabsf(v));
        q[i] = static_cast<uint8_t>(e4m3x2(__fdiv_rn(v, s), 0.0f) & 0xFFu);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    __shared__ float warp_max[kThreads / 32];
    if ((threadIdx.x & 31) == 0) warp_max[threadIdx.x / 32] = m;
    __syncthreads();
    if (threadIdx.x < 32) {
        m = threadIdx.x < kThreads / 32 ? warp_max[threadIdx.x] : 0.0f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (threadIdx.x == 0) atomicMax(amax_bits, __float_as_uint(m));
    }
}

// Turns the accumulated amax bits into the scale, in place.
__global__ void finalize_scale_kernel(unsigned int* amax_bits) {
    const float s = scale_from_amax(*amax_bits);
    *reinterpret_cast<float*>(amax_bits) = s;
}

// Grid for a grid-stride kernel: enough blocks for the work, at most one full wave of
// resident blocks (the kernel's occupancy x SMs), so no partial second wave trails.
template <typename Kernel>
int grid_for(Kernel kernel, size_t work_items) {
    static int per_sm = 0;  // per kernel instantiation; the same on every sm_100 device
    if (per_sm == 0) {
        int b = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, kernel, kThreads, 0) != cudaSuccess || b < 1) b = 1;
        per_sm = b;
    }
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const size_t blocks = (work_items + kThreads - 1) / kThreads;
    const size_t cap = static_cast<size_t>(sms) * per_sm;
    return static_cast<int>(blocks < 1 ? 1 : (blocks > cap ? cap : blocks));
}

template <typename T>
int run(const T* x, size_t n, uint8_t* q, float* d_scale, cudaStream_t stream) {
    unsigned int* acc = reinterpret_cast<unsigned int*>(d_scale);
    if (cudaMemsetAsync(acc, 0, sizeof(unsigned int), stream) != cudaSuccess) return HGEMM_ERR_CUDA;
    if (n > 0) {
        amax_kernel<T><<<grid_for(amax_kernel<T>, n / Vec<T>::kElems + 1), kThreads, 0, stream>>>(x, n, acc);
        quantize_kernel<T><<<grid_for(quantize_kernel<T>, n / 16 + 1), kThreads, 0, stream>>>(x, n, acc, q);
    }
    finalize_scale_kernel<<<1, 1, 0, stream>>>(acc);
    return cudaGetLastError() == cudaSuccess ? HGEMM_OK : HGEMM_ERR_CUDA;
}

// ---- OCP MX e4m3 quantiser: one e8m0 scale per 32 consecutive elements of a row --------
//
// X = floor(log2(amax)) - 8 (e4m3's largest binade), clamped to [-127, 127]; -127 when amax
// is 0, subnormal (then floor(log2) <= -127 anyway) or infinite; NaN elements do not count
// toward amax.  Scale byte X + 127; q = e4m3_satfinite(x * 2^-X), where 2^-X is a normal
// float, so the product is the correctly rounded x * 2^-X.  Each lane loads 32 bytes (8 fp32
// or 16 bf16); the 4 or 2 lanes of a block reduce amax with shuffles and write their q bytes;
// a block's first lane writes its scale byte into the blocked layout the MX GEMM reads.
// HBM-bound: x read once, q and the scales written once.

// Per input type: 16-byte loads per chunk and chunks in flight per thread (measured at
// 8192 x 8192 on B200: fp32 4 x 2 -> 58 us, 0.88 of copy bandwidth; bf16 2 x 2 -> 43 us).
template <typename T>
struct MxTune;
template <>
struct MxTune<float> {
    static constexpr int kVecs = 2, kUnroll = 4;
};
template <>
struct MxTune<__nv_bfloat16> {
    static constexpr int kVecs = 2, kUnroll = 2;
};

// Scale exponent X of a block from its amax (non-negative or NaN-free by construction).
__device__ __forceinline__ int mx_exponent(float amax) {
    const uint32_t biased = __float_as_uint(amax) >> 23;  // amax >= 0: no sign bit
    if (biased == 0u || biased == 255u) return -127;      // zero / subnormal / infinite
    const int x = static_cast<int>(biased) - 127 - 8;
    return x < -127 ? -127 : x;                           // at most 119: no upper clamp needed
}

// Byte offset of (row, group) in the blocked scale layout: 512-byte atoms of 128 rows x 4
// groups, row r group g at 16*(r%32) + 4*((r/32)%4) + g%4, atoms K-major within a row block.
__device__ __forceinline__ size_t mx_sf_offset(uint32_t row, uint32_t group, uint32_t k_atoms) {
    const size_t atom = static_cast<size_t>(row / 128u) * k_atoms + group / 4u;
    return atom * 512 + 16u * (row % 32u) + 4u * ((row / 32u) % 4u) + (group % 4u);
}

// Chunks of kVecs 16-byte loads (E = 4 * kVecs fp32 or 8 * kVecs bf16 elements); 32 / E
// lanes share a block.
template <typename T>
struct MxChunk {
    static constexpr int kVecs = MxTune<T>::kVecs;
    static constexpr int E = Vec<T>::kElems * kVecs;
    __device__ static void load(const T* x, size_t c, float (&v)[E]) {
#pragma unroll
        for (int i = 0; i < kVecs; ++i) {
            Vec<T>::load(x, c * kVecs + i, *reinterpret_cast<float(*)[Vec<T>::kElems]>(&v[i * Vec<T>::kElems]));
        }
    }
};

template <typename T>
__global__ void __launch_bounds__(kThreads) quantize_mx_kernel(const T* __restrict__ x, size_t nchunks,
                                                                uint32_t groups, uint32_t k_atoms,
                                                                uint8_t* __restrict__ q, uint8_t* __restrict__ sf) {
    constexpr int E = MxChunk<T>::E;
    constexpr int U = MxTune<T>::kUnroll;
    constexpr uint32_t LPB = 32 / E;  // lanes per 32-element block
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    const uint32_t lane = threadIdx.x & 31u;
    // Warp-uniform trip count (the loop test uses the warp's first chunk): every lane reaches
    // the full-warp shuffles; lanes past the end load zeros and store nothing.
    for (size_t c0 = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; c0 - lane < nchunks;
         c0 += U * stride) {
        float v[U][E];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const size_t c = c0 + u * stride;
            if (c < nchunks) {
                MxChunk<T>::load(x, c, v[u]);
            } else {
#pragma unroll
                for (int i = 0; i < E; ++i) v[u][i] = 0.0f;
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const size_t c = c0 + u * stride;
            float m = 0.0f;
#pragma unroll
            for (int i = 0; i < E; ++i) m = fmaxf(m, fabsf(v[u][i]));
            // A block's lanes are an aligned group of LPB (stride % 32 == 0).
#pragma unroll
            for (uint32_t o = 1; o < LPB; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            if (c >= nchunks) continue;
            const int X = mx_exponent(m);
            const float scale = __uint_as_float(static_cast<uint32_t>(127 - X) << 23);  // 2^-X
            uint32_t w[E / 4];
#pragma unroll
            for (int i = 0; i < E / 4; ++i) {
                w[i] = e4m3x2(__fmul_rn(v[u][4 * i], scale), __fmul_rn(v[u][4 * i + 1], scale)) |
                       (e4m3x2(__fmul_rn(v[u][4 * i + 2], scale), __fmul_rn(v[u][4 * i + 3], scale)) << 16);
            }
            if constexpr (E == 4) {
                reinterpret_cast<uint32_t*>(q)[c] = w[0];
            } else if constexpr (E == 8) {
                reinterpret_cast<uint2*>(q)[c] = make_uint2(w[0], w[1]);
            } else {
#pragma unroll
                for (int i = 0; i < E / 16; ++i) {
                    reinterpret_cast<uint4*>(q)[c * (E / 16) + i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
                }
            }
            if ((lane & (LPB - 1)) == 0u) {
                // Block index < 2^32 (checked on the host): 32-bit division, not the
                // emulated 64-bit one.
                const uint32_t block = static_cast<uint32_t>(c / LPB);
                const uint32_t row = block / groups;
                sf[mx_sf_offset(row, block - row * groups, k_atoms)] = static_cast<uint8_t>(X + 127);
            }
        }
    }
}

template <typename T>
int run_mx(const T* x, int rows, int K, uint8_t* q, uint8_t* sf, cudaStream_t stream) {
    const uint32_t groups = static_cast<uint32_t>(K / 32), k_atoms = static_cast<uint32_t>((K + 127) / 128);
    if (static_cast<size_t>(rows) * groups > 0xFFFFFFFFull) return HGEMM_ERR_UNSUPPORTED;  // >= 2^32 blocks
    const size_t sf_bytes = static_cast<size_t>((rows + 127) / 128) * k_atoms * 512;
    // Padding entries (rows past `rows`, groups past K/32) get 127 = 2^0.
    if (cudaMemsetAsync(sf, 127, sf_bytes, stream) != cudaSuccess) return HGEMM_ERR_CUDA;
    const size_t nchunks = static_cast<size_t>(rows) * K / MxChunk<T>::E;
    const int grid = grid_for(quantize_mx_kernel<T>, (nchunks + MxTune<T>::kUnroll - 1) / MxTune<T>::kUnroll);
    quantize_mx_kernel<T><<<grid, kThreads, 0, stream>>>(x, nchunks, groups, k_atoms, q, sf);
    return cudaGetLastError() == cudaSuccess ? HGEMM_OK : HGEMM_ERR_CUDA;
}

template <typename T>
int run_delayed(const T* x, size_t n, const float* scale_in, uint8_t* q, float* amax_out, cudaStream_t stream) {
    unsigned int* acc = reinterpret_cast<unsigned int*>(amax_out);
    if (cudaMemsetAsync(acc, 0, sizeof(unsigned int), stream) != cudaSuccess) return HGEMM_ERR_CUDA;
    if (n > 0) {
        quantize_delayed_kernel<T><<<grid_for(quantize_delayed_kernel<T>, n / (sizeof(T) == 4 ? 32 : 16) + 1), kThreads,
                                     0, stream>>>(
            x, n, scale_in, q, acc);
    }
    return cudaGetLastError() == cudaSuccess ? HGEMM_OK : HGEMM_ERR_CUDA;
}

}  // namespace hgq

extern "C" int hgemm_quantize_e4m3_delayed(const void* x, int x_dtype, size_t n, void* q, const float* d_scale_in,
                                           float* d_amax_out, hgemm_stream_t stream) {
    if (!d_scale_in || !d_amax_out || (n > 0 && (!x || !q))) return HGEMM_ERR_INVALID_VALUE;
    if (x_dtype != HGEMM_DTYPE_F32 && x_dtype != HGEMM_DTYPE_BF16) return HGEMM_ERR_INVALID_VALUE;
    if ((reinterpret_cast<uintptr_t>(x) & 15u) || (reinterpret_cast<uintptr_t>(q) & 15u) ||
        (reinterpret_cast<uintptr_t>(d_scale_in) & 3u) || (reinterpret_cast<uintptr_t>(d_amax_out) & 3u)) {
        return HGEMM_ERR_ALIGNMENT;
    }
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    uint8_t* const out = static_cast<uint8_t*>(q);
    if (x_dtype == HGEMM_DTYPE_F32) return hgq::run_delayed(static_cast<const float*>(x), n, d_scale_in, out, d_amax_out, s);
    return hgq::run_delayed(static_cast<const __nv_bfloat16*>(x), n, d_scale_in, out, d_amax_out, s);
}

extern "C" int hgemm_quantize_mx_e4m3(const void* x, int x_dtype, int rows, int K, void* q, void* sf_blocked,
                                      hgemm_stream_t stream) {
    if (rows < 0 || K < 0) return HGEMM_ERR_INVALID_VALUE;
    if (x_dtype != HGEMM_DTYPE_F32 && x_dtype != HGEMM_DTYPE_BF16) return HGEMM_ERR_INVALID_VALUE;
    if (K % 32 != 0) return HGEMM_ERR_ALIGNMENT;
    if (rows == 0 || K == 0) return HGEMM_OK;
    if (!x || !q || !sf_blocked) return HGEMM_ERR_INVALID_VALUE;
    if ((reinterpret_cast<uintptr_t>(x) & 15u) || (reinterpret_cast<uintptr_t>(q) & 15u)) return HGEMM_ERR_ALIGNMENT;
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    uint8_t* const qb = static_cast<uint8_t*>(q);
    uint8_t* const sf = static_cast<uint8_t*>(sf_blocked);
    if (x_dtype == HGEMM_DTYPE_F32) return hgq::run_mx(static_cast<const float*>(x), rows, K, qb, sf, s);
    return hgq::run_mx(static_cast<const __nv_bfloat16*>(x), rows, K, qb, sf, s);
}

extern "C" int hgemm_quantize_e4m3(const void* x, int x_dtype, size_t n, void* q, float* d_scale,
                                   hgemm_stream_t stream) {
    if (!d_scale || (n > 0 && (!x || !q))) return HGEMM_ERR_INVALID_VALUE;
    if (x_dtype != HGEMM_DTYPE_F32 && x_dtype != HGEMM_DTYPE_BF16) return HGEMM_ERR_INVALID_VALUE;
    if ((reinterpret_cast<uintptr_t>(x) & 15u) || (reinterpret_cast<uintptr_t>(q) & 15u) ||
        (reinterpret_cast<uintptr_t>(d_scale) & 3u)) {
        return HGEMM_ERR_ALIGNMENT;
    }
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    uint8_t* out = static_cast<uint8_t*>(q);
    if (x_dtype == HGEMM_DTYPE_F32) return hgq::run(static_cast<const float*>(x), n, out, d_scale, s);
    return hgq::run(static_cast<const __nv_bfloat16*>(x), n, out, d_scale, s);
}
