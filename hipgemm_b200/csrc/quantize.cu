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

// q = e4m3(x / scale): 16 elements (16 output bytes) per thread and step.
template <typename T>
__global__ void __launch_bounds__(kThreads) quantize_kernel(const T* __restrict__ x, size_t n,
                                                             const unsigned int* __restrict__ amax_bits,
                                                             uint8_t* __restrict__ q) {
    constexpr int E = Vec<T>::kElems;
    constexpr int LOADS = 16 / E;
    const float s = scale_from_amax(*amax_bits);
    const size_t ngroups = n / 16;
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t g = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; g < ngroups; g += stride) {
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

// Turns the accumulated amax bits into the scale, in place.
__global__ void finalize_scale_kernel(unsigned int* amax_bits) {
    const float s = scale_from_amax(*amax_bits);
    *reinterpret_cast<float*>(amax_bits) = s;
}

int grid_for(size_t work_items) {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const size_t blocks = (work_items + kThreads - 1) / kThreads;
    const size_t cap = static_cast<size_t>(sms) * 8;
    return static_cast<int>(blocks < 1 ? 1 : (blocks > cap ? cap : blocks));
}

template <typename T>
int run(const T* x, size_t n, uint8_t* q, float* d_scale, cudaStream_t stream) {
    unsigned int* acc = reinterpret_cast<unsigned int*>(d_scale);
    if (cudaMemsetAsync(acc, 0, sizeof(unsigned int), stream) != cudaSuccess) return HGEMM_ERR_CUDA;
    if (n > 0) {
        amax_kernel<T><<<grid_for(n / Vec<T>::kElems + 1), kThreads, 0, stream>>>(x, n, acc);
        quantize_kernel<T><<<grid_for(n / 16 + 1), kThreads, 0, stream>>>(x, n, acc, q);
    }
    finalize_scale_kernel<<<1, 1, 0, stream>>>(acc);
    return cudaGetLastError() == cudaSuccess ? HGEMM_OK : HGEMM_ERR_CUDA;
}

}  // namespace hgq

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
