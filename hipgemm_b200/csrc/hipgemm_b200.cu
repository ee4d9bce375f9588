// C-ABI of the B200 FP8 GEMM: argument checks, TMA tensor maps, configuration choice
// and launch.  Declarations and the contract live in include/hipgemm_b200.h.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <random>
#include <vector>

#include "../../include/hipgemm_b200.h"
#include "gemm_sm100.cuh"

namespace hg {
namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

constexpr int kMaxDevices = 64;

constexpr int kMaxConfigs = 16;

struct DeviceState {
    std::once_flag once;
    int status = HGEMM_ERR_NO_DEVICE;
    int num_sms = 0;
    // Persistent grid size per configuration: CTAs that can be resident at once.  For
    // CTA pairs this comes from cudaOccupancyMaxActiveClusters, which can be below
    // num_sms / 2 (clusters must fit inside one GPC).
    int resident_ctas[kMaxConfigs] = {};
};

DeviceState g_devices[kMaxDevices];
std::once_flag g_encode_once;
EncodeTiledFn g_encode = nullptr;

// ---- kernel configurations ----------------------------------------------------------

struct KernelConfig {
    const char* name;
    int bm;          // output tile rows (256 for a CTA pair)
    int bn;          // output tile columns
    int ctas;        // CTAs per tile (2 = cta_group::2 pair)
    int b_box_rows;  // rows of B one CTA loads per K block
    double eff;      // relative per-SM efficiency used by the automatic choice
    int smem_bytes;
    const void* kernel;  // __global__ function pointer
    int (*launch)(const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, const GemmParams&, int grid,
                  cudaStream_t);
};

template <int BN, int STAGES>
int launch_1cta(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const GemmParams& p, int grid,
                cudaStream_t stream) {
    using Cfg = GemmConfig<BN, STAGES>;
    fp8_gemm_tn_sm100<BN, STAGES><<<grid, Cfg::kNumThreads, Cfg::SMEM_BYTES, stream>>>(ta, tb, tc, p);
    return cudaGetLastError() == cudaSuccess ? HGEMM_OK : HGEMM_ERR_CUDA;
}

template <int BN, int STAGES>
KernelConfig make_1cta(const char* name, double eff) {
    return KernelConfig{name, 128, BN, 1, BN, eff, GemmConfig<BN, STAGES>::SMEM_BYTES,
                        reinterpret_cast<const void*>(&fp8_gemm_tn_sm100<BN, STAGES>), &launch_1cta<BN, STAGES>};
}

template <int BN, int STAGES>
int launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const GemmParams& p, int grid,
                cudaStream_t stream) {
    using Cfg = PairConfig<BN, STAGES>;
    // The cluster shape (2, 1, 1) is compiled into the kernel; grid is a multiple of 2.
    fp8_gemm_tn_sm100_pair<BN, STAGES><<<grid, Cfg::kNumThreads, Cfg::SMEM_BYTES, stream>>>(ta, tb, tc, p);
    return cudaGetLastError() == cudaSuccess ? HGEMM_OK : HGEMM_ERR_CUDA;
}

template <int BN, int STAGES>
KernelConfig make_pair(const char* name, double eff) {
    return KernelConfig{name, 256, BN, 2, BN / 2, eff, PairConfig<BN, STAGES>::SMEM_BYTES,
                        reinterpret_cast<const void*>(&fp8_gemm_tn_sm100_pair<BN, STAGES>),
                        &launch_pair<BN, STAGES>};
}

const KernelConfig kConfigs[] = {
    {"auto", 0, 0, 0, 0, 0.0, 0, nullptr, nullptr},
    make_1cta<256, 4>("bn256_s4", 0.93),
    make_1cta<128, 6>("bn128_s6", 0.80),
    make_1cta<64, 8>("bn64_s8", 0.45),
    make_pair<256, 6>("pair256_s6", 1.0),
    make_pair<128, 8>("pair128_s8", 0.85),
};
constexpr int kNumConfigs = sizeof(kConfigs) / sizeof(kConfigs[0]);

void init_encode() {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
        g_encode = reinterpret_cast<EncodeTiledFn>(fn);
    }
}

int device_setup(int dev) {
    if (dev < 0 || dev >= kMaxDevices) return HGEMM_ERR_NO_DEVICE;
    DeviceState& st = g_devices[dev];
    std::call_once(st.once, [&]() {
        cudaDeviceProp prop{};
        if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return;
        if (prop.major != 10) return;  // built for sm_100a only
        std::call_once(g_encode_once, init_encode);
        if (!g_encode) {
            st.status = HGEMM_ERR_CUDA;
            return;
        }
        static_assert(kNumConfigs <= kMaxConfigs, "raise kMaxConfigs");
        for (int c = 1; c < kNumConfigs; ++c) {
            const KernelConfig& k = kConfigs[c];
            if (cudaFuncSetAttribute(k.kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, k.smem_bytes) !=
                cudaSuccess) {
                st.status = HGEMM_ERR_CUDA;
                return;
            }
            if (k.ctas == 1) {
                st.resident_ctas[c] = prop.multiProcessorCount;
                continue;
            }
            cudaLaunchConfig_t cfg{};
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = k.ctas;
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            cfg.gridDim = dim3(static_cast<unsigned>(k.ctas * (prop.multiProcessorCount / k.ctas)), 1, 1);
            cfg.blockDim = dim3(192, 1, 1);
            cfg.dynamicSmemBytes = static_cast<size_t>(k.smem_bytes);
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            int clusters = 0;
            if (cudaOccupancyMaxActiveClusters(&clusters, k.kernel, &cfg) != cudaSuccess || clusters <= 0) {
                cudaGetLastError();
                st.status = HGEMM_ERR_CUDA;
                return;
            }
            st.resident_ctas[c] = clusters * k.ctas;
        }
        st.num_sms = prop.multiProcessorCount;
        st.status = HGEMM_OK;
    });
    return st.status;
}

const DeviceState* current_device_setup(int* rc) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        *rc = HGEMM_ERR_NO_DEVICE;
        return nullptr;
    }
    *rc = device_setup(dev);
    return *rc == HGEMM_OK ? &g_devices[dev] : nullptr;
}

bool encode_2d(CUtensorMap* map, CUtensorMapDataType dtype, size_t elem_bytes, const void* ptr, uint64_t inner,
               uint64_t outer, uint32_t box_inner, uint32_t box_outer) {
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {inner * elem_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    return g_encode(map, dtype, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Estimated relative time of a configuration: waves of output tiles over the SMs (CTA
// pairs count as one tile slot per two SMs) times the per-SM share of one tile,
// divided by the configuration's measured relative efficiency at large sizes.
int choose_config(int M, int N, const DeviceState& dev) {
    int best = 1;
    double best_cost = 1e300;
    for (int c = 1; c < kNumConfigs; ++c) {
        const KernelConfig& k = kConfigs[c];
        const long tiles = static_cast<long>((M + k.bm - 1) / k.bm) * ((N + k.bn - 1) / k.bn);
        const long slots = std::max(1, dev.resident_ctas[c] / k.ctas);
        const long waves = (tiles + slots - 1) / slots;
        const double cost = static_cast<double>(waves) * (k.bm / k.ctas) * k.bn / k.eff;
        if (cost < best_cost - 1e-9) {
            best_cost = cost;
            best = c;
        }
    }
    return best;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int run_gemm(const void* A, const void* B, void* C, int M, int N, int K, const float* sa, const float* sb,
             cudaStream_t stream, int config) {
    if (M < 0 || N < 0 || K < 0) return HGEMM_ERR_INVALID_VALUE;
    if (config < 0 || config >= kNumConfigs) return HGEMM_ERR_INVALID_VALUE;
    if (M == 0 || N == 0) return HGEMM_OK;
    if (!C || (K > 0 && (!A || !B))) return HGEMM_ERR_INVALID_VALUE;
    if (K % 16 != 0 || N % 8 != 0) return HGEMM_ERR_ALIGNMENT;
    if (!aligned16(C) || (K > 0 && (!aligned16(A) || !aligned16(B)))) return HGEMM_ERR_ALIGNMENT;
    int rc = HGEMM_OK;
    const DeviceState* dev = current_device_setup(&rc);
    if (rc != HGEMM_OK) return rc;
    if (K == 0) {
        // An empty sum: every element is bf16(+0), as the reference's acc = 0.0f gives.
        return cudaMemsetAsync(C, 0, static_cast<size_t>(M) * N * 2, stream) == cudaSuccess ? HGEMM_OK
                                                                                              : HGEMM_ERR_CUDA;
    }
    const int c = config == 0 ? choose_config(M, N, *dev) : config;
    const KernelConfig& kc = kConfigs[c];

    CUtensorMap ta, tb, tc;
    if (!encode_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, A, static_cast<uint64_t>(K), static_cast<uint64_t>(M), 128,
                   128) ||
        !encode_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, B, static_cast<uint64_t>(K), static_cast<uint64_t>(N), 128,
                   static_cast<uint32_t>(kc.b_box_rows)) ||
        !encode_2d(&tc, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, C, static_cast<uint64_t>(N), static_cast<uint64_t>(M), 64,
                   32)) {
        return HGEMM_ERR_CUDA;
    }
    GemmParams p{};
    p.M = M;
    p.N = N;
    p.K = K;
    p.num_m_blocks = (M + kc.bm - 1) / kc.bm;
    p.num_n_blocks = (N + kc.bn - 1) / kc.bn;
    p.num_k_blocks = (K + 127) / 128;
    p.group_m = kc.ctas == 2 ? 8 : 16;
    p.scale_a = sa;
    p.scale_b = sb;
    const long tiles = static_cast<long>(p.num_m_blocks) * p.num_n_blocks;
    const int slots = std::max(1, dev->resident_ctas[c] / kc.ctas);
    const int grid = static_cast<int>(std::min<long>(tiles, slots)) * kc.ctas;
    return kc.launch(ta, tb, tc, p, grid, stream);
}

}  // namespace
}  // namespace hg

extern "C" {

int hgemm_fp8_tn(const void* A, const void* B, void* C, int M, int N, int K, const float* d_scale_a,
                 const float* d_scale_b, hgemm_stream_t stream) {
    return hg::run_gemm(A, B, C, M, N, K, d_scale_a, d_scale_b, reinterpret_cast<cudaStream_t>(stream), 0);
}

int hgemm_fp8_tn_config(const void* A, const void* B, void* C, int M, int N, int K, const float* d_scale_a,
                        const float* d_scale_b, hgemm_stream_t stream, int config) {
    return hg::run_gemm(A, B, C, M, N, K, d_scale_a, d_scale_b, reinterpret_cast<cudaStream_t>(stream), config);
}

int hgemm_fp8_tn_rows(const void* A, const void* B, void* C, int M, int N, int K, int row_begin, int row_end,
                      const float* d_scale_a, const float* d_scale_b, hgemm_stream_t stream) {
    if (M < 0 || N < 0 || K < 0 || row_begin < 0 || row_end < row_begin || row_end > M) {
        return HGEMM_ERR_INVALID_VALUE;
    }
    if (row_end == row_begin || N == 0) return HGEMM_OK;
    if (!A || !C) return HGEMM_ERR_INVALID_VALUE;
    const uint8_t* a = static_cast<const uint8_t*>(A) + static_cast<size_t>(row_begin) * K;
    uint8_t* c = static_cast<uint8_t*>(C) + static_cast<size_t>(row_begin) * N * 2;
    return hg::run_gemm(a, B, c, row_end - row_begin, N, K, d_scale_a, d_scale_b,
                        reinterpret_cast<cudaStream_t>(stream), 0);
}

int hgemm_num_configs(void) { return hg::kNumConfigs; }

int hgemm_config_resident_ctas(int config) {
    if (config <= 0 || config >= hg::kNumConfigs) return HGEMM_ERR_INVALID_VALUE;
    int rc = HGEMM_OK;
    const hg::DeviceState* dev = hg::current_device_setup(&rc);
    return dev ? dev->resident_ctas[config] : rc;
}

const char* hgemm_config_name(int config) {
    if (config < 0 || config >= hg::kNumConfigs) return nullptr;
    return hg::kConfigs[config].name;
}

int hgemm_device_status(uint32_t* status_out) {
    uint32_t v = 0;
    if (cudaMemcpyFromSymbol(&v, hg::g_status, sizeof(v)) != cudaSuccess) return HGEMM_ERR_CUDA;
    const uint32_t zero = 0;
    if (cudaMemcpyToSymbol(hg::g_status, &zero, sizeof(zero)) != cudaSuccess) return HGEMM_ERR_CUDA;
    if (status_out) *status_out = v;
    return v == 0 ? HGEMM_OK : HGEMM_ERR_DEVICE_TIMEOUT;
}

const char* hgemm_error_string(int code) {
    switch (code) {
        case HGEMM_OK: return "ok";
        case HGEMM_ERR_INVALID_VALUE: return "invalid value (null operand, negative size or bad row range)";
        case HGEMM_ERR_ALIGNMENT: return "alignment: need K % 16 == 0, N % 8 == 0 and 16-byte aligned A, B, C";
        case HGEMM_ERR_UNSUPPORTED: return "unsupported size";
        case HGEMM_ERR_CUDA: return "CUDA runtime/driver call failed";
        case HGEMM_ERR_NO_DEVICE: return "no sm_100 CUDA device is current";
        case HGEMM_ERR_DEVICE_TIMEOUT: return "a bounded wait inside a kernel expired";
        default: return "unknown status";
    }
}

const char* hgemm_version(void) { return "hipgemm_b200 0.1.0 (sm_100a)"; }

// ---- host utilities (utils.hpp mirror) ----------------------------------------------

uint8_t hgemm_host_fp8_encode(float x) {
    return static_cast<uint8_t>(__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3));
}

void hgemm_host_fp8_encode_array(const float* x, size_t n, uint8_t* out) {
    for (size_t i = 0; i < n; ++i) out[i] = hgemm_host_fp8_encode(x[i]);
}

uint16_t hgemm_host_bf16_rne(float x) {
    const __nv_bfloat16 b = __float2bfloat16_rn(x);
    uint16_t bits;
    std::memcpy(&bits, &b, 2);
    return bits;
}

void hgemm_host_init_random(uint8_t* out, size_t n, uint64_t seed, float mean, float stddev) {
    std::mt19937 gen(static_cast<std::mt19937::result_type>(seed));
    std::normal_distribution<float> dis(mean, stddev);
    for (size_t i = 0; i < n; ++i) out[i] = hgemm_host_fp8_encode(dis(gen));
}

float hgemm_host_quantize_e4m3(const float* x, size_t n, uint8_t* q) {
    float amax = 0.0f;
    for (size_t i = 0; i < n; ++i) amax = std::max(amax, std::fabs(x[i]));
    const float scale = amax > 0.0f ? amax / 448.0f : 1.0f;
    for (size_t i = 0; i < n; ++i) q[i] = hgemm_host_fp8_encode(x[i] / scale);
    return scale;
}

float hgemm_host_make_quantized(uint8_t* q, size_t n, uint64_t seed, float mean, float stddev) {
    std::vector<float> x(n);
    std::mt19937 gen(static_cast<std::mt19937::result_type>(seed));
    std::normal_distribution<float> dis(mean, stddev);
    for (size_t i = 0; i < n; ++i) x[i] = dis(gen);
    return hgemm_host_quantize_e4m3(x.data(), n, q);
}

}  // extern "C"
