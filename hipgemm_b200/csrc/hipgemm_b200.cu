// C-ABI of the B200 FP8 GEMM: argument checks, TMA tensor maps, configuration choice
// and launch.  Declarations and the contract live in include/hipgemm_b200.h.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <random>
#include <vector>

#include "hipgemm_b200.h"
#include "gemm_sm100.cuh"

namespace hg {
namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

constexpr int kMaxDevices = 64;

// Tile rows per raster group (measured best for pairs too: 8192^3 2948 against 2874 TFLOP/s
// with 8).  HG_GROUP_M overrides it at build time for sweeps.
#ifndef HG_GROUP_M
#define HG_GROUP_M 16
#endif
constexpr int kGroupM = HG_GROUP_M;

constexpr int kMaxConfigs = 16;

struct DeviceState {
    // Set-up runs under the mutex until it succeeds once; `ready` then makes every later call
    // a single atomic load.  A failed set-up is not cached (a later call tries again), except
    // a device this library was not built for, which stays refused.
    std::mutex setup_mutex;
    std::atomic<bool> ready{false};
    bool wrong_arch = false;
    int num_sms = 0;
    // Persistent grid size per configuration: CTAs that can be resident at once.  For
    // CTA pairs this comes from cudaOccupancyMaxActiveClusters, which can be below
    // num_sms / 2 (clusters must fit inside one GPC).
    int resident_ctas[kMaxConfigs] = {};
    int mx_resident_ctas[kMaxConfigs] = {};  // the same for the MX configurations
    // Stream-K workspaces: a library-owned stream-ordered pool, created by the first call that
    // needs library-allocated scratch (never by device_setup, so that entry points with their
    // own scratch never create one).
    std::mutex pool_mutex;
    cudaMemPool_t pool = nullptr;
};

DeviceState g_devices[kMaxDevices];
std::once_flag g_encode_once;
EncodeTiledFn g_encode = nullptr;
using AddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
AddressRangeFn g_address_range = nullptr;

// ---- kernel configurations ----------------------------------------------------------

struct KernelConfig {
    const char* name;
    int ctas;        // CTAs per tile (2 = cta_group::2 pair, launched as a 2-CTA cluster)
    int bm;          // output tile rows (128 * ctas)
    int bn;          // output tile columns
    int b_box_rows;  // rows of B one CTA loads per K block (bn / ctas)
    double eff;      // relative per-SM throughput at large sizes (measured), for the choice
    int smem_bytes;
    int partial_floats;  // one CTA's fp32 partial tile (stream-K workspace unit)
    int epi_cols;        // columns per C store box (64: 128-byte swizzle, 32: 64-byte swizzle)
    const void* kernel;  // __global__ function pointer
    int (*launch)(const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, const GemmParams&,
                  const PeerOutputs&, const SfMaps&, int grid, cudaStream_t);
    int kbs;    // K blocks per stage (2: 3-D operand maps, which need K % 128 == 0)
    int split;  // > 1: split-K over clusters of `split` CTAs, one tile per cluster
};

template <int CTAS, int BN, int STAGES, bool MX = false, int KBS = 1, int SPLIT = 1>
int launch_kernel(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const GemmParams& p,
                  const PeerOutputs& peers, const SfMaps& sfm, int grid, cudaStream_t stream) {
    using S = KernelShape<CTAS, BN, STAGES, MX, KBS, SPLIT>;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
    cfg.blockDim = dim3(S::kNumThreads, 1, 1);
    cfg.dynamicSmemBytes = static_cast<size_t>(S::SMEM_BYTES);
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    unsigned n_attr = 0;
    if (CTAS * SPLIT > 1) {
        attr[n_attr].id = cudaLaunchAttributeClusterDimension;
        attr[n_attr].val.clusterDim.x = CTAS * SPLIT;
        attr[n_attr].val.clusterDim.y = 1;
        attr[n_attr].val.clusterDim.z = 1;
        ++n_attr;
    }
    // Programmatic dependent launch: the kernel may be scheduled while the stream's previous
    // kernel (one of ours) finishes; it touches no global memory before griddepcontrol.wait.
    attr[n_attr].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n_attr].val.programmaticStreamSerializationAllowed = 1;
    ++n_attr;
    cfg.attrs = attr;
    cfg.numAttrs = n_attr;
    const cudaError_t e =
        cudaLaunchKernelEx(&cfg, fp8_gemm_tn_sm100<CTAS, BN, STAGES, MX, KBS, SPLIT>, ta, tb, tc, p, peers, sfm);
    return e == cudaSuccess ? HGEMM_OK : HGEMM_ERR_CUDA;
}

template <int CTAS, int BN, int STAGES, bool MX = false, int KBS = 1, int SPLIT = 1>
KernelConfig make_config(const char* name, double eff) {
    using S = KernelShape<CTAS, BN, STAGES, MX, KBS, SPLIT>;
    return KernelConfig{name,         CTAS,
                        S::BM,        BN,
                        S::B_ROWS,    eff,
                        S::SMEM_BYTES, S::PARTIAL_FLOATS,
                        S::EPI_COLS,
                        reinterpret_cast<const void*>(&fp8_gemm_tn_sm100<CTAS, BN, STAGES, MX, KBS, SPLIT>),
                        &launch_kernel<CTAS, BN, STAGES, MX, KBS, SPLIT>,
                        KBS,          SPLIT};
}

const KernelConfig kConfigs[] = {
    {"auto", 0, 0, 0, 0, 0.0, 0, 0, 0, nullptr, nullptr},
    make_config<1, 256, 4>("bn256_s4", 0.93),
    make_config<1, 128, 6>("bn128_s6", 0.70),
    make_config<1, 64, 8>("bn64_s8", 0.35),
    make_config<2, 256, 6>("pair256_s6", 1.0),
    make_config<2, 128, 8>("pair128_s8", 0.62),
    // 0.84: per CTA pair a 256x224 tile took as long as a 256x256 one on B200 (CUDA-graph replay,
    // same process): 1024 x 7168 x 2048 17.0 against 16.0 us, 4000 x 5120 x 7168 113 against
    // 109 us, 1024 x 8192 x 8192 and 2048 x 8192 x 8192 level.  A narrower tile never needs fewer
    // waves, so with this factor the automatic choice no longer takes it; it stays available
    // as an explicit configuration.
    make_config<2, 224, 6>("pair224_s6", 0.84),
    make_config<1, 128, 5, false, 1, 2>("bn128_s5_k2", 0.85),
    make_config<1, 128, 5, false, 1, 4>("bn128_s5_k4", 0.70),
};
constexpr int kNumConfigs = sizeof(kConfigs) / sizeof(kConfigs[0]);

// MX block-scaled kernels (index c + 1 of hgemm_fp8_tn_mx_config; 0 = choose).  256 x 256
// tiles on CTA pairs and 128 x 256 tiles, both with one accumulator (early release), and
// 128 x 128 tiles with two for grids too small to fill the GPU with the wide tiles.  The
// "x2" kernels stage two K blocks per TMA load (K % 128 == 0 only): measured at 8192^3 on
// B200, 620-630 K cycles against 690-705 K for the pair, and +15 % for the 128 x 128 tile;
// the plain kernel gains nothing from it (515 K cycles either way).  eff: measured per-SM
// throughput at 8192^3 relative to the best config.
const KernelConfig kMxConfigs[] = {
    make_config<1, 256, 4, true>("mx_bn256_s4", 0.85),
    make_config<1, 128, 5, true>("mx_bn128_s5", 0.51),
    make_config<2, 256, 6, true>("mx_pair256_s6", 0.90),
    make_config<2, 256, 3, true, 2>("mx_pair256_s3x2", 1.0),
    make_config<1, 128, 3, true, 2>("mx_bn128_s3x2", 0.60),
};
constexpr int kNumMxConfigs = sizeof(kMxConfigs) / sizeof(kMxConfigs[0]);

// Fewest estimated tile-time units: waves of tiles over the resident slots (CTAs or CTA
// pairs) times the tile's per-SM MMA work (BM * BN / (128 * 128 * CTAS)) over its efficiency.
int choose_mx_config(int M, int N, int K, const int* resident_ctas) {
    int best = 0;
    double best_cost = 0.0;
    for (int c = 0; c < kNumMxConfigs; ++c) {
        const KernelConfig& k = kMxConfigs[c];
        if (k.kbs > 1 && K % 128 != 0) continue;
        const long long tiles = static_cast<long long>((M + k.bm - 1) / k.bm) * ((N + k.bn - 1) / k.bn);
        const long long slots = resident_ctas[c] / k.ctas;
        if (slots < 1) continue;
        const long long waves = (tiles + slots - 1) / slots;
        const double cost = static_cast<double>(waves) * (k.bm * k.bn / (128.0 * 128.0 * k.ctas)) / k.eff;
        if (best_cost == 0.0 || cost < best_cost) {
            best = c;
            best_cost = cost;
        }
    }
    return best;
}

void init_encode() {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
        g_encode = reinterpret_cast<EncodeTiledFn>(fn);
    }
    fn = nullptr;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
        g_address_range = reinterpret_cast<AddressRangeFn>(fn);
    }
}

int device_setup(int dev) {
    if (dev < 0 || dev >= kMaxDevices) return HGEMM_ERR_NO_DEVICE;
    DeviceState& st = g_devices[dev];
    if (st.ready.load(std::memory_order_acquire)) return HGEMM_OK;
    std::lock_guard<std::mutex> lock(st.setup_mutex);
    if (st.ready.load(std::memory_order_relaxed)) return HGEMM_OK;
    if (st.wrong_arch) return HGEMM_ERR_NO_DEVICE;
    cudaDeviceProp prop{};
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) {
        cudaGetLastError();
        return HGEMM_ERR_NO_DEVICE;
    }
    if (prop.major != 10) {  // built for sm_100a only
        st.wrong_arch = true;
        return HGEMM_ERR_NO_DEVICE;
    }
    std::call_once(g_encode_once, init_encode);
    if (!g_encode) return HGEMM_ERR_CUDA;
    static_assert(kNumConfigs <= kMaxConfigs && kNumMxConfigs <= kMaxConfigs, "raise kMaxConfigs");
    // Shared memory opt-in, then the CTAs that can be resident at once (0 on failure).
    auto resident = [&](const KernelConfig& k) -> int {
        if (cudaFuncSetAttribute(k.kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, k.smem_bytes) != cudaSuccess) {
            cudaGetLastError();
            return 0;
        }
        const int csize = k.ctas * k.split;  // CTAs per cluster
        if (csize == 1) return prop.multiProcessorCount;
        cudaLaunchConfig_t cfg{};
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = csize;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.gridDim = dim3(static_cast<unsigned>(csize * (prop.multiProcessorCount / csize)), 1, 1);
        cfg.blockDim = dim3(192, 1, 1);
        cfg.dynamicSmemBytes = static_cast<size_t>(k.smem_bytes);
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int clusters = 0;
        if (cudaOccupancyMaxActiveClusters(&clusters, k.kernel, &cfg) != cudaSuccess || clusters <= 0) {
            cudaGetLastError();
            return 0;
        }
        return clusters * csize;
    };
    for (int c = 1; c < kNumConfigs; ++c) {
        st.resident_ctas[c] = resident(kConfigs[c]);
        if (st.resident_ctas[c] == 0) return HGEMM_ERR_CUDA;
    }
    for (int c = 0; c < kNumMxConfigs; ++c) {
        st.mx_resident_ctas[c] = resident(kMxConfigs[c]);
        if (st.mx_resident_ctas[c] == 0) return HGEMM_ERR_CUDA;
    }
    st.num_sms = prop.multiProcessorCount;
    st.ready.store(true, std::memory_order_release);
    return HGEMM_OK;
}

// The device's stream-K workspace pool, created on first use.  It keeps its memory (release
// threshold = max) so repeated calls do not map pages again.  A failed creation is not
// cached: the next call tries again.
cudaMemPool_t workspace_pool(int dev) {
    DeviceState& st = g_devices[dev];
    std::lock_guard<std::mutex> lock(st.pool_mutex);
    if (st.pool) return st.pool;
    cudaMemPoolProps props{};
    props.allocType = cudaMemAllocationTypePinned;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = dev;
    cudaMemPool_t pool = nullptr;
    if (cudaMemPoolCreate(&pool, &props) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    uint64_t threshold = UINT64_MAX;
    cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &threshold);
    st.pool = pool;
    return pool;
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
               uint64_t outer, uint32_t box_inner, uint32_t box_outer,
               CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B, uint64_t row_stride_bytes = 0) {
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {row_stride_bytes ? row_stride_bytes : inner * elem_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    return g_encode(map, dtype, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// An e4m3 operand (rows x K bytes, row-major) for a kernel with `kbs` K blocks per stage.
// kbs = 1: 2-D, x = K byte, y = row, box 128 x box_rows.  kbs = 2: 3-D, x = byte in a
// 128-byte K chunk, y = row, z = chunk (stride 128 bytes), box 128 x box_rows x 2, which lands
// in shared memory as two K-block tiles back to back; needs K % 128 == 0, or the last chunk
// would read the next row's bytes instead of zeros.
bool encode_operand(CUtensorMap* map, const void* ptr, int K, int rows, int box_rows, int kbs) {
    if (kbs == 1) {
        return encode_2d(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, ptr, static_cast<uint64_t>(K),
                         static_cast<uint64_t>(rows), 128, static_cast<uint32_t>(box_rows));
    }
    const cuuint64_t dims[3] = {128, static_cast<cuuint64_t>(rows), static_cast<cuuint64_t>(K / 128)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(K), 128};
    const cuuint32_t box[3] = {128, static_cast<cuuint32_t>(box_rows), static_cast<cuuint32_t>(kbs)};
    const cuuint32_t estr[3] = {1, 1, 1};
    return g_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// An MX scale-factor tensor in the blocked layout as a 3-D map: x = 128 bytes, y = k_rows
// 128-byte rows along K (4 per atom), z = row_blocks 128-row blocks; box 128 x 4 kbs x
// box_blocks (the atoms of kbs K blocks).  Out-of-range rows and blocks read as zeros.
bool encode_sf_3d(CUtensorMap* map, const void* ptr, uint64_t k_rows, uint64_t row_blocks, uint32_t box_blocks,
                  int kbs) {
    const cuuint64_t dims[3] = {128, k_rows, row_blocks};
    const cuuint64_t strides[2] = {128, k_rows * 128};
    const cuuint32_t box[3] = {128, static_cast<cuuint32_t>(kSfRowsPerAtom * kbs), box_blocks};
    const cuuint32_t estr[3] = {1, 1, 1};
    return g_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// ---- schedule -------------------------------------------------------------------------

// Minimum K blocks (of 128) per stream-K slot: below this a slot's partial-tile write and
// reduction cost more than the load balance gains.
constexpr int kMinSkUnits = 8;

struct Schedule {
    int config;
    long tiles;
    int slots;   // resident slots (CTAs or CTA pairs) = persistent grid / ctas
    int grid;    // CTAs launched
    int dp_tiles;
    int sk_tiles;
    int sk_slots;
    size_t partial_bytes;  // workspace: partial tiles
    size_t counter_bytes;  // workspace: per-tile counters (zeroed before each launch)
};

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Splits `tiles` output tiles of `kblocks` K blocks over `slots` persistent slots into a
// data-parallel prefix and a stream-K suffix (sc.dp_tiles, sc.sk_tiles, sc.sk_slots).
void split_schedule(Schedule& sc, int kblocks, int schedule) {
    sc.dp_tiles = static_cast<int>(sc.tiles);
    sc.sk_tiles = 0;
    sc.sk_slots = 0;
    // The automatic schedule is data-parallel.  Measured on B200 (1024 x 8192 x 8192,
    // 4096^3, 128 x 8192 x 8192): even with the partial-tile traffic removed, splitting the
    // last waves along K did not beat whole tiles except on the skinny shape, where the
    // reduction of ~5 partials per tile costs more than the balance gains.  A partly idle
    // last wave runs its tiles faster (less contention for power and L2), which makes
    // wave quantisation cheaper here than SM counts suggest.
    if (schedule == HGEMM_SCHEDULE_STREAM_K) {
        const long full = sc.tiles / sc.slots, rem = sc.tiles % sc.slots;
        // Stream-K over the partial last wave when it gives every slot enough K; else
        // over the last full wave plus the partial one.
        long sk = rem;
        if (sk == 0 || sk * kblocks < static_cast<long>(kMinSkUnits) * sc.slots) sk = std::min<long>(sc.tiles, rem + sc.slots);
        if (full == 0) sk = sc.tiles;
        const long units = sk * kblocks;
        const long sk_slots = std::max<long>(1, std::min<long>(sc.slots, units / kMinSkUnits));
        sc.sk_tiles = static_cast<int>(sk);
        sc.dp_tiles = static_cast<int>(sc.tiles - sk);
        sc.sk_slots = static_cast<int>(sk_slots);
    }
}

// resident_ctas[c]: CTAs of configuration c resident at once (DeviceState::resident_ctas; the
// host-only test entry points pass their own).
Schedule make_schedule(int M, int N, int K, int config, int schedule, const int* resident_ctas) {
    const KernelConfig& k = kConfigs[config];
    Schedule sc{};
    sc.config = config;
    const long mblocks = (M + k.bm - 1) / k.bm, nblocks = (N + k.bn - 1) / k.bn;
    const int kblocks = (K + 127) / 128;
    sc.tiles = mblocks * nblocks;
    if (k.split > 1) {
        // Split-K clusters: one cluster per tile, every tile at once (clusters beyond the
        // resident ones start as earlier ones finish; no cluster waits on another).
        sc.slots = std::max(1, resident_ctas[config] / (k.ctas * k.split));
        sc.dp_tiles = static_cast<int>(sc.tiles);
        sc.grid = static_cast<int>(sc.tiles) * k.ctas * k.split;
        return sc;
    }
    sc.slots = std::max(1, resident_ctas[config] / k.ctas);
    split_schedule(sc, kblocks, schedule);
    if (sc.sk_tiles > 0) {
        sc.partial_bytes = align_up(static_cast<size_t>(sc.sk_slots) * 2 * k.ctas * k.partial_floats * 4, 256);
        sc.counter_bytes = align_up(static_cast<size_t>(sc.sk_tiles) * k.ctas * 4, 256);
    }
    sc.grid = static_cast<int>(std::min<long>(sc.tiles, sc.slots)) * k.ctas;
    if (sc.sk_tiles > 0) sc.grid = sc.slots * k.ctas;
    return sc;
}

Schedule make_schedule(int M, int N, int K, int config, int schedule, const DeviceState& dev) {
    return make_schedule(M, N, K, config, schedule, dev.resident_ctas);
}

// Estimated relative time of a configuration under the data-parallel schedule: waves of
// tiles over the resident slots times the per-SM share of one tile ((bm / ctas) x bn per
// K block), divided by the configuration's measured relative efficiency.
// Split-K cluster configurations take part only when `allow_split` (HGEMM_SCHEDULE_AUTO): an
// explicit data-parallel or stream-K schedule keeps whole-K tiles, and with them the same
// summation order, so the same bits, for any tile shape.
// full_rows: only configurations whose C stores write 128-byte row segments (64-column
// chunks), for the fused all-gather.  Its stores to peer memory cross NVLink, where 64-byte
// segments ran at two thirds of the rate: measured at 8 GPUs, 1024 x 8192 x 8192 per rank,
// 0.325 ms per step with the 224-wide tile against 0.231 ms with the 256-wide one.
int choose_config(int M, int N, int K, const int* resident_ctas, bool allow_split, bool full_rows = false) {
    int best = 1;
    double best_cost = 1e300;
    for (int c = 1; c < kNumConfigs; ++c) {
        const KernelConfig& k = kConfigs[c];
        if (k.kbs > 1 && K % 128 != 0) continue;
        if (full_rows && k.epi_cols != 64) continue;
        const Schedule sc = make_schedule(M, N, K, c, HGEMM_SCHEDULE_DATA_PARALLEL, resident_ctas);
        // Split-K only where every cluster fits at once and each part keeps some depth.
        // (Measured on B200: with fewer than 16 K blocks per part the exchange and the
        // cluster start cost more than the split gains, e.g. 128 x 7168 x 2048.)
        if (k.split > 1 && (!allow_split || sc.tiles > sc.slots || (K + 127) / 128 < 16 * k.split)) continue;
        const double area = static_cast<double>(k.bm / k.ctas) * k.bn / k.split;
        const double work_per_slot = static_cast<double>((sc.tiles + sc.slots - 1) / sc.slots);
        const double cost = work_per_slot * area / k.eff;
        if (cost < best_cost - 1e-9) {
            best_cost = cost;
            best = c;
        }
    }
    return best;
}

int choose_config(int M, int N, int K, const DeviceState& dev, bool allow_split, bool full_rows = false) {
    return choose_config(M, N, K, dev.resident_ctas, allow_split, full_rows);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_args(const void* A, const void* B, void* C, int M, int N, int K, int config, int schedule) {
    if (M < 0 || N < 0 || K < 0) return HGEMM_ERR_INVALID_VALUE;
    if (config < 0 || config >= kNumConfigs) return HGEMM_ERR_INVALID_VALUE;
    if (schedule < HGEMM_SCHEDULE_AUTO || schedule > HGEMM_SCHEDULE_STREAM_K) return HGEMM_ERR_INVALID_VALUE;
    if (M == 0 || N == 0) return HGEMM_OK;
    if (!C || (K > 0 && (!A || !B))) return HGEMM_ERR_INVALID_VALUE;
    if (K % 16 != 0 || N % 8 != 0) return HGEMM_ERR_ALIGNMENT;
    if (!aligned16(C) || (K > 0 && (!aligned16(A) || !aligned16(B)))) return HGEMM_ERR_ALIGNMENT;
    return HGEMM_OK;
}

// Per-thread cache of launch plans for the last few distinct calls without peer outputs: the
// configuration, the schedule and the four tensor maps (A, B, and C with 32- and 128-row
// boxes).  A hit skips the configuration choice and the tensor-map encodings, which are most of
// the host time of a call (measured on B200: ~4 us per call before, with three maps).  A plan
// depends only on the key's fields, so a buffer freed and reallocated at the same address with
// the same shape may reuse it.
struct PlanKey {
    const void* a;
    const void* b;
    const void* c;
    int M, N, K, ldc, config, schedule, dev;
};
struct PlanSlot {
    PlanKey key;
    bool valid;
    int cfg;
    Schedule sc;
    CUtensorMap ta, tb, tc, tcw;
};
// Fully associative, replaced round-robin: a caller that rotates through up to 32 buffer sets
// (as a benchmark over inputs larger than L2 does) hits on every call.  (A direct-mapped table
// indexed by a hash of the key let two of the sets share a slot and evict each other.)
constexpr int kPlanCacheSlots = 32;
thread_local PlanSlot t_plans[kPlanCacheSlots];
thread_local int t_plan_next = 0;

bool same_key(const PlanKey& x, const PlanKey& y) {
    return x.a == y.a && x.b == y.b && x.c == y.c && x.M == y.M && x.N == y.N && x.K == y.K && x.ldc == y.ldc &&
           x.config == y.config && x.schedule == y.schedule && x.dev == y.dev;
}

PlanSlot* find_plan(const PlanKey& k) {
    for (int i = 0; i < kPlanCacheSlots; ++i) {
        if (t_plans[i].valid && same_key(t_plans[i].key, k)) return &t_plans[i];
    }
    return nullptr;
}

PlanSlot& new_plan_slot() {
    PlanSlot& slot = t_plans[t_plan_next];
    t_plan_next = (t_plan_next + 1) % kPlanCacheSlots;
    return slot;
}

// workspace == nullptr: the library allocates it from its pool, stream-ordered.
// peer_c[0..n_peer): more M x N outputs (same layout as C) that receive every C tile too.
// ldc: C's row stride in elements (0: N), so that C can be a block of a wider matrix.
int run_gemm(const void* A, const void* B, void* C, int M, int N, int K, const float* sa, const float* sb,
             cudaStream_t stream, int config, int schedule, void* workspace, size_t workspace_bytes,
             void* const* peer_c = nullptr, int n_peer = 0, int ldc = 0, int debug_stall = 0) {
    int rc = check_args(A, B, C, M, N, K, config, schedule);
    if (rc != HGEMM_OK || M == 0 || N == 0) return rc;
    if (ldc == 0) ldc = N;
    if (ldc < N || ldc % 8 != 0 || (ldc != N && n_peer > 0)) return HGEMM_ERR_INVALID_VALUE;
    const DeviceState* dev = current_device_setup(&rc);
    if (rc != HGEMM_OK) return rc;
    if (K == 0) {
        // An empty sum: every element is bf16(+0), as the reference's acc = 0.0f gives.
        for (int i = -1; i < n_peer; ++i) {
            void* dst = i < 0 ? C : peer_c[i];
            if (cudaMemset2DAsync(dst, static_cast<size_t>(ldc) * 2, 0, static_cast<size_t>(N) * 2,
                                  static_cast<size_t>(M), stream) != cudaSuccess) {
                return HGEMM_ERR_CUDA;
            }
        }
        return HGEMM_OK;
    }
    if (n_peer < 0 || n_peer > kMaxPeerOutputs) return HGEMM_ERR_INVALID_VALUE;
    const PlanKey key{A, B, C, M, N, K, ldc, config, schedule, static_cast<int>(dev - g_devices)};
    PlanSlot* const cached = (n_peer == 0 && debug_stall == 0) ? find_plan(key) : nullptr;
    int c = 0;
    Schedule sc{};
    CUtensorMap ta, tb, tc;
    PeerOutputs peers{};
    if (cached) {
        c = cached->cfg;
        sc = cached->sc;
        ta = cached->ta;
        tb = cached->tb;
        tc = cached->tc;
        peers.wide[0] = cached->tcw;
    } else {
        c = config == 0 ? choose_config(M, N, K, *dev, schedule == HGEMM_SCHEDULE_AUTO, n_peer > 0) : config;
        const KernelConfig& kn = kConfigs[c];
        if (kn.kbs > 1 && K % 128 != 0) return HGEMM_ERR_UNSUPPORTED;  // (never chosen automatically then)
        sc = make_schedule(M, N, K, c, schedule, *dev);
        const CUtensorMapSwizzle csw = kn.epi_cols == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
        // C with 32-row boxes (per-warp stores) and 128-row boxes (CTA-wide stores of whole tiles).
        if (!encode_operand(&ta, A, K, M, 128, kn.kbs) || !encode_operand(&tb, B, K, N, kn.b_box_rows, kn.kbs) ||
            !encode_2d(&tc, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, C, static_cast<uint64_t>(N), static_cast<uint64_t>(M),
                       static_cast<uint32_t>(kn.epi_cols), 32, csw, static_cast<uint64_t>(ldc) * 2) ||
            !encode_2d(&peers.wide[0], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, C, static_cast<uint64_t>(N),
                       static_cast<uint64_t>(M), static_cast<uint32_t>(kn.epi_cols), 128, csw,
                       static_cast<uint64_t>(ldc) * 2)) {
            return HGEMM_ERR_CUDA;
        }
        if (n_peer == 0 && debug_stall == 0) {
            PlanSlot& slot = new_plan_slot();
            slot.key = key;
            slot.cfg = c;
            slot.sc = sc;
            slot.ta = ta;
            slot.tb = tb;
            slot.tc = tc;
            slot.tcw = peers.wide[0];
            slot.valid = true;
        }
    }
    const KernelConfig& kc = kConfigs[c];
    const CUtensorMapSwizzle c_swizzle = kc.epi_cols == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
    for (int i = 0; i < n_peer; ++i) {
        if (!encode_2d(&peers.maps[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, peer_c[i], static_cast<uint64_t>(N),
                       static_cast<uint64_t>(M), static_cast<uint32_t>(kc.epi_cols), 32, c_swizzle) ||
            !encode_2d(&peers.wide[1 + i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, peer_c[i], static_cast<uint64_t>(N),
                       static_cast<uint64_t>(M), static_cast<uint32_t>(kc.epi_cols), 128, c_swizzle)) {
            return HGEMM_ERR_CUDA;
        }
    }
    peers.count = n_peer;
    GemmParams p{};
    p.M = M;
    p.N = N;
    p.K = K;
    p.num_m_blocks = (M + kc.bm - 1) / kc.bm;
    p.num_n_blocks = (N + kc.bn - 1) / kc.bn;
    p.num_k_blocks = (K + 127) / 128;
    p.group_m = kGroupM;
    p.scale_a = sa;
    p.scale_b = sb;
    p.dp_tiles = sc.dp_tiles;
    p.sk_tiles = sc.sk_tiles;
    p.sk_slots = sc.sk_slots;
    p.split_k = kc.split;
    p.debug_stall_first_stage = debug_stall;
    const SfMaps no_sf{};
    if (sc.sk_tiles == 0) return kc.launch(ta, tb, tc, p, peers, no_sf, sc.grid, stream);

    const size_t need = sc.partial_bytes + sc.counter_bytes;
    void* ws = workspace;
    if (ws) {
        if (workspace_bytes < need || (reinterpret_cast<uintptr_t>(ws) & 255u)) return HGEMM_ERR_INVALID_VALUE;
    } else {
        const cudaMemPool_t pool = workspace_pool(static_cast<int>(dev - g_devices));
        if (!pool) return HGEMM_ERR_CUDA;
        if (cudaMallocFromPoolAsync(&ws, need, pool, stream) != cudaSuccess) {
            cudaGetLastError();
            return HGEMM_ERR_CUDA;
        }
    }
    p.partials = static_cast<float*>(ws);
    p.counters = reinterpret_cast<int*>(static_cast<uint8_t*>(ws) + sc.partial_bytes);
    rc = cudaMemsetAsync(p.counters, 0, sc.counter_bytes, stream) == cudaSuccess ? HGEMM_OK : HGEMM_ERR_CUDA;
    if (rc == HGEMM_OK) rc = kc.launch(ta, tb, tc, p, peers, no_sf, sc.grid, stream);
    if (!workspace && cudaFreeAsync(ws, stream) != cudaSuccess && rc == HGEMM_OK) rc = HGEMM_ERR_CUDA;
    return rc;
}

int run_gemm_mx(const void* A, const void* B, void* C, int M, int N, int K, const void* sfa, const void* sfb,
                const float* sa, const float* sb, int config, cudaStream_t stream) {
    if (config < 0 || config > kNumMxConfigs) return HGEMM_ERR_INVALID_VALUE;
    int rc = check_args(A, B, C, M, N, K, 0, HGEMM_SCHEDULE_DATA_PARALLEL);
    if (rc != HGEMM_OK || M == 0 || N == 0) return rc;
    if (K % 32 != 0) return HGEMM_ERR_ALIGNMENT;
    if (K > 0 && (!sfa || !sfb)) return HGEMM_ERR_INVALID_VALUE;
    if ((reinterpret_cast<uintptr_t>(sfa) & 15u) || (reinterpret_cast<uintptr_t>(sfb) & 15u)) return HGEMM_ERR_ALIGNMENT;
    // The two-K-block kernels read A and B as 128-byte K chunks, which needs K % 128 == 0.
    if (config > 0 && kMxConfigs[config - 1].kbs > 1 && K % 128 != 0) return HGEMM_ERR_UNSUPPORTED;
    const DeviceState* dev = current_device_setup(&rc);
    if (rc != HGEMM_OK) return rc;
    if (K == 0) {
        return cudaMemsetAsync(C, 0, static_cast<size_t>(M) * N * 2, stream) == cudaSuccess ? HGEMM_OK
                                                                                              : HGEMM_ERR_CUDA;
    }
    const int ci = config > 0 ? config - 1 : choose_mx_config(M, N, K, dev->mx_resident_ctas);
    const KernelConfig& kc = kMxConfigs[ci];
    CUtensorMap ta, tb, tc;
    if (!encode_operand(&ta, A, K, M, 128, kc.kbs) || !encode_operand(&tb, B, K, N, kc.b_box_rows, kc.kbs) ||
        !encode_2d(&tc, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, C, static_cast<uint64_t>(N), static_cast<uint64_t>(M),
                   static_cast<uint32_t>(kc.epi_cols), 32,
                   kc.epi_cols == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B)) {
        return HGEMM_ERR_CUDA;
    }
    GemmParams p{};
    p.M = M;
    p.N = N;
    p.K = K;
    p.num_m_blocks = (M + kc.bm - 1) / kc.bm;
    p.num_n_blocks = (N + kc.bn - 1) / kc.bn;
    p.num_k_blocks = (K + 127) / 128;
    p.group_m = kGroupM;
    p.scale_a = sa;
    p.scale_b = sb;
    p.dp_tiles = p.num_m_blocks * p.num_n_blocks;
    p.sf_k_atoms = (K + 127) / 128;
    // Scale factors as (128 bytes, 4 rows per atom along K, 128-row blocks); boxes of one
    // atom along K by 1 (A) or BN / 128 (B) row blocks, no swizzle.
    SfMaps sfm{};
    const uint64_t k_rows = static_cast<uint64_t>(p.sf_k_atoms) * kSfRowsPerAtom;
    if (!encode_sf_3d(&sfm.a, sfa, k_rows, static_cast<uint64_t>((M + 127) / 128), 1, kc.kbs) ||
        !encode_sf_3d(&sfm.b, sfb, k_rows, static_cast<uint64_t>((N + 127) / 128),
                      static_cast<uint32_t>(kc.bn / 128), kc.kbs)) {
        return HGEMM_ERR_CUDA;
    }
    PeerOutputs peers{};
    if (!encode_2d(&peers.wide[0], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, C, static_cast<uint64_t>(N),
                   static_cast<uint64_t>(M), static_cast<uint32_t>(kc.epi_cols), 128,
                   kc.epi_cols == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B)) {
        return HGEMM_ERR_CUDA;
    }
    const int slots = dev->mx_resident_ctas[ci] / kc.ctas;
    const int grid = kc.ctas * std::min(p.dp_tiles, slots);
    return kc.launch(ta, tb, tc, p, peers, sfm, grid, stream);
}

}  // namespace
}  // namespace hg

extern "C" {

int hgemm_fp8_tn_mx(const void* A, const void* B, void* C, int M, int N, int K, const void* SFA, const void* SFB,
                    const float* d_scale_a, const float* d_scale_b, hgemm_stream_t stream) {
    return hg::run_gemm_mx(A, B, C, M, N, K, SFA, SFB, d_scale_a, d_scale_b, 0, reinterpret_cast<cudaStream_t>(stream));
}

int hgemm_fp8_tn_mx_config(const void* A, const void* B, void* C, int M, int N, int K, const void* SFA,
                           const void* SFB, const float* d_scale_a, const float* d_scale_b, int config,
                           hgemm_stream_t stream) {
    return hg::run_gemm_mx(A, B, C, M, N, K, SFA, SFB, d_scale_a, d_scale_b, config,
                           reinterpret_cast<cudaStream_t>(stream));
}

int hgemm_mx_num_configs(void) { return hg::kNumMxConfigs + 1; }

const char* hgemm_mx_config_name(int config) {
    if (config == 0) return "auto";
    if (config < 0 || config > hg::kNumMxConfigs) return nullptr;
    return hg::kMxConfigs[config - 1].name;
}

size_t hgemm_mx_sf_bytes(int rows, int K) {
    if (rows <= 0 || K <= 0) return 0;
    return static_cast<size_t>((rows + 127) / 128) * static_cast<size_t>((K + 127) / 128) * 512;
}

int hgemm_host_mx_sf_to_blocked(const uint8_t* sf, int rows, int K, uint8_t* blocked) {
    if (rows < 0 || K < 0 || K % 32 != 0 || (rows > 0 && K > 0 && (!sf || !blocked))) return HGEMM_ERR_INVALID_VALUE;
    if (rows == 0 || K == 0) return HGEMM_OK;  // nothing to write
    const int groups = K / 32, k_atoms = (K + 127) / 128;
    // Padding (rows past `rows`, groups past K/32) holds 127 = 2^0, a finite scale.
    std::memset(blocked, 127, hgemm_mx_sf_bytes(rows, K));
    for (int r = 0; r < rows; ++r) {
        for (int g = 0; g < groups; ++g) {
            const size_t atom = static_cast<size_t>(r / 128) * k_atoms + g / 4;
            const int rr = r % 128;
            blocked[atom * 512 + 16 * (rr % 32) + 4 * (rr / 32) + (g % 4)] = sf[static_cast<size_t>(r) * groups + g];
        }
    }
    return HGEMM_OK;
}

int hgemm_debug_stalled_gemm(const void* A, const void* B, void* C, int M, int N, int K, int config,
                             hgemm_stream_t stream) {
    if (K <= 0) return HGEMM_ERR_INVALID_VALUE;  // the hook needs a first K block to withhold
    return hg::run_gemm(A, B, C, M, N, K, nullptr, nullptr, reinterpret_cast<cudaStream_t>(stream), config,
                        HGEMM_SCHEDULE_DATA_PARALLEL, nullptr, 0, nullptr, 0, 0, 1);
}

int hgemm_fp8_tn(const void* A, const void* B, void* C, int M, int N, int K, const float* d_scale_a,
                 const float* d_scale_b, hgemm_stream_t stream) {
    return hg::run_gemm(A, B, C, M, N, K, d_scale_a, d_scale_b, reinterpret_cast<cudaStream_t>(stream), 0,
                        HGEMM_SCHEDULE_AUTO, nullptr, 0);
}

int hgemm_fp8_tn_config(const void* A, const void* B, void* C, int M, int N, int K, const float* d_scale_a,
                        const float* d_scale_b, hgemm_stream_t stream, int config) {
    return hg::run_gemm(A, B, C, M, N, K, d_scale_a, d_scale_b, reinterpret_cast<cudaStream_t>(stream), config,
                        HGEMM_SCHEDULE_AUTO, nullptr, 0);
}

int hgemm_fp8_tn_ex(const void* A, const void* B, void* C, int M, int N, int K, const float* d_scale_a,
                    const float* d_scale_b, hgemm_stream_t stream, int config, int schedule, void* workspace,
                    size_t workspace_bytes) {
    return hg::run_gemm(A, B, C, M, N, K, d_scale_a, d_scale_b, reinterpret_cast<cudaStream_t>(stream), config,
                        schedule, workspace, workspace_bytes);
}

int hgemm_workspace_bytes(int M, int N, int K, int config, int schedule, size_t* bytes_out) {
    const int rc0 = hg::check_args(reinterpret_cast<const void*>(16), reinterpret_cast<const void*>(16),
                                   reinterpret_cast<void*>(16), M, N, K, config, schedule);
    if (rc0 != HGEMM_OK) return rc0;
    if (!bytes_out) return HGEMM_ERR_INVALID_VALUE;
    *bytes_out = 0;
    if (M == 0 || N == 0 || K == 0) return HGEMM_OK;
    int rc = HGEMM_OK;
    const hg::DeviceState* dev = hg::current_device_setup(&rc);
    if (!dev) return rc;
    const int c = config == 0 ? hg::choose_config(M, N, K, *dev, schedule == HGEMM_SCHEDULE_AUTO) : config;
    const hg::Schedule sc = hg::make_schedule(M, N, K, c, schedule, *dev);
    *bytes_out = sc.sk_tiles > 0 ? sc.partial_bytes + sc.counter_bytes : 0;
    return HGEMM_OK;
}

int hgemm_plan(int M, int N, int K, int config, int schedule, int* plan_out) {
    const int rc0 = hg::check_args(reinterpret_cast<const void*>(16), reinterpret_cast<const void*>(16),
                                   reinterpret_cast<void*>(16), M, N, K, config, schedule);
    if (rc0 != HGEMM_OK) return rc0;
    if (!plan_out || M <= 0 || N <= 0 || K <= 0) return HGEMM_ERR_INVALID_VALUE;
    int rc = HGEMM_OK;
    const hg::DeviceState* dev = hg::current_device_setup(&rc);
    if (!dev) return rc;
    const int c = config == 0 ? hg::choose_config(M, N, K, *dev, schedule == HGEMM_SCHEDULE_AUTO) : config;
    const hg::Schedule sc = hg::make_schedule(M, N, K, c, schedule, *dev);
    plan_out[0] = c;
    plan_out[1] = sc.grid;
    plan_out[2] = static_cast<int>(sc.tiles);
    plan_out[3] = sc.dp_tiles;
    plan_out[4] = sc.sk_tiles;
    plan_out[5] = sc.sk_slots;
    return HGEMM_OK;
}

int hgemm_debug_schedule(long long tiles, int slots, int kblocks, int schedule, int* out3) {
    if (tiles <= 0 || slots <= 0 || kblocks <= 0 || !out3) return HGEMM_ERR_INVALID_VALUE;
    hg::Schedule sc{};
    sc.tiles = tiles;
    sc.slots = slots;
    hg::split_schedule(sc, kblocks, schedule);
    out3[0] = sc.dp_tiles;
    out3[1] = sc.sk_tiles;
    out3[2] = sc.sk_slots;
    return HGEMM_OK;
}

int hgemm_debug_choose(int M, int N, int K, int schedule, const int* resident_ctas, int n_configs) {
    if (M <= 0 || N <= 0 || K <= 0 || !resident_ctas || n_configs != hg::kNumConfigs) return HGEMM_ERR_INVALID_VALUE;
    if (schedule < HGEMM_SCHEDULE_AUTO || schedule > HGEMM_SCHEDULE_STREAM_K) return HGEMM_ERR_INVALID_VALUE;
    for (int c = 1; c < n_configs; ++c) {
        if (resident_ctas[c] <= 0) return HGEMM_ERR_INVALID_VALUE;
    }
    return hg::choose_config(M, N, K, resident_ctas, schedule == HGEMM_SCHEDULE_AUTO);
}

int hgemm_debug_split_work(int kblocks, int split, int tiles, int cta, int* out3) {
    if (kblocks <= 0 || split < 2 || tiles <= 0 || cta < 0 || !out3) return HGEMM_ERR_INVALID_VALUE;
    hg::GemmParams p{};
    p.num_k_blocks = kblocks;
    p.dp_tiles = tiles;
    p.split_k = split;
    hg::Work w;
    if (!hg::get_work(p, cta, 0, 0, w)) return 0;
    out3[0] = w.tile;
    out3[1] = w.kb_begin;
    out3[2] = w.kb_end;
    return hg::get_work(p, cta, 0, 1, w) ? 2 : 1;  // a second item would be a bug
}

int hgemm_debug_work_items(int kblocks, int nslots, int dp_tiles, int sk_tiles, int sk_slots, int slot, int* out,
                           int max_items) {
    if (kblocks <= 0 || nslots <= 0 || slot < 0 || slot >= nslots || !out || sk_slots < 0 ||
        (sk_tiles > 0 && sk_slots <= 0)) {
        return HGEMM_ERR_INVALID_VALUE;
    }
    hg::GemmParams p{};
    p.num_k_blocks = kblocks;
    p.dp_tiles = dp_tiles;
    p.sk_tiles = sk_tiles;
    p.sk_slots = sk_slots;
    int n = 0;
    hg::Work w;
    for (int idx = 0; n < max_items && hg::get_work(p, slot, nslots, idx, w); ++idx, ++n) {
        int* o = out + 6 * n;
        o[0] = w.tile;
        o[1] = w.kb_begin;
        o[2] = w.kb_end;
        o[3] = w.piece;
        o[4] = 0;
        o[5] = 0;
        if (w.piece >= 0) {
            const long long u0 = static_cast<long long>(w.tile - dp_tiles) * kblocks;
            o[4] = hg::sk_slot_of_unit(p, u0);                // first contributor
            o[5] = hg::sk_slot_of_unit(p, u0 + kblocks - 1);  // last contributor
        }
    }
    return n;
}

int hgemm_fp8_tn_rows_allgather(const void* A, const void* B, void* const* C_ranks, int nranks, int rank, int M,
                                int N, int K, int row_begin, int row_end, const float* d_scale_a,
                                const float* d_scale_b, hgemm_stream_t stream) {
    if (nranks < 1 || nranks > hg::kMaxPeerOutputs + 1 || rank < 0 || rank >= nranks || !C_ranks) {
        return HGEMM_ERR_INVALID_VALUE;
    }
    if (M < 0 || N < 0 || K < 0 || row_begin < 0 || row_end < row_begin || row_end > M) {
        return HGEMM_ERR_INVALID_VALUE;
    }
    for (int i = 0; i < nranks; ++i) {
        if (!C_ranks[i]) return HGEMM_ERR_INVALID_VALUE;
        if (reinterpret_cast<uintptr_t>(C_ranks[i]) & 15u) return HGEMM_ERR_ALIGNMENT;
    }
    if (row_end == row_begin || N == 0) return HGEMM_OK;
    if (!A) return HGEMM_ERR_INVALID_VALUE;
    const size_t row_bytes = static_cast<size_t>(N) * 2;
    const uint8_t* a = static_cast<const uint8_t*>(A) + static_cast<size_t>(row_begin) * K;
    void* local = static_cast<uint8_t*>(C_ranks[rank]) + static_cast<size_t>(row_begin) * row_bytes;
    void* peers[hg::kMaxPeerOutputs];
    int n = 0;
    for (int i = 0; i < nranks; ++i) {
        if (i != rank) peers[n++] = static_cast<uint8_t*>(C_ranks[i]) + static_cast<size_t>(row_begin) * row_bytes;
    }
    return hg::run_gemm(a, B, local, row_end - row_begin, N, K, d_scale_a, d_scale_b,
                        reinterpret_cast<cudaStream_t>(stream), 0, HGEMM_SCHEDULE_DATA_PARALLEL, nullptr, 0, peers, n);
}

}  // extern "C"

namespace hg {
namespace {

// Streams and events of the host-buffer pipeline, kept per host thread and device so that a
// call does not create and destroy them (and two threads never share them).
constexpr int kMaxPanels = 4;
struct HostPipe {
    bool ready = false;
    cudaStream_t s_in = nullptr, s_mm = nullptr, s_out = nullptr;
    cudaEvent_t ev_start = nullptr, ev_done = nullptr;
    cudaEvent_t ev_in[2 * kMaxPanels] = {};  // one per arriving panel
    cudaEvent_t ev_mm[2 * kMaxPanels] = {};  // one per rectangle computed
};
thread_local HostPipe t_pipes[kMaxDevices];

HostPipe* host_pipe(int dev) {
    HostPipe& hp = t_pipes[dev];
    if (hp.ready) return &hp;
    bool ok = cudaStreamCreateWithFlags(&hp.s_in, cudaStreamNonBlocking) == cudaSuccess &&
              cudaStreamCreateWithFlags(&hp.s_mm, cudaStreamNonBlocking) == cudaSuccess &&
              cudaStreamCreateWithFlags(&hp.s_out, cudaStreamNonBlocking) == cudaSuccess &&
              cudaEventCreateWithFlags(&hp.ev_start, cudaEventDisableTiming) == cudaSuccess &&
              cudaEventCreateWithFlags(&hp.ev_done, cudaEventDisableTiming) == cudaSuccess;
    for (int i = 0; ok && i < 2 * kMaxPanels; ++i) {
        ok = cudaEventCreateWithFlags(&hp.ev_in[i], cudaEventDisableTiming) == cudaSuccess &&
             cudaEventCreateWithFlags(&hp.ev_mm[i], cudaEventDisableTiming) == cudaSuccess;
    }
    if (!ok) {
        cudaGetLastError();
        return nullptr;  // (partially created objects are kept for the next attempt's leak-free retry)
    }
    hp.ready = true;
    return &hp;
}

// Panel boundaries of n rows: up to kMaxPanels panels of equal size in multiples of 256 rows
// (whole pair tiles), at least 512 rows each.
int split_panels(int n, int* bounds) {
    const int want = std::max(1, std::min(kMaxPanels, n / 512));
    const int step = ((n + want - 1) / want + 255) / 256 * 256;
    int k = 0;
    for (int b = 0; b < n; b += step) bounds[k++] = b;
    bounds[k] = n;
    return k;
}

}  // namespace
}  // namespace hg

extern "C" {

int hgemm_fp8_tn_from_host(const void* A_host, const void* B_host, void* C_host, int M, int N, int K,
                           const float* h_scales, void* d_A, void* d_B, void* d_C, float* d_scales,
                           hgemm_stream_t stream) {
    const int rc0 = hg::check_args(d_A, d_B, d_C, M, N, K, 0, HGEMM_SCHEDULE_AUTO);
    if (rc0 != HGEMM_OK) return rc0;
    if (M == 0 || N == 0) return HGEMM_OK;
    if (!C_host || (K > 0 && (!A_host || !B_host)) || (h_scales && !d_scales)) return HGEMM_ERR_INVALID_VALUE;
    int rc = HGEMM_OK;
    const hg::DeviceState* dev = hg::current_device_setup(&rc);
    if (!dev) return rc;
    hg::HostPipe* hp = hg::host_pipe(static_cast<int>(dev - hg::g_devices));
    if (!hp) return HGEMM_ERR_CUDA;
    const cudaStream_t user = reinterpret_cast<cudaStream_t>(stream);

    // A arrives in row panels and B in column panels (rows of B), alternately, on one stream.
    // Each arrival makes one new rectangle of C computable: a new A panel against every B panel
    // already in, or a new B panel against every A panel already in.  That rectangle is one
    // GEMM on a second stream and one 2-D copy back to C_host on a third, so both copy
    // directions stay busy.  Measured at 8192^3 on B200 over PCIe: 4 panels per operand 3.67 ms,
    // against 3.73 ms for 8 and 3.90 ms for 16 (more, smaller GEMMs and copies), and 3.73 ms
    // for the earlier scheme of one GEMM per 2048 x 2048 block.
    int rb[hg::kMaxPanels + 1], cb[hg::kMaxPanels + 1];
    const int pm = hg::split_panels(M, rb), pn = hg::split_panels(N, cb);
    auto fail = [&](int code) {
        cudaGetLastError();
        return code;
    };

    // Everything starts after the work already queued on the caller's stream.
    bool ok = cudaEventRecord(hp->ev_start, user) == cudaSuccess &&
              cudaStreamWaitEvent(hp->s_in, hp->ev_start, 0) == cudaSuccess &&
              cudaStreamWaitEvent(hp->s_mm, hp->ev_start, 0) == cudaSuccess &&
              cudaStreamWaitEvent(hp->s_out, hp->ev_start, 0) == cudaSuccess;
    if (ok && h_scales) {
        ok = cudaMemcpyAsync(d_scales, h_scales, 2 * sizeof(float), cudaMemcpyHostToDevice, hp->s_in) == cudaSuccess;
    }

    const uint8_t* ha = static_cast<const uint8_t*>(A_host);
    const uint8_t* hb = static_cast<const uint8_t*>(B_host);
    uint8_t* da = static_cast<uint8_t*>(d_A);
    uint8_t* db = static_cast<uint8_t*>(d_B);
    uint8_t* dc = static_cast<uint8_t*>(d_C);
    uint8_t* hc = static_cast<uint8_t*>(C_host);
    const float* sa = h_scales ? d_scales : nullptr;
    const float* sb = h_scales ? d_scales + 1 : nullptr;
    const size_t ldc_bytes = static_cast<size_t>(N) * 2;

    int na = 0, nbp = 0, arrival = 0;
    while (ok && (na < pm || nbp < pn)) {
        const bool take_a = na < pm && (na <= nbp || nbp >= pn);
        const int* bounds = take_a ? rb : cb;
        const int idx = take_a ? na : nbp;
        const size_t off = static_cast<size_t>(bounds[idx]) * K;
        const size_t bytes = static_cast<size_t>(bounds[idx + 1] - bounds[idx]) * K;
        if (bytes) {
            ok = cudaMemcpyAsync((take_a ? da : db) + off, (take_a ? ha : hb) + off, bytes, cudaMemcpyHostToDevice,
                                 hp->s_in) == cudaSuccess;
        }
        ok = ok && cudaEventRecord(hp->ev_in[arrival], hp->s_in) == cudaSuccess &&
             cudaStreamWaitEvent(hp->s_mm, hp->ev_in[arrival], 0) == cudaSuccess;
        if (take_a) ++na; else ++nbp;
        // The newly computable rectangle: rows [r0, r1) x columns [c0, c1).
        const int r0 = take_a ? rb[na - 1] : 0, r1 = take_a ? rb[na] : rb[na];
        const int c0 = take_a ? 0 : cb[nbp - 1], c1 = take_a ? cb[nbp] : cb[nbp];
        if (ok && r1 > r0 && c1 > c0) {
            rc = hg::run_gemm(da + static_cast<size_t>(r0) * K, db + static_cast<size_t>(c0) * K,
                              dc + static_cast<size_t>(r0) * ldc_bytes + static_cast<size_t>(c0) * 2, r1 - r0, c1 - c0,
                              K, sa, sb, hp->s_mm, 0, HGEMM_SCHEDULE_DATA_PARALLEL, nullptr, 0, nullptr, 0, N);
            if (rc != HGEMM_OK) break;
            cudaEvent_t e = hp->ev_mm[arrival];
            ok = cudaEventRecord(e, hp->s_mm) == cudaSuccess && cudaStreamWaitEvent(hp->s_out, e, 0) == cudaSuccess &&
                 cudaMemcpy2DAsync(hc + static_cast<size_t>(r0) * ldc_bytes + static_cast<size_t>(c0) * 2, ldc_bytes,
                                   dc + static_cast<size_t>(r0) * ldc_bytes + static_cast<size_t>(c0) * 2, ldc_bytes,
                                   static_cast<size_t>(c1 - c0) * 2, static_cast<size_t>(r1 - r0),
                                   cudaMemcpyDeviceToHost, hp->s_out) == cudaSuccess;
        }
        ++arrival;
    }
    // The caller's stream resumes once every rectangle is back on the host.  The copy stream
    // also orders after the GEMM stream (K == 0 or empty rectangles leave nothing to copy).
    ok = ok && cudaEventRecord(hp->ev_done, hp->s_mm) == cudaSuccess &&
         cudaStreamWaitEvent(hp->s_out, hp->ev_done, 0) == cudaSuccess &&
         cudaEventRecord(hp->ev_done, hp->s_out) == cudaSuccess && cudaStreamWaitEvent(user, hp->ev_done, 0) == cudaSuccess;
    if (rc != HGEMM_OK) return fail(rc);
    return ok ? HGEMM_OK : fail(HGEMM_ERR_CUDA);
}

int hgemm_ipc_export(const void* ptr, void* handle_out, size_t* offset_out) {
    if (!ptr || !handle_out || !offset_out) return HGEMM_ERR_INVALID_VALUE;
    int rc = HGEMM_OK;
    if (!hg::current_device_setup(&rc)) return rc;
    if (!hg::g_address_range) return HGEMM_ERR_CUDA;
    CUdeviceptr base = 0;
    size_t size = 0;
    if (hg::g_address_range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) return HGEMM_ERR_CUDA;
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)) != cudaSuccess) {
        cudaGetLastError();
        return HGEMM_ERR_CUDA;
    }
    std::memcpy(handle_out, &h, sizeof(h));
    *offset_out = static_cast<size_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
    return HGEMM_OK;
}

int hgemm_ipc_import(const void* handle, void** base_out) {
    if (!handle || !base_out) return HGEMM_ERR_INVALID_VALUE;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    if (cudaIpcOpenMemHandle(base_out, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        cudaGetLastError();
        return HGEMM_ERR_CUDA;
    }
    return HGEMM_OK;
}

int hgemm_ipc_close(void* base) {
    if (!base) return HGEMM_ERR_INVALID_VALUE;
    if (cudaIpcCloseMemHandle(base) != cudaSuccess) {
        cudaGetLastError();
        return HGEMM_ERR_CUDA;
    }
    return HGEMM_OK;
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
                        reinterpret_cast<cudaStream_t>(stream), 0, HGEMM_SCHEDULE_AUTO, nullptr, 0);
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

int hgemm_debug_workspace_pool_created(int device) {
    if (device < 0 || device >= hg::kMaxDevices) return HGEMM_ERR_INVALID_VALUE;
    hg::DeviceState& st = hg::g_devices[device];
    std::lock_guard<std::mutex> lock(st.pool_mutex);
    return st.pool ? 1 : 0;
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

// ---- allocation-free stream-K entry point -------------------------------------------------
//
// Some callers may not allocate device memory at all: a serving engine that has already
// handed every byte of the GPU to its own allocator, a plugin host whose policy forbids
// driver allocations, or a latency-critical path that cannot afford cudaMalloc's implicit
// device-wide synchronisation.  hgemm_fp8_tn_static_scratch gives them the stream-K
// schedule with its scratch in a fixed array that lives in this file.

namespace hg {
namespace {

// 8 MiB per GPU, reserved by every GPU that loads this library until the process exits.
constexpr size_t kStaticScratchBytes = static_cast<size_t>(8) << 20;
static __device__ __align__(256) uint8_t g_static_scratch[kStaticScratchBytes];

struct StaticScratch {
    std::mutex mutex;
    void* ptr = nullptr;  // device address of g_static_scratch on this device, once looked up
};
StaticScratch g_static_scratch_ptrs[kMaxDevices];

// The array's device address on device `d` (current), looked up on the first call that
// succeeds; a failed lookup is not cached, so a later call retries it.
void* static_scratch_address(int d) {
    StaticScratch& st = g_static_scratch_ptrs[d];
    std::lock_guard<std::mutex> lock(st.mutex);
    if (!st.ptr) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_static_scratch) == cudaSuccess && p) {
            st.ptr = p;
        } else {
            cudaGetLastError();
        }
    }
    return st.ptr;
}

}  // namespace
}  // namespace hg

extern "C" int hgemm_fp8_tn_static_scratch(const void* A, const void* B, void* C, int M, int N, int K,
                                           const float* d_scale_a, const float* d_scale_b, hgemm_stream_t stream) {
    int rc = hg::check_args(A, B, C, M, N, K, 0, HGEMM_SCHEDULE_STREAM_K);
    if (rc != HGEMM_OK || M == 0 || N == 0) return rc;
    const hg::DeviceState* dev = hg::current_device_setup(&rc);
    if (!dev) return rc;
    int d = -1;
    if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= hg::kMaxDevices) {
        cudaGetLastError();
        return HGEMM_ERR_NO_DEVICE;
    }
    // In host code g_static_scratch names a host-side stand-in, not device memory: the
    // device address comes from cudaGetSymbolAddress, once per device, with it current.
    void* const scratch = hg::static_scratch_address(d);
    if (!scratch) return HGEMM_ERR_CUDA;
    if (K > 0) {
        const int c = hg::choose_config(M, N, K, *dev, false);
        const hg::Schedule sc = hg::make_schedule(M, N, K, c, HGEMM_SCHEDULE_STREAM_K, *dev);
        if (sc.partial_bytes + sc.counter_bytes > hg::kStaticScratchBytes) return HGEMM_ERR_UNSUPPORTED;
    }
    // run_gemm zeroes the tile counters in the scratch (cudaMemsetAsync on `stream`) before
    // the launch; the partial tiles are always written before they are read.  With a
    // workspace given, run_gemm never touches the library's workspace pool.
    return hg::run_gemm(A, B, C, M, N, K, d_scale_a, d_scale_b, reinterpret_cast<cudaStream_t>(stream), 0,
                        HGEMM_SCHEDULE_STREAM_K, scratch, hg::kStaticScratchBytes);
}
