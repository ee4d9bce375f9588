// FP8 e4m3 TN GEMM for sm_100a: C[M,N] (bf16) = scale_a * scale_b * A[M,K] . B[N,K]^T,
// fp32 accumulation in tensor memory.
//
// Replaces the reference's CDNA4 kernel fp8_gemm_4wave_256x256x128<M,N,K>
// (fp8_4wave.hpp:334-567).  Same operands and layout (A row-major M x K, B_T row-major
// N x K, C row-major M x N), but built the Blackwell way:
//   * TMA 2-D tiled loads with 128-byte swizzle into a STAGES-deep shared-memory ring
//     (replaces buffer_load...lds + the XOR swizzle of fp8_4wave.hpp:80-177);
//   * one warp issues tcgen05.mma kind::f8f6f4 (M=128, N=BN, K=32) accumulating in
//     tensor memory (replaces the 16x16x128 MFMA register tiles, :24-74, and the
//     LDS->VGPR fragment loads, :179-212);
//   * warp specialisation with mbarrier hand-off (producer / MMA / 4 epilogue warps)
//     instead of the hand-interleaved 4-wave schedule (:244-332, :428-463);
//   * a persistent grid walks output tiles in GROUP_M-grouped raster order, the
//     analogue of the reference's WGM=4 L2 swizzle (:357-377);
//   * two accumulator buffers in tensor memory so the epilogue of tile i overlaps the
//     MMAs of tile i+1; the epilogue scales, rounds to bf16 (RNE, where the reference
//     truncates, :214-217) and writes through shared memory with TMA stores, which clip
//     ragged M/N edges (the reference requires M%256 == N%256 == 0 and K%128 == 0).
#pragma once

#include <cuda.h>
#include <cstdint>

#include "ptx.cuh"

namespace hg {

struct GemmParams {
    int M, N, K;
    int num_m_blocks, num_n_blocks, num_k_blocks;
    int group_m;  // tile rows per raster group
    const float* scale_a;  // device pointers, nullptr = 1.0
    const float* scale_b;
};

// Status codes recorded by an expired bounded wait: role << 8 | site.
enum : uint32_t {
    kErrProducerEmpty = 0x0101,
    kErrMmaTmemEmpty = 0x0201,
    kErrMmaFull = 0x0202,
    kErrMmaDrain = 0x0203,
    kErrEpiTmemFull = 0x0301,
};

// Output tile -> (m block, n block) with GROUP_M tile rows per raster group: inside a
// group the walk goes down the rows first, then across the columns, so the CTAs that
// run at the same time share both A row panels and B column panels in L2.
__device__ __forceinline__ void tile_coords(int tile, const GemmParams& p, int& mb, int& nb) {
    const int per_group = p.group_m * p.num_n_blocks;
    const int group = tile / per_group;
    const int first_m = group * p.group_m;
    const int rows_in_group = min(p.num_m_blocks - first_m, p.group_m);
    const int r = tile - group * per_group;
    mb = first_m + r % rows_in_group;
    nb = r / rows_in_group;
}

template <int BN, int STAGES>
struct GemmConfig {
    static constexpr int BM = 128;
    static constexpr int BK = 128;  // bytes of K per stage = one 128-byte swizzle row
    static constexpr int UMMA_K = 32;
    static constexpr int kNumThreads = 192;  // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
    static constexpr int A_BYTES = BM * BK;
    static constexpr int B_BYTES = BN * BK;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int EPI_COLS = 64;                 // bf16 columns per staged chunk (128 B)
    static constexpr int EPI_BUF_BYTES = 32 * EPI_COLS * 2;  // one warp's 32 rows x 128 B
    static constexpr int OFF_A = 0;
    static constexpr int OFF_B = OFF_A + STAGES * A_BYTES;
    static constexpr int OFF_EPI = OFF_B + STAGES * B_BYTES;
    static constexpr int OFF_BAR = OFF_EPI + 4 * 2 * EPI_BUF_BYTES;
    static constexpr int NUM_BARS = 2 * STAGES + 5;  // full, empty, tmem_full x2, tmem_empty x2, drain
    static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
    static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;  // + slack to align the base to 1024 B
    static constexpr uint32_t TMEM_COLS = 2 * BN < 32 ? 32 : 2 * BN;
    static constexpr uint32_t IDESC = idesc_e4m3_f32(BM, BN);
    static_assert(BN % 64 == 0 && BN >= 64 && BN <= 256, "BN must be 64, 128, 192 or 256");
    static_assert((TMEM_COLS & (TMEM_COLS - 1)) == 0, "tensor memory allocations are powers of two");
    static_assert(SMEM_BYTES <= 232448, "exceeds 227 KB of shared memory per CTA");
};

template <int BN, int STAGES>
__global__ void __launch_bounds__(192, 1)
    fp8_gemm_tn_sm100(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                      const __grid_constant__ CUtensorMap tm_c, const GemmParams p) {
    using Cfg = GemmConfig<BN, STAGES>;
    extern __shared__ uint8_t smem_raw[];
    // 128-byte swizzle atoms need 1024-byte alignment.
    const uint32_t raw_base = smem_u32(smem_raw);
    const uint32_t base = (raw_base + 1023u) & ~1023u;
    uint8_t* const smem_gen = smem_raw + (base - raw_base);

    const uint32_t warp = threadIdx.x / 32;
    const uint32_t lane = threadIdx.x % 32;

    const uint32_t bar_full = base + Cfg::OFF_BAR;
    const uint32_t bar_empty = bar_full + STAGES * 8;
    const uint32_t bar_tfull = bar_empty + STAGES * 8;
    const uint32_t bar_tempty = bar_tfull + 2 * 8;
    const uint32_t bar_drain = bar_tempty + 2 * 8;
    const uint32_t tmem_slot = base + Cfg::OFF_MISC;
    volatile uint32_t* const tmem_slot_ptr = reinterpret_cast<volatile uint32_t*>(smem_gen + Cfg::OFF_MISC);
    volatile uint32_t* const abort_flag = reinterpret_cast<volatile uint32_t*>(smem_gen + Cfg::OFF_MISC + 4);

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(bar_full + 8 * s, 1);
            mbar_init(bar_empty + 8 * s, 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(bar_tfull + 8 * a, 1);
            mbar_init(bar_tempty + 8 * a, 128);
        }
        mbar_init(bar_drain, 1);
        *abort_flag = 0u;
        fence_mbarrier_init();
        fence_proxy_async_smem();
        prefetch_tmap(&tm_a);
        prefetch_tmap(&tm_b);
        prefetch_tmap(&tm_c);
    }
    if (warp == 1) {
        tmem_alloc<1>(tmem_slot, Cfg::TMEM_COLS);
        tmem_relinquish<1>();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot_ptr;

    const int num_tiles = p.num_m_blocks * p.num_n_blocks;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
                int mb, nb;
                tile_coords(tile, p, mb, nb);
                for (int kb = 0; kb < p.num_k_blocks; ++kb) {
                    if (!mbar_wait(bar_empty + 8 * stage, phase ^ 1u, abort_flag, kErrProducerEmpty)) {
                        ok = false;
                        break;
                    }
                    const uint32_t full = bar_full + 8 * stage;
                    mbar_arrive_expect_tx(full, Cfg::STAGE_BYTES);
                    tma_load_2d(base + Cfg::OFF_A + stage * Cfg::A_BYTES, &tm_a, kb * Cfg::BK, mb * Cfg::BM, full);
                    tma_load_2d(base + Cfg::OFF_B + stage * Cfg::B_BYTES, &tm_b, kb * Cfg::BK, nb * BN, full);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            // On abort, give copies already in flight time to land before the CTA exits.
            if (!ok) sleep_ns_bounded(1000000);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (one thread) ----------------
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
                if (!mbar_wait(bar_tempty + 8 * acc, acc_phase ^ 1u, abort_flag, kErrMmaTmemEmpty)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
                for (int kb = 0; kb < p.num_k_blocks; ++kb) {
                    if (!mbar_wait(bar_full + 8 * stage, phase, abort_flag, kErrMmaFull)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t a_desc = sw128_kmajor_desc(base + Cfg::OFF_A + stage * Cfg::A_BYTES);
                    const uint64_t b_desc = sw128_kmajor_desc(base + Cfg::OFF_B + stage * Cfg::B_BYTES);
#pragma unroll
                    for (int k = 0; k < Cfg::BK / Cfg::UMMA_K; ++k) {
                        // Advancing the start address by 32 B walks K inside the swizzle
                        // atom: the hardware applies the XOR pattern to the final address.
                        const uint64_t koff = static_cast<uint64_t>((k * Cfg::UMMA_K) >> 4);
                        mma_f8f6f4<1>(d_tmem, a_desc + koff, b_desc + koff, Cfg::IDESC, (kb | k) != 0 ? 1u : 0u);
                    }
                    mma_commit<1>(bar_empty + 8 * stage);  // frees the stage when these MMAs finish
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                mma_commit<1>(bar_tfull + 8 * acc);  // accumulator ready for the epilogue
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
            if (!ok) {
                // Let MMAs already issued finish before tensor memory is released.
                mma_commit<1>(bar_drain);
                volatile uint32_t never = 0;
                mbar_wait(bar_drain, 0, &never, kErrMmaDrain);
            }
        }
    } else {
        // ---------------- epilogue: 4 warps, TMEM -> regs -> smem -> TMA store ----------------
        const uint32_t quad = warp % 4;  // tensor-memory lanes [32*quad, 32*quad + 32)
        const uint32_t epi_idx = warp - 2;
        const float sa = p.scale_a ? *p.scale_a : 1.0f;
        const float sb = p.scale_b ? *p.scale_b : 1.0f;
        const float s = sa * sb;
        const uint32_t stage_base = base + Cfg::OFF_EPI + epi_idx * 2 * Cfg::EPI_BUF_BYTES;
        int acc = 0;
        uint32_t acc_phase = 0;
        uint32_t chunk_ctr = 0;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
            int mb, nb;
            tile_coords(tile, p, mb, nb);
            // Warp-uniform decision: the tcgen05.ld below is .sync.aligned.
            const bool ready = mbar_wait(bar_tfull + 8 * acc, acc_phase, abort_flag, kErrEpiTmemFull);
            if (!__all_sync(0xffffffffu, ready)) break;
            tc_fence_after();
            const int row0 = mb * Cfg::BM + static_cast<int>(quad) * 32;
#pragma unroll 1
            for (int c = 0; c < BN / Cfg::EPI_COLS; ++c) {
                uint32_t v[64];
                const uint32_t taddr = tmem_base + ((quad * 32u) << 16) + static_cast<uint32_t>(acc * BN + c * 64);
                tmem_ld_32x32b_x32(taddr, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
                tmem_ld_32x32b_x32(taddr + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
                tmem_ld_wait();
                uint32_t packed[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    packed[j] = pack_bf16x2_rn(__fmul_rn(__uint_as_float(v[2 * j]), s),
                                               __fmul_rn(__uint_as_float(v[2 * j + 1]), s));
                }
                const uint32_t buf = chunk_ctr & 1u;
                // The store issued two chunks ago read this buffer; wait until it has.
                if (lane == 0) bulk_wait_group_read<1>();
                __syncwarp();
                const uint32_t row_addr = stage_base + buf * Cfg::EPI_BUF_BYTES + lane * 128u;
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const uint32_t slot = static_cast<uint32_t>(q) ^ (lane & 7u);  // 128-byte swizzle
                    st_shared_v4(row_addr + slot * 16u, packed[4 * q], packed[4 * q + 1], packed[4 * q + 2],
                                 packed[4 * q + 3]);
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    const int col0 = nb * BN + c * Cfg::EPI_COLS;
                    if (row0 < p.M && col0 < p.N) {
                        tma_store_2d(&tm_c, col0, row0, stage_base + buf * Cfg::EPI_BUF_BYTES);
                    }
                    bulk_commit_group();
                }
                ++chunk_ctr;
            }
            tc_fence_before();
            mbar_arrive(bar_tempty + 8 * acc);
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
        if (lane == 0) bulk_wait_group<0>();
        __syncwarp();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc<1>(tmem_base, Cfg::TMEM_COLS);
    }
}


// ======================================================================================
// CTA-pair variant (cta_group::2): a cluster of two CTAs on two SMs computes one
// 256 x BN output tile with M=256 tcgen05.mma instructions issued by the even CTA.
// Each CTA stages its own half of A (128 rows) and its own half of B (BN/2 rows) per
// K block, so per-SM operand traffic per MAC is a third lower than the 128 x 256
// single-CTA tile (32 KB instead of 48 KB per 4 M MACs per SM); each CTA's tensor
// memory receives its 128 rows of the accumulator and each CTA runs its own epilogue.
//
// Synchronisation without any multicast form: tcgen05.commit always targets a barrier
// of the issuing (even) CTA, and the even CTA forwards each completion to its peer with
// a remote mbarrier.arrive (release.cluster) that the peer acquires at cluster scope:
//   full[s]    even CTA only; expects both CTAs' TMA bytes (the odd CTA's loads name
//              the even CTA's barrier through mapa and the cta_group::2 TMA form);
//   empty[s]   even: MMA commit; odd: forwarded by the even producer after its own wait;
//   tfull[a]   even: MMA commit; odd: forwarded by the even CTA's first epilogue warp;
//   tempty[a]  even CTA only; one arrive per epilogue warp of both CTAs (count 8).
// ======================================================================================

template <int BN, int STAGES>
struct PairConfig {
    static constexpr int BM = 256;       // pair tile rows (128 per CTA)
    static constexpr int BK = 128;
    static constexpr int UMMA_K = 32;
    static constexpr int kNumThreads = 192;
    static constexpr int A_BYTES = 128 * BK;        // this CTA's half of A
    static constexpr int B_BYTES = (BN / 2) * BK;   // this CTA's half of B
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int EPI_COLS = 64;
    static constexpr int EPI_BUF_BYTES = 32 * EPI_COLS * 2;
    static constexpr int OFF_A = 0;
    static constexpr int OFF_B = OFF_A + STAGES * A_BYTES;
    static constexpr int OFF_EPI = OFF_B + STAGES * B_BYTES;
    static constexpr int OFF_BAR = OFF_EPI + 4 * 2 * EPI_BUF_BYTES;
    static constexpr int NUM_BARS = 2 * STAGES + 5;
    static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
    static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;
    static constexpr uint32_t TMEM_COLS = 2 * BN;
    static constexpr uint32_t IDESC = idesc_e4m3_f32(BM, BN);
    static_assert(BN == 128 || BN == 256, "pair tiles are 256 x 128 or 256 x 256");
    static_assert(((BN / 2) * BK) % 1024 == 0, "B half-tile must keep 1024-byte alignment");
    static_assert(SMEM_BYTES <= 232448, "exceeds 227 KB of shared memory per CTA");
};

template <int BN, int STAGES>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(192, 1)
    fp8_gemm_tn_sm100_pair(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                           const __grid_constant__ CUtensorMap tm_c, const GemmParams p) {
    using Cfg = PairConfig<BN, STAGES>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_base = smem_u32(smem_raw);
    const uint32_t base = (raw_base + 1023u) & ~1023u;
    uint8_t* const smem_gen = smem_raw + (base - raw_base);

    const uint32_t warp = threadIdx.x / 32;
    const uint32_t lane = threadIdx.x % 32;
    const uint32_t rank = cluster_ctarank();  // 0 = even CTA (issues the MMAs), 1 = odd
    const uint32_t peer = rank ^ 1u;
    const bool leader = rank == 0;

    const uint32_t bar_full = base + Cfg::OFF_BAR;
    const uint32_t bar_empty = bar_full + STAGES * 8;
    const uint32_t bar_tfull = bar_empty + STAGES * 8;
    const uint32_t bar_tempty = bar_tfull + 2 * 8;
    const uint32_t bar_drain = bar_tempty + 2 * 8;
    const uint32_t tmem_slot = base + Cfg::OFF_MISC;
    volatile uint32_t* const tmem_slot_ptr = reinterpret_cast<volatile uint32_t*>(smem_gen + Cfg::OFF_MISC);
    volatile uint32_t* const abort_flag = reinterpret_cast<volatile uint32_t*>(smem_gen + Cfg::OFF_MISC + 4);

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(bar_full + 8 * s, 1);
            mbar_init(bar_empty + 8 * s, 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(bar_tfull + 8 * a, 1);
            mbar_init(bar_tempty + 8 * a, 8);
        }
        mbar_init(bar_drain, 1);
        *abort_flag = 0u;
        fence_mbarrier_init();
        fence_proxy_async_smem();
        prefetch_tmap(&tm_a);
        prefetch_tmap(&tm_b);
        prefetch_tmap(&tm_c);
    }
    if (warp == 1) {
        tmem_alloc<2>(tmem_slot, Cfg::TMEM_COLS);  // collective with the peer's warp 1
        tmem_relinquish<2>();
    }
    tc_fence_before();
    cluster_sync();  // barriers of both CTAs initialised, tensor memory allocated
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot_ptr;

    const int num_tiles = p.num_m_blocks * p.num_n_blocks;
    const int pair_id = static_cast<int>(blockIdx.x >> 1);
    const int num_pairs = static_cast<int>(gridDim.x >> 1);

    if (warp == 0) {
        // ---------------- TMA producer (both CTAs) ----------------
        if (lane == 0) {
            const uint32_t full_leader0 = mapa_shared(bar_full, 0);
            const uint32_t peer_empty0 = mapa_shared(bar_empty, peer);
            int stage = 0;
            uint32_t phase = 0;
            bool first_pass = true;
            bool ok = true;
            for (int tile = pair_id; tile < num_tiles && ok; tile += num_pairs) {
                int mb, nb;
                tile_coords(tile, p, mb, nb);
                const int a_row = mb * Cfg::BM + static_cast<int>(rank) * 128;
                const int b_row = nb * BN + static_cast<int>(rank) * (BN / 2);
                for (int kb = 0; kb < p.num_k_blocks; ++kb) {
                    if (!mbar_wait<true>(bar_empty + 8 * stage, phase ^ 1u, abort_flag, kErrProducerEmpty)) {
                        ok = false;
                        break;
                    }
                    const uint32_t a_dst = base + Cfg::OFF_A + stage * Cfg::A_BYTES;
                    const uint32_t b_dst = base + Cfg::OFF_B + stage * Cfg::B_BYTES;
                    if (leader) {
                        // The MMAs that read this stage have finished in both CTAs: tell the peer.
                        if (!first_pass) mbar_arrive_cluster(peer_empty0 + 8 * stage);
                        const uint32_t full = bar_full + 8 * stage;
                        mbar_arrive_expect_tx(full, 2 * Cfg::STAGE_BYTES);
                        tma_load_2d(a_dst, &tm_a, kb * Cfg::BK, a_row, full);
                        tma_load_2d(b_dst, &tm_b, kb * Cfg::BK, b_row, full);
                    } else {
                        const uint32_t full = full_leader0 + 8 * stage;
                        tma_load_2d_pair(a_dst, &tm_a, kb * Cfg::BK, a_row, full);
                        tma_load_2d_pair(b_dst, &tm_b, kb * Cfg::BK, b_row, full);
                    }
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                        first_pass = false;
                    }
                }
            }
            if (!ok) sleep_ns_bounded(1000000);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (even CTA, one thread) ----------------
        if (leader && lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            for (int tile = pair_id; tile < num_tiles && ok; tile += num_pairs) {
                if (!mbar_wait<true>(bar_tempty + 8 * acc, acc_phase ^ 1u, abort_flag, kErrMmaTmemEmpty)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
                for (int kb = 0; kb < p.num_k_blocks; ++kb) {
                    if (!mbar_wait<true>(bar_full + 8 * stage, phase, abort_flag, kErrMmaFull)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t a_desc = sw128_kmajor_desc(base + Cfg::OFF_A + stage * Cfg::A_BYTES);
                    const uint64_t b_desc = sw128_kmajor_desc(base + Cfg::OFF_B + stage * Cfg::B_BYTES);
#pragma unroll
                    for (int k = 0; k < Cfg::BK / Cfg::UMMA_K; ++k) {
                        const uint64_t koff = static_cast<uint64_t>((k * Cfg::UMMA_K) >> 4);
                        mma_f8f6f4<2>(d_tmem, a_desc + koff, b_desc + koff, Cfg::IDESC, (kb | k) != 0 ? 1u : 0u);
                    }
                    mma_commit<2>(bar_empty + 8 * stage);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                mma_commit<2>(bar_tfull + 8 * acc);
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
            if (!ok) {
                mma_commit<2>(bar_drain);
                volatile uint32_t never = 0;
                mbar_wait(bar_drain, 0, &never, kErrMmaDrain);
            }
        }
    } else {
        // ---------------- epilogue (both CTAs): own 128 rows x BN ----------------
        const uint32_t quad = warp % 4;
        const uint32_t epi_idx = warp - 2;
        const float sa = p.scale_a ? *p.scale_a : 1.0f;
        const float sb = p.scale_b ? *p.scale_b : 1.0f;
        const float s = sa * sb;
        const uint32_t stage_base = base + Cfg::OFF_EPI + epi_idx * 2 * Cfg::EPI_BUF_BYTES;
        const uint32_t peer_tfull0 = mapa_shared(bar_tfull, peer);
        const uint32_t leader_tempty0 = mapa_shared(bar_tempty, 0);
        int acc = 0;
        uint32_t acc_phase = 0;
        uint32_t chunk_ctr = 0;
        for (int tile = pair_id; tile < num_tiles; tile += num_pairs) {
            int mb, nb;
            tile_coords(tile, p, mb, nb);
            const bool ready = mbar_wait<true>(bar_tfull + 8 * acc, acc_phase, abort_flag, kErrEpiTmemFull);
            if (!__all_sync(0xffffffffu, ready)) break;
            if (leader && epi_idx == 0 && lane == 0) mbar_arrive_cluster(peer_tfull0 + 8 * acc);
            tc_fence_after();
            const int row0 = mb * Cfg::BM + static_cast<int>(rank) * 128 + static_cast<int>(quad) * 32;
#pragma unroll 1
            for (int c = 0; c < BN / Cfg::EPI_COLS; ++c) {
                uint32_t v[64];
                const uint32_t taddr = tmem_base + ((quad * 32u) << 16) + static_cast<uint32_t>(acc * BN + c * 64);
                tmem_ld_32x32b_x32(taddr, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
                tmem_ld_32x32b_x32(taddr + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
                tmem_ld_wait();
                uint32_t packed[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    packed[j] = pack_bf16x2_rn(__fmul_rn(__uint_as_float(v[2 * j]), s),
                                               __fmul_rn(__uint_as_float(v[2 * j + 1]), s));
                }
                const uint32_t buf = chunk_ctr & 1u;
                if (lane == 0) bulk_wait_group_read<1>();
                __syncwarp();
                const uint32_t row_addr = stage_base + buf * Cfg::EPI_BUF_BYTES + lane * 128u;
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const uint32_t slot = static_cast<uint32_t>(q) ^ (lane & 7u);
                    st_shared_v4(row_addr + slot * 16u, packed[4 * q], packed[4 * q + 1], packed[4 * q + 2],
                                 packed[4 * q + 3]);
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    const int col0 = nb * BN + c * Cfg::EPI_COLS;
                    if (row0 < p.M && col0 < p.N) {
                        tma_store_2d(&tm_c, col0, row0, stage_base + buf * Cfg::EPI_BUF_BYTES);
                    }
                    bulk_commit_group();
                }
                ++chunk_ctr;
            }
            // All lanes' tensor-memory reads are complete (wait::ld); release the buffer.
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if (leader) {
                    mbar_arrive(bar_tempty + 8 * acc);
                } else {
                    mbar_arrive_cluster(leader_tempty0 + 8 * acc);
                }
            }
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
        if (lane == 0) bulk_wait_group<0>();
        __syncwarp();
    }

    tc_fence_before();
    cluster_sync();  // no CTA leaves while its peer may still signal its barriers
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc<2>(tmem_base, Cfg::TMEM_COLS);
    }
}

}  // namespace hg
