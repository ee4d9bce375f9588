// FP8 e4m3 TN GEMM for sm_100a: C[M,N] (bf16) = scale_a * scale_b * A[M,K] . B[N,K]^T,
// fp32 accumulation in tensor memory.
//
// Replaces the reference's CDNA4 kernel fp8_gemm_4wave_256x256x128<M,N,K>
// (fp8_4wave.hpp:334-567).  Same operands and layout (A row-major M x K, B_T row-major
// N x K, C row-major M x N), but built the Blackwell way:
//   * TMA 2-D tiled loads with 128-byte swizzle into a STAGES-deep shared-memory ring
//     (replaces buffer_load...lds + the XOR swizzle of fp8_4wave.hpp:80-177);
//   * one thread issues tcgen05.mma kind::f8f6f4 (K=32 per instruction) accumulating in
//     tensor memory (replaces the 16x16x128 MFMA register tiles, :24-74, and the
//     LDS->VGPR fragment loads, :179-212);
//   * warp specialisation with mbarrier hand-off (producer / MMA / 4 epilogue warps)
//     instead of the hand-interleaved 4-wave schedule (:244-332, :428-463);
//   * a persistent grid walks output tiles in GROUP_M-grouped raster order, the
//     analogue of the reference's WGM=4 L2 swizzle (:357-377), and splits the last
//     one-to-two waves of tiles along K across all slots ("stream-K") so short or
//     wave-quantised problems keep every SM busy;
//   * two accumulator buffers in tensor memory so the epilogue of tile i overlaps the
//     MMAs of tile i+1; the epilogue scales, rounds to bf16 (RNE, where the reference
//     truncates, :214-217) and writes through shared memory with TMA stores, which clip
//     ragged M/N edges (the reference requires M%256 == N%256 == 0 and K%128 == 0).
//
// One kernel template covers two shapes of the work:
//   CTAS = 1: one CTA computes a 128 x BN tile with M=128 MMAs;
//   CTAS = 2: a cluster of two CTAs on two SMs computes a 256 x BN tile with M=256
//             MMAs (cta_group::2) issued by the even CTA.  Each CTA stages its own 128
//             rows of A and BN/2 rows of B per K block, so per-SM operand traffic per
//             MAC is a third lower than the 128 x 256 single-CTA tile; each CTA's tensor
//             memory holds its 128 accumulator rows and each CTA runs its own epilogue.
//
// MX = true is the OCP MX variant: tcgen05.mma kind::mxf8f6f4.block_scale, with one e8m0
// scale per 32 K elements of every row of A and B (the reference's MFMA builtin is this
// instruction with its scales fixed at 2^0, fp8_4wave.hpp:53-58).  Each stage also carries
// the K block's scale-factor atoms (two 3-D TMA boxes per CTA, on the operand barrier); the
// MMA thread copies them into per-stage tensor-memory columns with tcgen05.cp before the
// block's four MMAs.  For BN = 256 the scale factors take the columns a second accumulator
// would use, so there is one accumulator and the epilogue releases it as soon as the tile is
// drained (EARLY_RELEASE).
//
// SPLIT > 1 is split-K over a cluster of SPLIT single CTAs, for problems whose tiles would
// leave most SMs idle (a 128-row M with long K): CTA r of a cluster computes K part r of the
// cluster's tile, and the CTAs exchange partial rows through distributed shared memory (bulk
// copies into each other's idle stage rings) so that each finishes 128 / SPLIT rows.
//
// CTA-pair synchronisation uses no multicast form: tcgen05.commit always targets a
// barrier of the even CTA, and the even CTA forwards each completion to its peer with a
// remote mbarrier.arrive that the peer acquires at cluster scope:
//   full[s]    even CTA only; expects both CTAs' TMA bytes (the odd CTA's loads name the
//              even CTA's barrier through mapa and the cta_group::2 TMA form);
//   empty[s]   even: MMA commit; odd: forwarded by the even producer after its own wait;
//   tfull[a]   even: MMA commit; odd: forwarded by the even CTA's first epilogue warp;
//   tempty[a]  even CTA only; one arrive per epilogue warp of both CTAs (count 8).
#pragma once

#include <cuda.h>
#include <cstdint>

#include "ptx.cuh"

namespace hg {

struct GemmParams {
    int M, N, K;
    int num_m_blocks, num_n_blocks, num_k_blocks;
    int group_m;           // tile rows per raster group
    const float* scale_a;  // device pointers, nullptr = 1.0
    const float* scale_b;
    // Hybrid schedule.  The first dp_tiles tiles (raster order) are whole-tile items dealt
    // round-robin to the slots (CTAs, or CTA pairs).  The last sk_tiles tiles are cut into
    // k-block units; slot s < sk_slots owns units [sk_begin(s), sk_begin(s + 1)).  A tile
    // shared by several slots is reduced by whichever contributor finishes last: each one
    // writes its fp32 partial to `partials`, then bumps the tile's counter.
    int dp_tiles;
    int sk_tiles;
    int sk_slots;
    float* partials;  // [slot][piece 0/1][cta][128 x BN] fp32 (layout: partial_offset)
    int* counters;    // [sk tile][cta]; zero on entry, left zero on exit
    // MX block scaling (the MX kernels only): e8m0 scale factors, one per 32 K elements of a
    // row, in 512-byte atoms of 128 rows x 4 K-groups (byte 16*(r%32) + 4*(r/32) + g),
    // atom (row block i, K block j) at offset (i * sf_k_atoms + j) * 512, read through the
    // SfMaps tensor maps.
    int sf_k_atoms;
    // Split-K clusters (the SPLIT > 1 kernels only; 1 otherwise): CTA r of each cluster of
    // split_k CTAs computes K blocks [r KB / split_k, (r + 1) KB / split_k) of tile
    // blockIdx.x / split_k, and the cluster sums the partials through distributed shared memory.
    int split_k;
    // Test hook (hgemm_debug_stalled_gemm only): the producer registers the first stage's
    // bytes but issues no copies for it, so that stage never fills and every role's bounded
    // wait expires; the kernel then records a status, drains and returns.
    int debug_stall_first_stage;
};

// MX scale factors as 3-D TMA tensors over the blocked bytes: x = 128 bytes, y = 128-byte
// rows along K (4 per 512-byte atom, 4 * ceil(K/128) per row block), z = 128-row block
// (stride ceil(K/128) * 512 bytes).  A box of 4 rows by 1 (A) or BN / 128 (B) row blocks
// fetches one K block's atoms in one load; blocks past M or N read as zeros (the MX kernels
// only; zero otherwise).
struct SfMaps {
    CUtensorMap a;
    CUtensorMap b;
};
constexpr int kSfRowsPerAtom = 4;

// Extra outputs for the fused all-gather: the same C rows on other GPUs (peer memory
// mapped into this process), written by TMA stores of the same staged tiles.
constexpr int kMaxPeerOutputs = 7;
struct PeerOutputs {
    CUtensorMap maps[kMaxPeerOutputs];
    // The same outputs as C stores of 128-row boxes (one CTA's rows at once): wide[0] is this
    // GPU's C, wide[1 + i] peer i's (so wide[d] for destination d = 0 .. count).  Whole
    // data-parallel tiles are stored through these.
    CUtensorMap wide[kMaxPeerOutputs + 1];
    int count;
};

// Status codes recorded by an expired bounded wait: role << 8 | site.
enum : uint32_t {
    kErrProducerEmpty = 0x0101,
    kErrMmaTmemEmpty = 0x0201,
    kErrMmaFull = 0x0202,
    kErrMmaDrain = 0x0203,
    kErrEpiTmemFull = 0x0301,
    kErrSplitFull = 0x0303,  // split-K: the peers' partial columns never all arrived
};

// Output tile -> (m block, n block) with GROUP_M tile rows per raster group: inside a
// group the walk goes down the rows first, then across the columns, so the CTAs that
// run at the same time share both A row panels and B column panels in L2.
__host__ __device__ __forceinline__ void tile_coords(int tile, const GemmParams& p, int& mb, int& nb) {
    const int per_group = p.group_m * p.num_n_blocks;
    const int group = tile / per_group;
    const int first_m = group * p.group_m;
    const int rows_in_group = p.num_m_blocks - first_m < p.group_m ? p.num_m_blocks - first_m : p.group_m;
    const int r = tile - group * per_group;
    mb = first_m + r % rows_in_group;
    nb = r / rows_in_group;
    // Odd groups walk the columns backwards, so a group starts on the B panels its
    // predecessor used last, still in L2 (measured at 8192^3: DRAM reads 238 -> 227 MB per
    // launch; 16384 x 28672 x 8192: 1455 -> 1423 MB).
    if (group & 1) nb = p.num_n_blocks - 1 - nb;
}

struct Work {
    int tile;      // raster tile index
    int kb_begin;  // k blocks [kb_begin, kb_end) of that tile
    int kb_end;
    int piece;     // -1: the whole tile (store C directly); 0/1: this slot's first/last partial
};

__host__ __device__ __forceinline__ long long sk_begin(const GemmParams& p, int s) {
    return static_cast<long long>(s) * (static_cast<long long>(p.sk_tiles) * p.num_k_blocks) / p.sk_slots;
}

// Item `idx` (0-based) of slot `slot` out of `nslots`; false once the slot has no more.
// Every role of a CTA (and both CTAs of a pair) walks the same sequence:
//   1. this slot's partial stream-K pieces (at most two: the tail of its first tile,
//      piece 0, and the head of its last tile, piece 1), so that the reductions of
//      shared tiles run while the MMAs continue with whole tiles;
//   2. whole tiles of its stream-K range;
//   3. its data-parallel tiles slot, slot + nslots, ...
// Split-K clusters (p.split_k > 1) instead: one item per CTA, its K part of one tile (piece 2).
__host__ __device__ __forceinline__ bool get_work(const GemmParams& p, int slot, int nslots, int idx, Work& w) {
    const int KB = p.num_k_blocks;
    if (p.split_k > 1) {
        if (idx > 0) return false;
        // 32-bit arithmetic: KB < 2^24 and split_k <= 4 (a 64-bit divide is a long subroutine).
        const int part = slot % p.split_k;
        w.tile = slot / p.split_k;
        w.kb_begin = part * KB / p.split_k;
        w.kb_end = (part + 1) * KB / p.split_k;
        w.piece = 2;
        return w.tile < p.dp_tiles;
    }
    int n_part = 0, n_full = 0, t_first = 0, t_last = -1;
    long long u0 = 0, u1 = 0;
    bool first_partial = false, last_partial = false;
    if (slot < p.sk_slots) {
        u0 = sk_begin(p, slot);
        u1 = sk_begin(p, slot + 1);
        if (u1 > u0) {
            t_first = static_cast<int>(u0 / KB);
            t_last = static_cast<int>((u1 - 1) / KB);
            const long long first_end = t_first == t_last ? u1 : static_cast<long long>(t_first + 1) * KB;
            first_partial = u0 != static_cast<long long>(t_first) * KB || first_end != static_cast<long long>(t_first + 1) * KB;
            last_partial = t_last != t_first && u1 != static_cast<long long>(t_last + 1) * KB;
            n_part = (first_partial ? 1 : 0) + (last_partial ? 1 : 0);
            n_full = (t_last - t_first + 1) - n_part;
        }
    }
    if (idx < n_part) {
        const bool first = first_partial && idx == 0;
        const int t = first ? t_first : t_last;
        w.tile = p.dp_tiles + t;
        w.kb_begin = first ? static_cast<int>(u0 - static_cast<long long>(t) * KB) : 0;
        w.kb_end = (first && t_first != t_last) ? KB : static_cast<int>(u1 - static_cast<long long>(t) * KB);
        if (!first) w.kb_end = static_cast<int>(u1 - static_cast<long long>(t) * KB);
        w.piece = first ? 0 : 1;
        return true;
    }
    idx -= n_part;
    if (idx < n_full) {
        w.tile = p.dp_tiles + t_first + (first_partial ? 1 : 0) + idx;
        w.kb_begin = 0;
        w.kb_end = KB;
        w.piece = -1;
        return true;
    }
    idx -= n_full;
    const int dp_count = p.dp_tiles > slot ? (p.dp_tiles - slot + nslots - 1) / nslots : 0;
    if (idx < dp_count) {
        w.tile = slot + idx * nslots;
        w.kb_begin = 0;
        w.kb_end = KB;
        w.piece = -1;
        return true;
    }
    return false;
}

// The stream-K slot whose unit range contains unit u (u < sk_tiles * num_k_blocks).
__host__ __device__ __forceinline__ int sk_slot_of_unit(const GemmParams& p, long long u) {
    const long long U = static_cast<long long>(p.sk_tiles) * p.num_k_blocks;
    int s = static_cast<int>(u * p.sk_slots / U);
    while (s + 1 < p.sk_slots && sk_begin(p, s + 1) <= u) ++s;
    while (s > 0 && sk_begin(p, s) > u) --s;
    return s;
}

// Float offset, inside one 128 x BN partial, of columns [32*c32 + 4*j4, +4) of the row
// that thread (quad, lane) owns.  Lanes are the fastest-varying index, so the 32 lanes
// of a warp access 512 contiguous bytes for each (c32, j4): full-line transactions.
template <int BN>
__device__ __forceinline__ uint32_t partial_offset(uint32_t quad, uint32_t c32, uint32_t j4, uint32_t lane) {
    return (((quad * (BN / 32) + c32) * 8u + j4) * 32u + lane) * 4u;
}

__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Barrier over `count` threads that also ANDs a predicate across them.
__device__ __forceinline__ bool named_bar_all(uint32_t id, uint32_t count, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred pi, po;\n\t"
        "setp.ne.u32 pi, %1, 0;\n\t"
        "bar.red.and.pred po, %2, %3, pi;\n\t"
        "selp.u32 %0, 1, 0, po;\n\t}\n"
        : "=r"(r)
        : "r"(static_cast<uint32_t>(pred)), "r"(id), "r"(count)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ void st_global_v4(float* p, float a, float b, float c, float d) {
    asm volatile("st.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}

// KBS: K blocks per stage.  With KBS = 2 every operand arrives in one TMA load per two K
// blocks (a 3-D box of 128-byte K chunks: two 16-byte-aligned swizzled K-block tiles back to
// back), and the MX scale factors of both K blocks in one box each: half the TMA instructions
// per K block, which matters because each costs the TMA unit a fixed time whatever its size.
// SPLIT > 1: split-K over a cluster of SPLIT single CTAs (see the epilogue).
template <int CTAS, int BN, int STAGES, bool MX = false, int KBS = 1, int SPLIT = 1>
struct KernelShape {
    static constexpr int BM = 128 * CTAS;   // output tile rows
    static constexpr int BK = 128;          // bytes of K per K block = one 128-byte swizzle row
    static constexpr int UMMA_K = 32;
    static constexpr int kNumThreads = 192;  // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
    static constexpr int B_ROWS = BN / CTAS;  // rows of B this CTA stages per K block
    static constexpr int KB_A_BYTES = 128 * BK;  // one K block of this CTA's A rows
    static constexpr int KB_B_BYTES = B_ROWS * BK;
    static constexpr int A_BYTES = KBS * KB_A_BYTES;  // per stage
    static constexpr int B_BYTES = KBS * KB_B_BYTES;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    // MX with BN > 128: the scale factors need tensor-memory columns that a second
    // accumulator would take, so there is one accumulator, and the epilogue frees it as soon
    // as the tile sits in registers (bf16), before its stores.
    static constexpr int ACC_BUFS = (MX && BN > 128) ? 1 : 2;
    static constexpr bool EARLY_RELEASE = ACC_BUFS == 1;
    // MX: per stage, with the operands and on the same barriers (scale factors are
    // latency-bound: they need the stage ring's full depth), KBS 512-byte atoms for this
    // CTA's 128 rows of A (one per K block), then KBS per 128 columns of the whole tile (a
    // pair's CTAs both hold all of B's), column block major: two loads per stage.
    static constexpr int SFB_ATOMS = (BN + 127) / 128;
    static constexpr int SF_BYTES = MX ? 512 * (1 + SFB_ATOMS) * KBS : 0;
    // full, empty, tfull x2, tempty x2, drain (+ split-K: peers' partials in)
    static constexpr int NUM_BARS = 2 * STAGES + 5 + (SPLIT > 1 ? 1 : 0);
    // bf16 columns per staged epilogue chunk: 64 (128-byte rows, 128-byte swizzle) when
    // BN allows and the staging fits beside the stage ring, else 32 (64-byte rows, 64-byte
    // swizzle; also the one-accumulator MX tile, to fit four stages).
    static constexpr bool EPI64_FITS =
        STAGES * (STAGE_BYTES + SF_BYTES) + 8 * 32 * 64 * 2 + NUM_BARS * 8 + 16 + 1024 <= 232448;
    static constexpr int EPI_COLS = (BN % 64 == 0 && !EARLY_RELEASE && EPI64_FITS && SPLIT == 1) ? 64 : 32;
    static constexpr int EPI_BUF_BYTES = 32 * EPI_COLS * 2;  // one warp's 32 rows
    static constexpr int OFF_A = 0;
    static constexpr int OFF_B = OFF_A + STAGES * A_BYTES;
    static constexpr int OFF_EPI = OFF_B + STAGES * B_BYTES;
    static constexpr int OFF_RECV = OFF_EPI + 4 * 2 * EPI_BUF_BYTES;  // split-K receive region
    static constexpr int OFF_SF = OFF_RECV + (SPLIT > 1 ? (SPLIT - 1) * 4 * (BN / SPLIT / 32) * 4096 : 0);
    static constexpr int OFF_BAR = OFF_SF + STAGES * SF_BYTES;
    static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
    static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;  // + slack to align the base to 1024 B
    // ACC_BUFS accumulators of BN fp32 columns, plus (MX) one set of scale-factor columns (4
    // per 128 rows of A and of B), rounded up to the power of two tcgen05.alloc takes.  Every
    // K block's copies reuse the same columns: tcgen05.cp and tcgen05.mma execute in issue
    // order, so a copy lands only after the MMAs issued before it have read the previous
    // block's factors (measured at 8192^3: 602 K cycles against 627 K with one set per K block
    // of the ring).
    static constexpr int SF_COLS = MX ? 4 * (1 + SFB_ATOMS) : 0;
    static constexpr int OFF_SF_COL = ACC_BUFS * BN;
    static constexpr int COLS_USED = ACC_BUFS * BN + SF_COLS;
    static constexpr uint32_t TMEM_COLS =
        COLS_USED <= 32 ? 32 : (COLS_USED <= 64 ? 64 : (COLS_USED <= 128 ? 128 : (COLS_USED <= 256 ? 256 : 512)));
    static constexpr uint32_t IDESC = idesc_e4m3_f32(BM, BN);
    static constexpr int PARTIAL_FLOATS = 128 * BN;  // one CTA's share of a partial tile
    static_assert(CTAS == 1 || CTAS == 2, "one CTA or a CTA pair");
    static_assert(!MX || BN % 128 == 0, "MX tiles cover whole 128-row scale-factor atoms of B");
    static_assert(COLS_USED <= 512, "tensor memory holds 512 columns");
    static_assert(BN % 32 == 0 && BN >= 64 && BN <= 256, "BN must be a multiple of 32 in [64, 256]");
    static_assert(CTAS == 1 || BN % 16 == 0, "M=256 MMAs need N % 16 == 0");
    static_assert(KB_B_BYTES % 1024 == 0, "B tiles must keep 1024-byte alignment");
    static_assert(KBS == 1 || KBS == 2, "one or two K blocks per stage");
    // Split-K: each CTA of the cluster finishes OWN_COLS columns of the tile (all 128 rows, so
    // all four epilogue warps share the work).  As soon as its own MMAs are done, each warp
    // stages its 32 rows of every other rank's columns in its (now idle) stage ring and sends
    // them with one bulk copy per owner into the owner's dedicated receive region:
    //   [RECV_OFF, + RECV_BYTES): one SLOT_BYTES block per (peer, warp quad), peers in rank order
    //   without the owner itself; a block holds OWN_CH chunks of 32 rows x 32 fp32 columns.
    // Inside a 4 KB chunk, row r's 16-byte unit u sits at unit u ^ (r & 7): eight lanes (rows)
    // touching the same unit hit eight different bank groups.
    static constexpr int OWN_COLS = BN / SPLIT;
    static constexpr int OWN_CH = OWN_COLS / 32;
    static constexpr int SPLIT_CHUNK_BYTES = 32 * 32 * 4;
    static constexpr int SLOT_BYTES = OWN_CH * SPLIT_CHUNK_BYTES;
    static constexpr int RECV_BYTES = SPLIT > 1 ? (SPLIT - 1) * 4 * SLOT_BYTES : 0;
    static constexpr uint32_t SPLIT_TX_BYTES = static_cast<uint32_t>(RECV_BYTES);
    static_assert(SPLIT == 1 || SPLIT == 2 || SPLIT == 4, "split-K clusters of 2 or 4");
    static_assert(SPLIT == 1 || (CTAS == 1 && !MX), "split-K: single-CTA plain tiles");
    static_assert(SPLIT == 1 || BN % (32 * SPLIT) == 0, "split-K owners take whole 32-column chunks");
    static_assert(RECV_BYTES <= STAGES * STAGE_BYTES, "the send staging lives in the stage ring");
    static_assert(SPLIT == 1 || (OWN_CH <= 2 && EPI_BUF_BYTES == 32 * 32 * 2), "split-K stores 32 x 32 chunks");
    static_assert((TMEM_COLS & (TMEM_COLS - 1)) == 0, "tensor memory allocations are powers of two");
    static_assert(SMEM_BYTES <= 232448, "exceeds 227 KB of shared memory per CTA");
};

// KBS = 2 reads A and B through 3-D maps (x = 128 bytes of K, y = row, z = 128-byte K chunk);
// KBS = 1 through 2-D maps (x = K byte, y = row).
template <int CTAS, int BN, int STAGES, bool MX = false, int KBS = 1, int SPLIT = 1>
__global__ void __launch_bounds__(192, 1)
    fp8_gemm_tn_sm100(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                      const __grid_constant__ CUtensorMap tm_c, const GemmParams p,
                      const __grid_constant__ PeerOutputs peers, const __grid_constant__ SfMaps sfm) {
    using S = KernelShape<CTAS, BN, STAGES, MX, KBS, SPLIT>;
    extern __shared__ uint8_t smem_raw[];
    // 128-byte swizzle atoms need 1024-byte alignment.
    const uint32_t raw_base = smem_u32(smem_raw);
    const uint32_t base = (raw_base + 1023u) & ~1023u;
    uint8_t* const smem_gen = smem_raw + (base - raw_base);

    const uint32_t warp = threadIdx.x / 32;
    const uint32_t lane = threadIdx.x % 32;
    const uint32_t rank = CTAS == 2 ? cluster_ctarank() : 0u;  // 0 issues the MMAs
    const uint32_t peer = rank ^ 1u;
    const bool leader = rank == 0;
    constexpr bool kPair = CTAS == 2;

    const uint32_t bar_full = base + S::OFF_BAR;
    const uint32_t bar_empty = bar_full + STAGES * 8;
    const uint32_t bar_tfull = bar_empty + STAGES * 8;
    const uint32_t bar_tempty = bar_tfull + 2 * 8;
    const uint32_t bar_drain = bar_tempty + 2 * 8;
    const uint32_t bar_skfull = bar_drain + 8;  // split-K: this CTA's columns in from every peer (tx bytes)
    const uint32_t tmem_slot = base + S::OFF_MISC;
    volatile uint32_t* const tmem_slot_ptr = reinterpret_cast<volatile uint32_t*>(smem_gen + S::OFF_MISC);
    volatile uint32_t* const abort_flag = reinterpret_cast<volatile uint32_t*>(smem_gen + S::OFF_MISC + 4);
    volatile int* const bcast = reinterpret_cast<volatile int*>(smem_gen + S::OFF_MISC + 8);

    const int slot = static_cast<int>(blockIdx.x) / CTAS;
    const int nslots = static_cast<int>(gridDim.x) / CTAS;

    // Set-up, spread over three warps.  On an SM that has not run this code yet, the first
    // pass through it and the first reads of the kernel parameters cost about a microsecond
    // of instruction and constant fetches; the producer spends that time working out its first
    // work item while another warp initialises the barriers, so its first copies go out as
    // soon as griddep_wait returns.
    if (warp == 2 && lane == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(bar_full + 8 * s, 1);
            mbar_init(bar_empty + 8 * s, 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(bar_tfull + 8 * a, 1);
            mbar_init(bar_tempty + 8 * a, kPair ? 8 : 4);  // one arrive per epilogue warp
        }
        mbar_init(bar_drain, 1);
        if constexpr (SPLIT > 1) {
            mbar_init(bar_skfull, 1);
        }
        *abort_flag = 0u;
        fence_mbarrier_init();
        fence_proxy_async_smem();
    }
    Work w_first{};
    bool have_first = false;
    int mb_first = 0, nb_first = 0;
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tm_a);
        prefetch_tmap(&tm_b);
        prefetch_tmap(&tm_c);
        prefetch_tmap(&peers.wide[0]);
        if constexpr (MX) {
            prefetch_tmap(&sfm.a);
            prefetch_tmap(&sfm.b);
        }
        have_first = get_work(p, slot, nslots, 0, w_first);
        if (have_first) tile_coords(w_first.tile, p, mb_first, nb_first);
    }
    if (warp == 1) {
        // The MMA issuer's first work item, for the same reason as the producer's.
        if (lane == 0) have_first = get_work(p, slot, nslots, 0, w_first);
        tmem_alloc<CTAS>(tmem_slot, S::TMEM_COLS);  // for a pair: collective with the peer's warp 1
        tmem_relinquish<CTAS>();
    }
    tc_fence_before();
    if constexpr (kPair || SPLIT > 1) {
        cluster_sync();  // every CTA's barriers initialised (peers signal them), tensor memory allocated
    } else {
        __syncthreads();
    }
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot_ptr;
    // Everything above (barriers, tensor memory, descriptor prefetch) may overlap the previous
    // kernel's tail; global memory is read and written only after it has finished.
    griddep_launch_dependents();
    griddep_wait();

    if (warp == 0) {
        // ---------------- TMA producer (one thread per CTA) ----------------
        if (lane == 0) {
            const uint32_t full_leader0 = kPair ? mapa_shared(bar_full, 0) : bar_full;
            const uint32_t peer_empty0 = kPair ? mapa_shared(bar_empty, peer) : 0u;
            int stage = 0;
            uint32_t phase = 0;
            bool first_pass = true;
            bool ok = true;
            Work w = w_first;
            bool have = have_first;
            for (int idx = 0; ok && have; ++idx, have = get_work(p, slot, nslots, idx, w)) {
                int mb = mb_first, nb = nb_first;
                if (idx > 0) tile_coords(w.tile, p, mb, nb);
                const int a_row = mb * S::BM + static_cast<int>(rank) * 128;
                const int b_row = nb * BN + static_cast<int>(rank) * S::B_ROWS;
                for (int kb = w.kb_begin; kb < w.kb_end; kb += KBS) {
                    if (!mbar_wait<kPair>(bar_empty + 8 * stage, phase ^ 1u, abort_flag, kErrProducerEmpty)) {
                        ok = false;
                        break;
                    }
                    const uint32_t a_dst = base + S::OFF_A + stage * S::A_BYTES;
                    const uint32_t b_dst = base + S::OFF_B + stage * S::B_BYTES;
                    // MX: the stage's scale factors, A's for this CTA's 128 rows and B's for all
                    // of the tile's columns (full boxes: rows past M or N, or K blocks past K,
                    // read as zeros; so does the second K block of a stage past K).
                    const uint32_t sf_dst = base + S::OFF_SF + stage * S::SF_BYTES;
                    const int a_blk = mb * CTAS + static_cast<int>(rank);
                    const int b_blk = nb * S::SFB_ATOMS;
                    const int sf_y = kb * kSfRowsPerAtom;
                    // (Test hook: the first stage's bytes are expected but never copied.)
                    const bool stall = p.debug_stall_first_stage && idx == 0 && kb == w.kb_begin;
                    if (leader) {
                        // For a pair: the MMAs that read this stage finished in both CTAs.
                        if (kPair && !first_pass) mbar_arrive_cluster(peer_empty0 + 8 * stage);
                        const uint32_t full = bar_full + 8 * stage;
                        mbar_arrive_expect_tx(full, CTAS * (S::STAGE_BYTES + S::SF_BYTES));
                        if (!stall) {
                            if constexpr (KBS == 1) {
                                tma_load_2d(a_dst, &tm_a, kb * S::BK, a_row, full);
                                tma_load_2d(b_dst, &tm_b, kb * S::BK, b_row, full);
                            } else {
                                tma_load_3d(a_dst, &tm_a, 0, a_row, kb, full);
                                tma_load_3d(b_dst, &tm_b, 0, b_row, kb, full);
                            }
                            if constexpr (MX) {
                                tma_load_3d(sf_dst, &sfm.a, 0, sf_y, a_blk, full);
                                tma_load_3d(sf_dst + 512 * KBS, &sfm.b, 0, sf_y, b_blk, full);
                            }
                        }
                    } else if (!stall) {
                        const uint32_t full = full_leader0 + 8 * stage;
                        if constexpr (KBS == 1) {
                            tma_load_2d_pair(a_dst, &tm_a, kb * S::BK, a_row, full);
                            tma_load_2d_pair(b_dst, &tm_b, kb * S::BK, b_row, full);
                        } else {
                            tma_load_3d_pair(a_dst, &tm_a, 0, a_row, kb, full);
                            tma_load_3d_pair(b_dst, &tm_b, 0, b_row, kb, full);
                        }
                        if constexpr (MX) {
                            tma_load_3d_pair(sf_dst, &sfm.a, 0, sf_y, a_blk, full);
                            tma_load_3d_pair(sf_dst + 512 * KBS, &sfm.b, 0, sf_y, b_blk, full);
                        }
                    }
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                        first_pass = false;
                    }
                }
            }
            // On abort, give copies already in flight time to land before the CTA exits.
            if (!ok) sleep_ns_bounded(1000000);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (one thread of the even CTA) ----------------
        if (leader && lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            // MX: the scale factors of K block h of stage s go to the scale-factor columns (at
            // tsfa) with tcgen05.cp, which runs in issue order with the MMAs that read them.  In
            // shared memory A's atom of K block h is at 512 h, B's atom of column block c at
            // 512 (KBS (1 + c) + h).
            auto issue_sf_cp = [&](int s, int h, uint32_t tsfa) {
                const uint32_t sf_src = base + S::OFF_SF + s * S::SF_BYTES;
                tmem_cp_32x128b_warpx4<CTAS>(tsfa, sf_smem_desc(sf_src + 512 * h));
#pragma unroll
                for (int c = 0; c < S::SFB_ATOMS; ++c) {
                    tmem_cp_32x128b_warpx4<CTAS>(tsfa + 4 * (1 + c), sf_smem_desc(sf_src + 512 * (KBS * (1 + c) + h)));
                }
            };
            Work w = w_first;
            bool have = have_first;
            for (int idx = 0; ok && have; ++idx, have = get_work(p, slot, nslots, idx, w)) {
                if (!mbar_wait<kPair>(bar_tempty + 8 * acc, acc_phase ^ 1u, abort_flag, kErrMmaTmemEmpty)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
                for (int kb = w.kb_begin; kb < w.kb_end; kb += KBS) {
                    if (!mbar_wait<kPair>(bar_full + 8 * stage, phase, abort_flag, kErrMmaFull)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
#pragma unroll
                    for (int h = 0; h < KBS; ++h) {
                        if (h > 0 && kb + h >= w.kb_end) break;  // a stage's second K block past the range
                        const uint64_t a_desc =
                            sw128_kmajor_desc(base + S::OFF_A + stage * S::A_BYTES + h * S::KB_A_BYTES);
                        const uint64_t b_desc =
                            sw128_kmajor_desc(base + S::OFF_B + stage * S::B_BYTES + h * S::KB_B_BYTES);
                        if constexpr (MX) {
                            // Scale factors of this K block: A's at tsfa (4 columns), B's after them.
                            const uint32_t tsfa = tmem_base + static_cast<uint32_t>(S::OFF_SF_COL);
                            const uint32_t tsfb = tsfa + 4;
                            issue_sf_cp(stage, h, tsfa);
#pragma unroll
                            for (int k = 0; k < S::BK / S::UMMA_K; ++k) {
                                const uint64_t koff = static_cast<uint64_t>((k * S::UMMA_K) >> 4);
                                const uint32_t accumulate = (kb + h > w.kb_begin || k > 0) ? 1u : 0u;
                                // K slice k uses byte k of each scale-factor column.
                                const uint32_t sf_id = static_cast<uint32_t>(k);
                                mma_mxf8f6f4<CTAS>(d_tmem, a_desc + koff, b_desc + koff,
                                                   idesc_mx_e4m3(S::BM, BN, sf_id), tsfa | (sf_id << 30),
                                                   tsfb | (sf_id << 30), accumulate);
                            }
                        } else {
#pragma unroll
                            for (int k = 0; k < S::BK / S::UMMA_K; ++k) {
                                // Advancing the start address by 32 B walks K inside the swizzle
                                // atom: the hardware applies the XOR pattern to the final address.
                                const uint64_t koff = static_cast<uint64_t>((k * S::UMMA_K) >> 4);
                                const uint32_t accumulate = (kb + h > w.kb_begin || k > 0) ? 1u : 0u;
                                mma_f8f6f4<CTAS>(d_tmem, a_desc + koff, b_desc + koff, S::IDESC, accumulate);
                            }
                        }
                    }
                    mma_commit<CTAS>(bar_empty + 8 * stage);  // frees the stage when these MMAs finish
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                mma_commit<CTAS>(bar_tfull + 8 * acc);  // accumulator ready for the epilogue
                if (++acc == S::ACC_BUFS) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
            if (!ok) {
                // Let MMAs already issued finish before tensor memory is released.
                mma_commit<CTAS>(bar_drain);
                volatile uint32_t never = 0;
                mbar_wait(bar_drain, 0, &never, kErrMmaDrain);
            }
        }
    } else {
        // ------- epilogue: 4 warps, this CTA's 128 rows x BN: TMEM -> regs -> smem -> TMA store -------
        const uint32_t quad = warp % 4;  // tensor-memory lanes [32*quad, 32*quad + 32)
        const uint32_t epi_idx = warp - 2;
        const uint32_t epi_tid = epi_idx * 32 + lane;
        const float sa = p.scale_a ? *p.scale_a : 1.0f;
        const float sb = p.scale_b ? *p.scale_b : 1.0f;
        const float s = sa * sb;
        const uint32_t stage_base = base + S::OFF_EPI + epi_idx * 2 * S::EPI_BUF_BYTES;
        const uint32_t peer_tfull0 = kPair ? mapa_shared(bar_tfull, peer) : 0u;
        const uint32_t leader_tempty0 = kPair ? mapa_shared(bar_tempty, 0) : 0u;
        int acc = 0;
        uint32_t acc_phase = 0;
        uint32_t chunk_ctr = 0;

        constexpr int EC = S::EPI_COLS;

        // Stage EC bf16 values (packed pairs) of this thread's row in this warp's
        // double-buffered 32 x EC tile and TMA-store it at (row0, col0).
        auto store_packed = [&](const uint32_t* packed, int row0, int col0) {
            const uint32_t buf = chunk_ctr & 1u;
            // The store issued two chunks ago read this buffer; wait until it has.
            if (lane == 0) bulk_wait_group_read<1>();
            __syncwarp();
            const uint32_t row_addr = stage_base + buf * S::EPI_BUF_BYTES + lane * (EC * 2u);
#pragma unroll
            for (int q = 0; q < EC / 8; ++q) {
                // 16-byte group q of row `lane` in the TMA swizzle: 128-byte mode XORs with
                // row % 8, 64-byte mode with (row / 2) % 4 (address bits [7:9] / [7:8]).
                const uint32_t slot16 = EC == 64 ? (static_cast<uint32_t>(q) ^ (lane & 7u))
                                                 : (static_cast<uint32_t>(q) ^ ((lane >> 1) & 3u));
                st_shared_v4(row_addr + slot16 * 16u, packed[4 * q], packed[4 * q + 1], packed[4 * q + 2],
                             packed[4 * q + 3]);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                if (row0 < p.M && col0 < p.N) {
                    const uint32_t src = stage_base + buf * S::EPI_BUF_BYTES;
                    tma_store_2d(&tm_c, col0, row0, src);
                    // Fused all-gather: the same tile into every peer's copy of these rows.
                    for (int i = 0; i < peers.count; ++i) tma_store_2d(&peers.maps[i], col0, row0, src);
                }
                bulk_commit_group();  // an empty group when the store was skipped keeps the count exact
            }
            ++chunk_ctr;
        };

        // CTA-wide stores (whole data-parallel tiles): the four epilogue warps stage one
        // EC-column chunk of all 128 rows of this CTA, then a single thread issues one 128-row
        // TMA store.  Issuing a TMA store costs its thread ~150 ns (measured), a quarter of what
        // four 32-row stores per chunk cost; the issuing thread rotates over the warps' lane 0s.
        // Buffers alternate per chunk; a thread that issued a store waits for it to have read
        // shared memory before the next chunk's barrier, so that the buffer is free when chunk
        // c + 2 is staged into it.
        const uint32_t wide_base = base + S::OFF_EPI;
        uint32_t wide_ctr = 0;
        auto store_wide = [&](const uint32_t* packed, int cta_row0, int col0) {
            const uint32_t buf = wide_base + (wide_ctr & 1u) * 4u * S::EPI_BUF_BYTES;
            const uint32_t row_addr = buf + quad * S::EPI_BUF_BYTES + lane * (EC * 2u);
#pragma unroll
            for (int q = 0; q < EC / 8; ++q) {
                // The swizzle of row 32 quad + lane, whose row % 8 is lane % 8.
                const uint32_t slot16 = EC == 64 ? (static_cast<uint32_t>(q) ^ (lane & 7u))
                                                 : (static_cast<uint32_t>(q) ^ ((lane >> 1) & 3u));
                st_shared_v4(row_addr + slot16 * 16u, packed[4 * q], packed[4 * q + 1], packed[4 * q + 2],
                             packed[4 * q + 3]);
            }
            fence_proxy_async_smem();
            if (lane == 0) bulk_wait_group_read<0>();  // this thread's last store has read its buffer
            named_bar_sync(2, 128);
            // Destination d (0 = this GPU's C, 1 + i = peer i's copy) goes out from warp
            // (d + chunk) % 4: with peer outputs (the fused all-gather, up to 8 destinations) the
            // four warps' lane 0s issue them in parallel.
            if (lane == 0 && cta_row0 < p.M && col0 < p.N) {
                bool issued = false;
                for (int d = static_cast<int>((epi_idx - wide_ctr) & 3u); d <= peers.count; d += 4) {
                    tma_store_2d(&peers.wide[d], col0, cta_row0, buf);
                    issued = true;
                }
                if (issued) bulk_commit_group();
            }
            ++wide_ctr;
        };

        // Scale EC fp32 accumulators of this thread's row, round to bf16 (RNE) and store.
        auto store_chunk = [&](const float (&v)[EC], int row0, int col0) {
            uint32_t packed[EC / 2];
#pragma unroll
            for (int j = 0; j < EC / 2; ++j) {
                packed[j] = pack_bf16x2_rn(__fmul_rn(v[2 * j], s), __fmul_rn(v[2 * j + 1], s));
            }
            store_packed(packed, row0, col0);
        };

        auto release_accumulator = [&]() {
            // All lanes' tensor-memory reads are complete (tcgen05.wait::ld).
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if (leader) {
                    mbar_arrive(bar_tempty + 8 * acc);
                } else {
                    mbar_arrive_cluster(leader_tempty0 + 8 * acc);
                }
            }
            if (++acc == S::ACC_BUFS) {
                acc = 0;
                acc_phase ^= 1u;
            }
        };

        Work w;
        for (int idx = 0; get_work(p, slot, nslots, idx, w); ++idx) {
            int mb, nb;
            tile_coords(w.tile, p, mb, nb);
            // One decision for all four epilogue warps (the stream-K path below has
            // barriers among them, and tcgen05.ld is .sync.aligned).
            bool ready = mbar_wait<kPair>(bar_tfull + 8 * acc, acc_phase, abort_flag, kErrEpiTmemFull);
            ready = __all_sync(0xffffffffu, ready);
            ready = named_bar_all(1, 128, ready);
            __syncwarp();
            if (!ready) break;
            if (kPair && leader && epi_idx == 0 && lane == 0) mbar_arrive_cluster(peer_tfull0 + 8 * acc);
            tc_fence_after();
            const int row0 = mb * S::BM + static_cast<int>(rank) * 128 + static_cast<int>(quad) * 32;
            const uint32_t tmem_row = tmem_base + ((quad * 32u) << 16) + static_cast<uint32_t>(acc * BN);

            if constexpr (SPLIT > 1) {
                // ---- split-K: this CTA holds K part `krank` of the whole 128 x BN tile ----
                // 1. Every warp stages its 32 rows of each other rank's OWN_COLS columns (its stage
                //    ring is idle: its MMAs are done) and sends them with one bulk copy per owner
                //    into the owner's dedicated receive region, completing the owner's barrier.
                //    No handshake: the region is never used for anything else.
                // 2. Once every peer's columns are in, each warp adds the peers' partials (rank
                //    order) and its own from tensor memory, scales, rounds and stores its 32 rows of
                //    this rank's columns.  The order is fixed, so every call gives the same bits.
                const uint32_t krank = cluster_ctarank();
                if (epi_tid == 0) mbar_arrive_expect_tx(bar_skfull, S::SPLIT_TX_BYTES);
                const bool empty_part = w.kb_begin >= w.kb_end;  // fewer K blocks than ranks: zeros
                // Byte offset of row `lane`'s 16-byte unit u inside a 32 x 32 fp32 chunk.
                auto swz = [&](uint32_t u) { return lane * 128u + (((u ^ lane) & 7u) << 4); };
                const uint32_t stage_blk = base + S::OFF_A + epi_idx * ((SPLIT - 1) * S::SLOT_BYTES);
                {
                    // Items (owner, chunk) in order; tensor-memory loads run one item ahead.
                    constexpr int NITEMS = (SPLIT - 1) * S::OWN_CH;
                    auto item_col = [&](int it) {
                        const uint32_t o_idx = static_cast<uint32_t>(it / S::OWN_CH);  // among the others
                        const uint32_t owner = o_idx < krank ? o_idx : o_idx + 1u;
                        return owner * S::OWN_COLS + static_cast<uint32_t>(it % S::OWN_CH) * 32u;
                    };
                    uint32_t ra[32], rb[32];
                    if (!empty_part) tmem_ld_32x32b_x32(tmem_row + item_col(0), ra);
#pragma unroll
                    for (int it = 0; it < NITEMS; ++it) {
                        uint32_t(&cur)[32] = (it & 1) ? rb : ra;
                        uint32_t(&nxt)[32] = (it & 1) ? ra : rb;
                        if (!empty_part) {
                            tmem_ld_wait(cur);
                            if (it + 1 < NITEMS) tmem_ld_32x32b_x32(tmem_row + item_col(it + 1), nxt);
                        }
                        const uint32_t chunk = stage_blk + static_cast<uint32_t>(it) * S::SPLIT_CHUNK_BYTES;
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            if (empty_part) {
                                st_shared_v4(chunk + swz(j), 0u, 0u, 0u, 0u);
                            } else {
                                st_shared_v4(chunk + swz(j), cur[4 * j], cur[4 * j + 1], cur[4 * j + 2], cur[4 * j + 3]);
                            }
                        }
                        if (it % S::OWN_CH == S::OWN_CH - 1) {
                            // All of this owner's chunks are staged: send them.
                            fence_proxy_async_smem();  // the staged rows are visible to the bulk copy
                            __syncwarp();
                            if (lane == 0) {
                                const uint32_t o_idx = static_cast<uint32_t>(it / S::OWN_CH);
                                const uint32_t owner = o_idx < krank ? o_idx : o_idx + 1u;
                                const uint32_t slot_at_owner = krank < owner ? krank : krank - 1u;
                                const uint32_t src = stage_blk + o_idx * S::SLOT_BYTES;
                                const uint32_t dst = mapa_shared(
                                    base + S::OFF_RECV + (slot_at_owner * 4u + quad) * S::SLOT_BYTES, owner);
                                bulk_copy_to_peer(dst, src, S::SLOT_BYTES, mapa_shared(bar_skfull, owner));
                            }
                        }
                    }
                }
                bool ok = mbar_wait<true>(bar_skfull, 0, abort_flag, kErrSplitFull);
                ok = named_bar_all(1, 128, __all_sync(0xffffffffu, ok));
                if (!ok) break;
                // This warp's rows of this rank's columns: peers' partials (rank order), then its own.
                const int out_row0 = mb * S::BM + static_cast<int>(quad) * 32;
                const uint32_t buf0 = base + S::OFF_EPI + epi_idx * 2u * S::EPI_BUF_BYTES;
                uint32_t own[32];
                if (!empty_part) tmem_ld_32x32b_x32(tmem_row + krank * S::OWN_COLS, own);
#pragma unroll
                for (int c = 0; c < S::OWN_CH; ++c) {
                    float v[32];
#pragma unroll
                    for (int sl = 0; sl < SPLIT - 1; ++sl) {
                        const uint32_t blk = base + S::OFF_RECV + (static_cast<uint32_t>(sl) * 4u + quad) * S::SLOT_BYTES +
                                             static_cast<uint32_t>(c) * S::SPLIT_CHUNK_BYTES;
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            float x0, x1, x2, x3;
                            ld_shared_v4f(blk + swz(j), x0, x1, x2, x3);
                            if (sl == 0) {
                                v[4 * j] = x0; v[4 * j + 1] = x1; v[4 * j + 2] = x2; v[4 * j + 3] = x3;
                            } else {
                                v[4 * j] += x0; v[4 * j + 1] += x1; v[4 * j + 2] += x2; v[4 * j + 3] += x3;
                            }
                        }
                    }
                    if (!empty_part) {
                        tmem_ld_wait(own);
#pragma unroll
                        for (int j = 0; j < 32; ++j) v[j] += __uint_as_float(own[j]);
                        if (c + 1 < S::OWN_CH) tmem_ld_32x32b_x32(tmem_row + krank * S::OWN_COLS + (c + 1) * 32, own);
                    }
                    // Scale, round and stage (64-byte swizzle: 16-byte group q of row `lane` at
                    // q ^ ((lane / 2) % 4)) in this warp's staging buffer c, then store.
                    const uint32_t buf = buf0 + static_cast<uint32_t>(c) * S::EPI_BUF_BYTES;
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const uint32_t slot16 = static_cast<uint32_t>(q) ^ ((lane >> 1) & 3u);
                        st_shared_v4(buf + lane * 64u + slot16 * 16u,
                                     pack_bf16x2_rn(__fmul_rn(v[8 * q], s), __fmul_rn(v[8 * q + 1], s)),
                                     pack_bf16x2_rn(__fmul_rn(v[8 * q + 2], s), __fmul_rn(v[8 * q + 3], s)),
                                     pack_bf16x2_rn(__fmul_rn(v[8 * q + 4], s), __fmul_rn(v[8 * q + 5], s)),
                                     pack_bf16x2_rn(__fmul_rn(v[8 * q + 6], s), __fmul_rn(v[8 * q + 7], s)));
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        const int col0 = nb * BN + static_cast<int>(krank) * S::OWN_COLS + c * 32;
                        if (out_row0 < p.M && col0 < p.N) {
                            tma_store_2d(&tm_c, col0, out_row0, buf);
                            for (int i = 0; i < peers.count; ++i) tma_store_2d(&peers.maps[i], col0, out_row0, buf);
                        }
                        bulk_commit_group();
                    }
                }
                continue;
            }
            if constexpr (S::EARLY_RELEASE) {
                // Drain the row as bf16, then free the accumulator for the next tile's MMAs
                // while this one is stored (data-parallel tiles only).  The first two chunks
                // go straight to the warp's two staging buffers; the rest wait in registers.
                constexpr int kDirect = 2;
                constexpr int kHeld = BN / EC - kDirect;
                uint32_t held[kHeld * (EC / 2)];
#pragma unroll
                for (int c = 0; c < BN / EC; ++c) {
                    uint32_t chunk[EC / 2];
#pragma unroll
                    for (int h = 0; h < EC / 16; ++h) {
                        uint32_t r[16];
                        tmem_ld_32x32b_x16(tmem_row + c * EC + h * 16, r);
                        tmem_ld_wait(r);
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            chunk[8 * h + j] = pack_bf16x2_rn(__fmul_rn(__uint_as_float(r[2 * j]), s),
                                                              __fmul_rn(__uint_as_float(r[2 * j + 1]), s));
                        }
                    }
                    if (c < kDirect) {
                        store_packed(chunk, row0, nb * BN + c * EC);
                    } else {
#pragma unroll
                        for (int j = 0; j < EC / 2; ++j) held[(c - kDirect) * (EC / 2) + j] = chunk[j];
                    }
                }
                release_accumulator();
#pragma unroll
                for (int c = kDirect; c < BN / EC; ++c) {
                    store_packed(&held[(c - kDirect) * (EC / 2)], row0, nb * BN + c * EC);
                }
                continue;
            }
            if (w.piece < 0) {
                // The tensor-memory loads of chunk c + 1 are in flight while chunk c is scaled,
                // rounded and stored, and the accumulator is released as soon as its last chunk
                // is in registers (before that chunk's store).
                constexpr int NCH = BN / EC;
                const int cta_row0 = mb * S::BM + static_cast<int>(rank) * 128;
                // With a stream-K schedule, partial tiles store through the per-warp buffers,
                // which overlap the CTA-wide ones: every earlier store must have read its buffer
                // before this tile stages into them.  (With peer outputs every store is per warp.)
                if (p.sk_tiles > 0 && peers.count == 0) {
                    if (lane == 0) bulk_wait_group_read<0>();
                    named_bar_sync(2, 128);
                }
                uint32_t ra[EC], rb[EC];
                auto load_chunk = [&](int c, uint32_t (&r)[EC]) {
#pragma unroll
                    for (int h = 0; h < EC / 32; ++h) {
                        tmem_ld_32x32b_x32(tmem_row + c * EC + 32 * h, *reinterpret_cast<uint32_t(*)[32]>(&r[32 * h]));
                    }
                };
                load_chunk(0, ra);
#pragma unroll
                for (int c = 0; c < NCH; ++c) {
                    uint32_t(&cur)[EC] = (c & 1) ? rb : ra;
                    uint32_t(&nxt)[EC] = (c & 1) ? ra : rb;
                    tmem_ld_wait(*reinterpret_cast<uint32_t(*)[32]>(&cur[0]));
                    if constexpr (EC == 64) reg_fence(*reinterpret_cast<uint32_t(*)[32]>(&cur[32]));
                    if (c + 1 < NCH) {
                        load_chunk(c + 1, nxt);
                    } else {
                        release_accumulator();
                    }
                    uint32_t packed[EC / 2];
#pragma unroll
                    for (int j = 0; j < EC / 2; ++j) {
                        packed[j] = pack_bf16x2_rn(__fmul_rn(__uint_as_float(cur[2 * j]), s),
                                                   __fmul_rn(__uint_as_float(cur[2 * j + 1]), s));
                    }
                    if (peers.count > 0) {
                        // The fused all-gather stores per warp (32-row boxes, every warp's lane 0
                        // issuing its own stores to every destination), so that no chunk barrier
                        // couples the four warps to the slowest NVLink store.  (Measured at 8
                        // GPUs with the 224-wide tile, per-warp and CTA-wide stores gave the
                        // same 0.35 ms per step; the 64-byte row segments of that tile were the
                        // cost, so the fused call takes 64-column tiles: 0.231 ms.)
                        store_packed(packed, row0, nb * BN + c * EC);
                    } else {
                        store_wide(packed, cta_row0, nb * BN + c * EC);
                    }
                }
                if (p.sk_tiles > 0 && peers.count == 0) {
                    if (lane == 0) bulk_wait_group_read<0>();
                    named_bar_sync(2, 128);
                }
                continue;
            }

            // ---- a partial piece of a stream-K tile ----
            float* const part_base = p.partials;
            const size_t my_part = (static_cast<size_t>(slot * 2 + w.piece) * CTAS + rank) * S::PARTIAL_FLOATS;
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(tmem_row + c * 32, r);
                tmem_ld_wait();
#pragma unroll
                for (int j = 0; j < 32; j += 4) {
                    float* dst = part_base + my_part + partial_offset<BN>(quad, c, j / 4, lane);
                    st_global_v4(dst, __uint_as_float(r[j]), __uint_as_float(r[j + 1]), __uint_as_float(r[j + 2]),
                                 __uint_as_float(r[j + 3]));
                }
            }
            __threadfence();  // this thread's partial is visible GPU-wide before the count
            named_bar_sync(1, 128);
            const int ts = w.tile - p.dp_tiles;
            const long long t_u0 = static_cast<long long>(ts) * p.num_k_blocks;
            const int s_lo = sk_slot_of_unit(p, t_u0);
            const int s_hi = sk_slot_of_unit(p, t_u0 + p.num_k_blocks - 1);
            int* const counter = p.counters + ts * CTAS + rank;
            if (epi_tid == 0) *bcast = atomicAdd(counter, 1);
            named_bar_sync(1, 128);
            const int arrived_before = *bcast;
            if (arrived_before != s_hi - s_lo) {  // another contributor finishes this tile
                release_accumulator();
                continue;
            }

            // Last contributor: sum every partial in K order (deterministic whoever is
            // last), its own straight from tensor memory, then scale and store.
            __threadfence();
#pragma unroll 1
            for (int c = 0; c < BN / EC; ++c) {
                float v[EC];
#pragma unroll
                for (int j = 0; j < EC; ++j) v[j] = 0.0f;
#pragma unroll 1
                for (int sl = s_lo; sl <= s_hi; ++sl) {
                    if (sl == slot) {
                        uint32_t r[EC];
#pragma unroll
                        for (int h = 0; h < EC / 32; ++h) {
                            tmem_ld_32x32b_x32(tmem_row + c * EC + 32 * h,
                                               *reinterpret_cast<uint32_t(*)[32]>(&r[32 * h]));
                        }
                        tmem_ld_wait();
#pragma unroll
                        for (int j = 0; j < EC; ++j) v[j] += __uint_as_float(r[j]);
                        continue;
                    }
                    const int piece = (sk_begin(p, sl) / p.num_k_blocks == ts) ? 0 : 1;
                    const size_t part = (static_cast<size_t>(sl * 2 + piece) * CTAS + rank) * S::PARTIAL_FLOATS;
                    float4 x[EC / 4];
#pragma unroll
                    for (int h = 0; h < EC / 32; ++h) {
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            x[8 * h + j] = __ldcg(reinterpret_cast<const float4*>(
                                part_base + part + partial_offset<BN>(quad, (EC / 32) * c + h, j, lane)));
                        }
                    }
#pragma unroll
                    for (int j = 0; j < EC / 4; ++j) {
                        v[4 * j + 0] += x[j].x;
                        v[4 * j + 1] += x[j].y;
                        v[4 * j + 2] += x[j].z;
                        v[4 * j + 3] += x[j].w;
                    }
                }
                store_chunk(v, row0, nb * BN + c * EC);
            }
            release_accumulator();
            if (epi_tid == 0) *counter = 0;  // leave the workspace ready for the next call
        }
        if (lane == 0) bulk_wait_group<0>();
        __syncwarp();
    }

    tc_fence_before();
    if constexpr (kPair || SPLIT > 1) {
        cluster_sync();  // no CTA leaves while a peer may still signal its barriers or write its memory
    } else {
        __syncthreads();
    }
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc<CTAS>(tmem_base, S::TMEM_COLS);
    }
}

}  // namespace hg
