/*
 * hipgemm_b200 — FP8 e4m3 TN GEMM for NVIDIA B200 (sm_100a), C ABI.
 *
 *   C[M x N] (bf16, row-major) = scale_a * scale_b * A[M x K] . B[N x K]^T
 *
 * A and B are OCP e4m3 bytes, row-major with K contiguous (B is the reference's
 * B_T), accumulation is fp32 in tensor memory, the result is rounded to bf16 with
 * round-to-nearest-even.  Plain pointers and sizes only: no CUDA or torch types in
 * the signatures (hgemm_stream_t is the same type as cudaStream_t / CUstream).
 *
 * Drop-in boundary.  The reference exposes one __global__ template that the caller
 * launches itself (nirw4nna/hipgemm fp8_4wave.hpp:334-338, launched at test.cpp:79
 * and bench.cpp:55,78 with <<<(M*N)/(256*256), 256>>>), unscaled, void-returning,
 * errors surfaced by hipGetLastError + exit (utils.hpp:7-11).  Here the launch is a
 * function call that returns a status code; the template wrapper at the end of this
 * header keeps the reference's name and template shape.
 *
 * Threading: every entry point is stream-ordered and asynchronous (except those
 * marked synchronous), reentrant, and safe to call from several host threads.  The
 * first call on a device does a one-time set-up under a mutex (SM count, kernel
 * shared-memory attributes); make that first call before any stream capture.
 */
#ifndef HIPGEMM_B200_H
#define HIPGEMM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* hgemm_stream_t;

/* Status codes.  Never calls exit(); the reference's CHECK_HIP_ERROR (utils.hpp:7-11)
 * terminates the process instead. */
#define HGEMM_OK 0
#define HGEMM_ERR_INVALID_VALUE (-1)   /* null pointer for a non-empty operand, negative size, bad range */
#define HGEMM_ERR_ALIGNMENT (-2)       /* K % 16, N % 8, or a pointer not 16-byte aligned (TMA rules) */
#define HGEMM_ERR_UNSUPPORTED (-3)     /* a valid request this entry point does not serve (a forced
                                          two-K-block config with K % 128 != 0, a problem beyond a
                                          fixed scratch or index range) */
#define HGEMM_ERR_CUDA (-4)            /* a CUDA runtime/driver call failed (launch, tensor map, ...) */
#define HGEMM_ERR_NO_DEVICE (-5)       /* no CUDA device, or not an sm_100 device */
#define HGEMM_ERR_DEVICE_TIMEOUT (-6)  /* a bounded wait inside a kernel expired (see hgemm_device_status) */

/* Replaces fp8_gemm_4wave_256x256x128<M,N,K> (fp8_4wave.hpp:334-338) for any shape:
 *   C = bf16_rne((scale_a * scale_b) * sum_k A[m][k] * B[n][k])
 * A: M x K e4m3 row-major.  B: N x K e4m3 row-major.  C: M x N bf16 row-major,
 * write-only (fully overwritten; never read).  d_scale_a / d_scale_b: device pointers
 * to one fp32 each, or NULL for 1.0 (the reference is unscaled).
 * Requirements: M, N, K >= 0; K % 16 == 0 and N % 8 == 0 (TMA row strides are
 * multiples of 16 bytes); A, B, C 16-byte aligned.  M == 0 or N == 0 is a no-op;
 * K == 0 writes zeros.  Returns HGEMM_OK or a negative HGEMM_ERR_* code. */
int hgemm_fp8_tn(const void* A, const void* B, void* C, int M, int N, int K, const float* d_scale_a,
                 const float* d_scale_b, hgemm_stream_t stream);

/* Rows [row_begin, row_end) of the same product, written to rows [row_begin, row_end)
 * of C: the per-rank call of the M-sharded multi-GPU path (each rank holds all of B).
 * A and C are the FULL matrices' base pointers.  No counterpart in the reference,
 * which is single-GPU (its grid always covers all of M, test.cpp:79). */
int hgemm_fp8_tn_rows(const void* A, const void* B, void* C, int M, int N, int K, int row_begin, int row_end,
                      const float* d_scale_a, const float* d_scale_b, hgemm_stream_t stream);

/* The whole product from host buffers, as the reference's test.cpp:73-81 does it (copy A
 * and B in, launch, copy C out), pipelined: A and B go to the device in up to 4 row
 * panels each, alternately, on one internal stream; each arriving panel makes one rectangle
 * of C computable (the new panel against every panel of the other operand already in),
 * which is computed on a second stream and copied back to C_host on a third, so both copy
 * directions and the GEMMs overlap.  The internal streams and events are created on a
 * thread's first call on a device and kept for its later calls.  Host buffers should be
 * pinned (cudaMallocHost) for the copies to be asynchronous.  d_A (M x K), d_B (N x K), d_C (M x N bf16) and d_scales (2 floats) are
 * caller-owned device buffers; h_scales (2 host floats: scale_a, scale_b) or NULL for 1.0.
 * Stream-ordered with respect to `stream` at both ends; host buffers must stay valid
 * until that stream reaches this point.  No counterpart in the reference. */
int hgemm_fp8_tn_from_host(const void* A_host, const void* B_host, void* C_host, int M, int N, int K,
                           const float* h_scales, void* d_A, void* d_B, void* d_C, float* d_scales,
                           hgemm_stream_t stream);

/* The M-sharded call fused with the all-gather of C.  C_ranks[i] is rank i's full M x N
 * C buffer as mapped into this process (C_ranks[rank] is this GPU's own; the others are
 * peer memory opened with hgemm_ipc_import, 1 <= nranks <= 8).  Rows [row_begin, row_end)
 * are computed here and every finished C tile is TMA-stored into all nranks buffers, so
 * the exchange over NVLink overlaps the math tile by tile (the automatic choice takes a tile
 * whose stores write 128-byte row segments, the efficient size across NVLink).  When every rank's call has
 * completed (order a barrier after it on the stream, e.g. a one-element NCCL all-reduce),
 * every buffer holds the whole C.  A caller that reuses the buffers must also put a
 * barrier between its last read of C and the next call.  No counterpart in the
 * reference, which is single-GPU (its C is written by one kernel, test.cpp:79). */
int hgemm_fp8_tn_rows_allgather(const void* A, const void* B, void* const* C_ranks, int nranks, int rank, int M,
                                int N, int K, int row_begin, int row_end, const float* d_scale_a,
                                const float* d_scale_b, hgemm_stream_t stream);

/* CUDA IPC helpers for the buffers above (synchronous).  hgemm_ipc_export writes the 64-byte
 * handle of the allocation that contains `ptr` and ptr's offset inside it;
 * hgemm_ipc_import opens a handle from another process (returns the allocation's base:
 * add the offset), hgemm_ipc_close releases it. */
int hgemm_ipc_export(const void* ptr, void* handle_out, size_t* offset_out);
int hgemm_ipc_import(const void* handle, void** base_out);
int hgemm_ipc_close(void* base);

/* Same as hgemm_fp8_tn with the tile configuration forced (benchmarks and tests):
 * config 0 = automatic choice; see hgemm_config_name() for the others. */
int hgemm_fp8_tn_config(const void* A, const void* B, void* C, int M, int N, int K, const float* d_scale_a,
                        const float* d_scale_b, hgemm_stream_t stream, int config);

/* Schedules for hgemm_fp8_tn_ex. */
#define HGEMM_SCHEDULE_AUTO 0           /* the library's choice: data-parallel, or (automatic
                                           configuration only) split-K over CTA clusters for
                                           skinny problems with long K, whose bits differ from
                                           the whole-K kernels' */
#define HGEMM_SCHEDULE_DATA_PARALLEL 1  /* whole output tiles and whole K only, bits independent of
                                           the tiling; needs no workspace */
#define HGEMM_SCHEDULE_STREAM_K 2       /* split the last one-to-two waves of tiles along K across all
                                           SMs; partial tiles are reduced deterministically */

/* Full-control form: tile configuration (0 = automatic), schedule, and an optional
 * caller-owned device workspace (256-byte aligned, at least hgemm_workspace_bytes(); its
 * content on entry does not matter).  With workspace == NULL a stream-K schedule takes
 * its workspace from a library-owned stream-ordered pool (cudaMallocFromPoolAsync /
 * cudaFreeAsync on `stream`), which the first such call on a device creates
 * (cudaMemPoolCreate); make that first call before any stream capture.  Calls that share
 * a caller workspace must not overlap on the GPU.  No counterpart in the reference, whose
 * launch shape is fixed. */
int hgemm_fp8_tn_ex(const void* A, const void* B, void* C, int M, int N, int K, const float* d_scale_a,
                    const float* d_scale_b, hgemm_stream_t stream, int config, int schedule, void* workspace,
                    size_t workspace_bytes);

/* Synchronous (device set-up).  Workspace bytes hgemm_fp8_tn_ex needs for this problem
 * on the current device (0 when the schedule is data-parallel). */
int hgemm_workspace_bytes(int M, int N, int K, int config, int schedule, size_t* bytes_out);

/* Synchronous (device set-up).  The launch plan for this problem on the current device:
 * plan_out[0..5] = {config, grid CTAs, output tiles, data-parallel tiles, stream-K tiles,
 * stream-K slots}. */
int hgemm_plan(int M, int N, int K, int config, int schedule, int* plan_out);

/* Allocation-free variant of the stream-K schedule, for callers that may not allocate
 * device memory at all (an engine that already gave all GPU memory to its own allocator,
 * a plugin host that forbids driver allocations, a hot path that cannot take
 * cudaMalloc's device-wide synchronisation).  No counterpart in the reference, which
 * needs no scratch.  Same arguments and result contract as hgemm_fp8_tn; it runs the
 * HGEMM_SCHEDULE_STREAM_K schedule with its scratch in a fixed 8 MiB device array inside
 * this library (held by every GPU that loads the library until the process exits) and
 * calls no cudaMalloc, cudaFree, memory-pool or other allocating routine, on its first
 * call too: the library's workspace pool is never created on this path.
 * Limit: a problem whose stream-K scratch exceeds 8 MiB (see hgemm_workspace_bytes with
 * HGEMM_SCHEDULE_STREAM_K) is refused with HGEMM_ERR_UNSUPPORTED before anything is
 * launched; the data-parallel schedule (hgemm_fp8_tn_ex, HGEMM_SCHEDULE_DATA_PARALLEL)
 * needs no scratch for any size.
 * The first call on a device runs the library's one-time device set-up (device properties,
 * kernel attributes, occupancy queries) and looks up the array's device address; make that
 * first call before any stream capture.  A failed lookup is retried by the next call.
 * Every call shares the one array and finds the last call's contents in it (this entry
 * point clears what must start at zero), so calls that overlap on the GPU, from any stream
 * or thread, race: serialise them. */
int hgemm_fp8_tn_static_scratch(const void* A, const void* B, void* C, int M, int N, int K, const float* d_scale_a,
                                const float* d_scale_b, hgemm_stream_t stream);

/* Host-only views of the schedule arithmetic the kernels run (for tests):
 * hgemm_debug_schedule splits `tiles` tiles of `kblocks` K blocks over `slots` slots and
 * writes {data-parallel tiles, stream-K tiles, stream-K slots};
 * hgemm_debug_work_items lists slot `slot`'s work items, 6 ints each: {tile, first K
 * block, end K block, piece (-1 whole tile, 0/1 partial), first and last contributing
 * slot of a partial tile}; returns the count (or a negative status). */
int hgemm_debug_schedule(long long tiles, int slots, int kblocks, int schedule, int* out3);
int hgemm_debug_work_items(int kblocks, int nslots, int dp_tiles, int sk_tiles, int sk_slots, int slot, int* out,
                           int max_items);
/* The split-K configurations' work: CTA `cta` of a grid of clusters of `split` CTAs over
 * `tiles` tiles writes {tile, first K block, end K block}; returns the number of items the
 * CTA gets (1; 0 past the last tile) or a negative status. */
int hgemm_debug_split_work(int kblocks, int split, int tiles, int cta, int* out3);
/* The automatic configuration choice, on the host, for a device that keeps resident_ctas[c]
 * CTAs of configuration c resident at once (n_configs = hgemm_num_configs(); entry 0 unused):
 * what hgemm_fp8_tn with `schedule` would run.  Returns the configuration index or a
 * negative status. */
int hgemm_debug_choose(int M, int N, int K, int schedule, const int* resident_ctas, int n_configs);

/* Number of tile configurations and their names ("bn256_s4" ...); NULL past the end. */
int hgemm_num_configs(void);
const char* hgemm_config_name(int config);
/* Synchronous (device set-up).  CTAs of configuration `config` (>= 1) that the current
 * device keeps resident at once, i.e. the persistent grid size; negative on error. */
int hgemm_config_resident_ctas(int config);

/* Synchronous.  Reads and clears the current device's kernel status word: 0 when no
 * bounded wait has expired since the last call, else the code of the first one,
 * role << 8 | site: 0x0101 producer (stage free), 0x0201 / 0x0202 / 0x0203 MMA issuer
 * (accumulator free, stage full, drain), 0x0301 epilogue (accumulator full), 0x0303
 * split-K epilogue (peers' partial columns in). */
int hgemm_device_status(uint32_t* status_out);

/* Test hook: 1 if the library's stream-K workspace pool exists on `device` (it is created
 * by the first hgemm_fp8_tn_ex call there that needs library-allocated scratch), 0 if not,
 * HGEMM_ERR_INVALID_VALUE for a bad index.  Makes no CUDA call. */
int hgemm_debug_workspace_pool_created(int device);

/* Human-readable text for an HGEMM_* status code (static storage). */
const char* hgemm_error_string(int code);

/* Test hook for the failure path: runs the GEMM with its first stage's copies withheld (the
 * stage's barrier expects bytes that never arrive), so every bounded wait in the kernel
 * expires after its limit (about 2 s).  The kernel records a status (read it, and clear it, with
 * hgemm_device_status), drains and returns; the context stays usable and C is unspecified.
 * Not for production use. */
int hgemm_debug_stalled_gemm(const void* A, const void* B, void* C, int M, int N, int K, int config,
                             hgemm_stream_t stream);

/* Library version string. */
const char* hgemm_version(void);

/* ---- MX block scaling ------------------------------------------------------------------- */

/* OCP MX e4m3 GEMM (tcgen05 kind::mxf8f6f4.block_scale): every 32 consecutive K elements of
 * a row of A and of B carry their own e8m0 scale (2^(e - 127)), so
 *   C = bf16_rne((scale_a*scale_b) * sum_k A[m][k] 2^(SFA[m][k/32]-127) B[n][k] 2^(SFB[n][k/32]-127)).
 * SFA / SFB are in the blocked layout that tcgen05 consumes (hgemm_host_mx_sf_to_blocked
 * converts from row-major rows x K/32): 512-byte atoms of 128 rows x 4 K-groups, row r,
 * group g at byte 16*(r%32) + 4*(r/32) + g; atom (r/128, g/4) at ((r/128)*ceil(K/128) +
 * g/4) * 512; hgemm_mx_sf_bytes() bytes each, 16-byte aligned.  Padding entries must hold
 * a finite scale (not 0xFF).  K % 32 == 0 and N % 8 == 0.  The reference's MFMA builtin
 * is the block-scaled instruction with its scales fixed at zero (fp8_4wave.hpp:53-58);
 * this is that instruction with scales in use. */
int hgemm_fp8_tn_mx(const void* A, const void* B, void* C, int M, int N, int K, const void* SFA, const void* SFB,
                    const float* d_scale_a, const float* d_scale_b, hgemm_stream_t stream);
/* hgemm_fp8_tn_mx with its kernel chosen: 0 = by wave count (what hgemm_fp8_tn_mx does),
 * 1 = 128 x 256 tiles, one accumulator; 2 = 128 x 128 tiles; 3 = 256 x 256 tiles on CTA
 * pairs, one accumulator; 4 and 5 = configs 3 and 2 with two K blocks per TMA load (faster;
 * K % 128 == 0 only, else HGEMM_ERR_UNSUPPORTED, and config 0 picks them only then).
 * Names: hgemm_mx_config_name. */
int hgemm_fp8_tn_mx_config(const void* A, const void* B, void* C, int M, int N, int K, const void* SFA,
                           const void* SFB, const float* d_scale_a, const float* d_scale_b, int config,
                           hgemm_stream_t stream);
int hgemm_mx_num_configs(void);
const char* hgemm_mx_config_name(int config);
/* Bytes of a blocked scale-factor tensor for `rows` rows and K columns. */
size_t hgemm_mx_sf_bytes(int rows, int K);
/* Row-major (rows x K/32) e8m0 bytes -> the blocked layout above (host memory). */
int hgemm_host_mx_sf_to_blocked(const uint8_t* sf, int rows, int K, uint8_t* blocked);

/* ---- device quantiser ------------------------------------------------------------------- */

#define HGEMM_DTYPE_F32 0
#define HGEMM_DTYPE_BF16 1

/* Per-tensor e4m3 quantisation on the device, stream-ordered: *d_scale = amax(|x|) / 448
 * (1.0 for an all-zero tensor; NaN elements are ignored) and q[i] = e4m3(x[i] / scale),
 * IEEE division, round-to-nearest-even, saturating to +-448.  x: n fp32 or bf16 values
 * (x_dtype), q: n bytes, both 16-byte aligned; d_scale: one float of device memory (used
 * as the amax accumulator until the last step writes the scale).  The result feeds
 * hgemm_fp8_tn directly (q as A or B, d_scale as its scale).  The reference quantises on
 * the host without a scale (utils.hpp:27-33); this is the benchmark configs' amax/448
 * quantiser moved onto the GPU. */
int hgemm_quantize_e4m3(const void* x, int x_dtype, size_t n, void* q, float* d_scale, hgemm_stream_t stream);

/* Delayed scaling, one HBM pass: q = e4m3(x / *d_scale_in) (IEEE division, satfinite RNE; the
 * scale is used as given, typically amax/448 of the previous step), and *d_amax_out =
 * amax(|x|) of this tensor (NaNs ignored) for the next step's scale.  With *d_scale_in equal
 * to this tensor's own amax/448 the bytes equal hgemm_quantize_e4m3's.  x and q 16-byte
 * aligned, the two floats 4-byte aligned, all on the device.  Stream-ordered, no sync. */
int hgemm_quantize_e4m3_delayed(const void* x, int x_dtype, size_t n, void* q, const float* d_scale_in,
                                float* d_amax_out, hgemm_stream_t stream);

/* OCP MX e4m3 quantiser on the device: x (rows x K, fp32 or bf16 by x_dtype, row-major) ->
 * q (rows x K e4m3 bytes) and one e8m0 scale per 32 elements of a row, written in the
 * blocked layout hgemm_fp8_tn_mx reads (hgemm_mx_sf_bytes(rows, K) bytes; padding = 127).
 * X = floor(log2(amax)) - 8 clamped to [-127, 127] (-127 for a block whose amax is 0,
 * subnormal or infinite; NaNs do not count), scale byte X + 127, q = e4m3_satfinite(x * 2^-X).
 * K % 32 == 0 (HGEMM_ERR_ALIGNMENT); x and q 16-byte aligned; fewer than 2^32 blocks of 32
 * (HGEMM_ERR_UNSUPPORTED otherwise: 275 GB of bf16).  Stream-ordered, no sync. */
int hgemm_quantize_mx_e4m3(const void* x, int x_dtype, int rows, int K, void* q, void* sf_blocked,
                           hgemm_stream_t stream);

/* ---- host utilities mirroring the reference harness (utils.hpp) ---------------------- */

/* utils.hpp:27-33 init_random, generalised: std::mt19937(seed) feeding
 * std::normal_distribution<float>(mean, stddev), each draw converted to e4m3 with
 * CUDA's host conversion (OCP e4m3, round-to-nearest-even, saturate to finite).
 * The reference uses mean -1, stddev 1, seed 0. */
void hgemm_host_init_random(uint8_t* out, size_t n, uint64_t seed, float mean, float stddev);

/* The benchmark configs' per-tensor quantiser: draws n values from N(mean, stddev)
 * with std::mt19937(seed), scale = amax / 448 (fp32), q[i] = e4m3(x[i] / scale).
 * Returns the scale (1.0 for an all-zero tensor). */
float hgemm_host_make_quantized(uint8_t* q, size_t n, uint64_t seed, float mean, float stddev);

/* Quantise caller-provided fp32 values the same way; returns the scale. */
float hgemm_host_quantize_e4m3(const float* x, size_t n, uint8_t* q);

/* One value through CUDA's host e4m3 / bf16 conversions (for checks). */
uint8_t hgemm_host_fp8_encode(float x);
uint16_t hgemm_host_bf16_rne(float x);
/* n values through CUDA's host e4m3 conversion (satfinite, RNE). */
void hgemm_host_fp8_encode_array(const float* x, size_t n, uint8_t* out);

#ifdef __cplusplus
} /* extern "C" */

/* Header-only drop-in for the reference's launcher surface (fp8_4wave.hpp:334-338).
 * At a call site, `fp8_gemm_4wave_256x256x128<M, N, K><<<grid, 256>>>(A, B_T, C);`
 * becomes `fp8_gemm_4wave_256x256x128<M, N, K>(A, B_T, C);` (grid and block are
 * chosen inside), with optional per-tensor scales and a stream.  Unlike the reference
 * template it accepts any M, N (N % 8 == 0) and K (K % 16 == 0), and returns a
 * status code instead of requiring hipGetLastError. */
template <int M, int N, int K>
inline int fp8_gemm_4wave_256x256x128(const void* A, const void* B_T, void* C, const float* d_scale_a = nullptr,
                                      const float* d_scale_b = nullptr, hgemm_stream_t stream = nullptr) {
    static_assert(M >= 0 && N >= 0 && K >= 0, "sizes must be non-negative");
    static_assert(K % 16 == 0, "K must be a multiple of 16 (TMA row stride)");
    static_assert(N % 8 == 0, "N must be a multiple of 8 (TMA row stride of C)");
    return hgemm_fp8_tn(A, B_T, C, M, N, K, d_scale_a, d_scale_b, stream);
}
#endif /* __cplusplus */

#endif /* HIPGEMM_B200_H */
