/*
 * phantom_attn.h - C ABI of the B200 (sm_100a) fused attention forward.
 *
 *   O = softmax(Q K^T / sqrt(d)) V      per (batch, head), online (running max / sum) softmax
 *
 * This is the drop-in boundary for the attention kernels of b4batunde/Phantom-A100. Every entry
 * point below replaces one launcher of that project's `csrc/kernels/` layer (which returned a
 * cudaError_t and took typed device pointers) with a plain C function: untyped device pointers,
 * sizes, a dtype code and a CUDA stream. No torch types cross this boundary.
 *
 * Layout (all entry points): q, k, v, o are contiguous row-major (BH, N, d) device arrays, element
 * ((bh * N) + i) * d + c, as in the reference (csrc/kernels/fused_tc.cuh:60,92). The library
 * never writes q, k, v. o is written in full (rows < N) by the launch. Launches are asynchronous
 * on `stream` (a cudaStream_t, NULL = legacy default stream) and run on the current device.
 *
 * Errors: every call returns PHANTOM_ATTN_OK or an error code; phantom_attn_last_error() returns a
 * human-readable message for the last failing call on the calling thread. The message texts keep
 * the substrings the reference tests match ("head dimension", "float16", "not compiled",
 * "16-byte aligned", "shared memory"; reference csrc/common.cuh:27-33, attn_fused_tuned.cu:9-14).
 *
 * Device-side waits in the tensor-core kernel are bounded. A wait that expires (which only a
 * hardware or programming fault can cause) makes the kernel stop early and record a non-zero
 * status word on the device; phantom_attn_device_status() reads and clears it.
 */
#ifndef PHANTOM_ATTN_H_
#define PHANTOM_ATTN_H_

#ifdef __cplusplus
extern "C" {
#endif

/* dtype codes */
#define PHANTOM_ATTN_F32 0
#define PHANTOM_ATTN_F16 1
#define PHANTOM_ATTN_BF16 2

/* status codes */
#define PHANTOM_ATTN_OK 0
#define PHANTOM_ATTN_ERR_INVALID 1     /* bad pointer, shape, alignment or dtype             */
#define PHANTOM_ATTN_ERR_UNSUPPORTED 2 /* configuration not compiled (head dim, tile, dtype)  */
#define PHANTOM_ATTN_ERR_CUDA 3        /* a CUDA runtime or driver call failed                */
#define PHANTOM_ATTN_ERR_DEVICE 4      /* a device-side bounded wait expired (status word)    */

/* Library version, e.g. 10000 for 1.0.0. */
int phantom_attn_version(void);

/* Message for the last failing call on this thread ("" if none). Valid until the next call. */
const char* phantom_attn_last_error(void);

/*
 * v4 replacement: fused attention on 5th-generation tensor cores (tcgen05.mma, TMEM accumulators,
 * TMA-staged K/V ring). dtype PHANTOM_ATTN_F16 or PHANTOM_ATTN_BF16, head_dim 64 or 128, any
 * seq_len >= 1, causal 0/1. fp32 accumulation; P is rounded to fp16 for the P.V product (for bf16
 * inputs V is staged as fp16 first; a head whose V holds a finite value beyond the fp16 range uses
 * bf16 P and bf16 V instead).
 * Replaces attn::launch_fused_tc (reference csrc/kernels/fused_tc.cuh:187-196), which took
 * (const __half* q, k, v, __half* o, int BH, int N, bool causal, cudaStream_t) with d fixed at 64
 * and fp16 only; head_dim and dtype are explicit here because both are now selectable.
 */
int phantom_attn_fused_tc(const void* q, const void* k, const void* v, void* o, int BH, int N,
                          int head_dim, int dtype, int causal, void* stream);

/*
 * phantom_attn_fused_tc without any device-memory allocation, for callers that cannot allocate while
 * they run: plugin hosts that own every byte of device memory and hand a plugin only its inputs and
 * outputs, real-time loops that forbid allocator calls after start-up, and budgets where a hidden
 * allocation could fail at the worst moment. No counterpart in the reference (its fused_tc needed no
 * scratch; this library's bf16 path stages V as fp16 in scratch).
 *
 * Same arguments, checks, kernel and results as phantom_attn_fused_tc. Instead of allocating, it uses
 * a file-scope 64 MiB device array that every GPU loading the library holds until the process exits:
 * a 256-byte status region (the status word; the work counters of the kernel's persistent CTAs and a
 * word marking fp16-overflowing heads, all reset by every call), then, for bf16 inputs, the fp16 copy of
 * V (2 * BH * N * head_dim bytes) and
 * its overflow flags (128 bytes per head from BH = 20 on, up to 2 KiB per head below that, where V is
 * staged in more chunks per head). bf16 inputs needing more than 64 MiB in all (BH * N * head_dim
 * above about 33.5 million) are rejected with PHANTOM_ATTN_ERR_UNSUPPORTED; fp16 inputs need no
 * scratch and have no such limit. The first call on a device sets that device up (it resolves the
 * array's device address and zeroes the status word, synchronously), so make it before any stream
 * capture. Every call on a device shares the array: calls that overlap on the GPU (different streams,
 * or another thread) race on it and must be serialised by the caller. Bounded-wait expiries of this
 * path are recorded in a status word inside the array; phantom_attn_device_status() reads and clears
 * it (without allocating) and reports its bits together with PHANTOM_ATTN_STATUS_NOALLOC.
 */
int phantom_attn_fused_tc_noalloc(const void* q, const void* k, const void* v, void* o, int BH, int N,
                                  int head_dim, int dtype, int causal, void* stream);

/*
 * v3.1/v3.2 replacement. (br, bc) must be one of the reference's compiled tiles (64,32) (64,64)
 * (128,32) (128,64), else PHANTOM_ATTN_ERR_UNSUPPORTED with "not compiled". On sm_100a the work
 * runs on the tensor-core kernel above (its tile is fixed by the tcgen05 instruction shape); the
 * tile and double_buffer arguments are validated for interface compatibility only.
 * Replaces attn::launch_fused_tuned (reference csrc/kernels/fused_tuned.cuh:212-228).
 */
int phantom_attn_fused_tuned(const void* q, const void* k, const void* v, void* o, int BH, int N,
                             int head_dim, int dtype, int causal, int double_buffer, int br, int bc,
                             void* stream);

/*
 * v3 replacement: fused online-softmax attention on CUDA cores with fp32 arithmetic, for fp32,
 * fp16 and bf16 inputs and any head_dim in [1, 256]. Exact fp32 path (no tensor cores): meets the
 * reference's 1e-4 fp32 tolerance. Replaces attn::launch_fused (reference
 * csrc/kernels/fused.cuh:107-112), which compiled d == 64 only.
 */
int phantom_attn_fused(const void* q, const void* k, const void* v, void* o, int BH, int N,
                       int head_dim, int dtype, int causal, void* stream);

/*
 * v1 / v2 replacements (reference csrc/kernels/naive.cuh:56-64, tiled.cuh:109-117). The reference
 * materialised the BH x N x N fp32 score matrix in a caller-provided workspace; on sm_100a the same
 * result comes from the fused CUDA-core kernel, so no workspace argument exists.
 */
int phantom_attn_naive(const void* q, const void* k, const void* v, void* o, int BH, int N,
                       int head_dim, int dtype, int causal, void* stream);
int phantom_attn_tiled(const void* q, const void* k, const void* v, void* o, int BH, int N,
                       int head_dim, int dtype, int causal, void* stream);

/*
 * Reads and clears the device status words of the current device (synchronises the device).
 * *status = 0 when every kernel since the last call finished normally; otherwise a bit set of
 * where a bounded wait expired: bits 0-3 (copy, MMA, softmax and epilogue waits of the tensor-core
 * kernel), PHANTOM_ATTN_STATUS_PROBE (the test probe below), and PHANTOM_ATTN_STATUS_NOALLOC when
 * the bits came from phantom_attn_fused_tc_noalloc's own word. Allocates nothing. No counterpart in
 * the reference (its kernels had no waits).
 */
#define PHANTOM_ATTN_STATUS_NOALLOC 256
int phantom_attn_device_status(int* status);

/*
 * Test support for the failure path: launches (asynchronously, on `stream`) a one-warp kernel that
 * waits, with the same bounded mbarrier wait the attention kernels use, on a barrier that nothing
 * arrives on. The wait gives up after its limit (about a second), and the kernel sets bit 16
 * (PHANTOM_ATTN_STATUS_PROBE) of the device status word, and of phantom_attn_fused_tc_noalloc's word
 * once that entry point has been called on the device, and exits; the context stays usable, and
 * phantom_attn_device_status then reports and clears the bits. No counterpart in the reference.
 */
#define PHANTOM_ATTN_STATUS_PROBE 16
int phantom_attn_wait_expiry_probe(void* stream);

/*
 * Device memory the library takes besides the caller's tensors, for peak-memory reporting (the reference
 * benchmark recorded peak_memory_mb, bench/benchmark.py:96-102; its kernels allocated through torch).
 * The tensor-core entry points take per-call scratch (work counters and, for bf16 inputs, the overflow word,
 * the fp16 copy of V and its overflow flags; K/V-part partials) from a stream-ordered pool per device. *high_water = the most scratch in use at once
 * on the current device since the last reset, *reserved = bytes the pool holds now (it keeps freed
 * blocks for reuse); both 0 before any call needed scratch. reset = 1 restarts the high-water mark.
 * phantom_attn_fused_tc_noalloc uses its static array instead and is not counted.
 */
int phantom_attn_scratch_bytes(long long* high_water, long long* reserved, int reset);

/*
 * Number of kernel launches made by this library on the calling thread since the last reset
 * (reset = 1 clears it). Used by the benchmark to count the launches in a timed region.
 */
long long phantom_attn_launch_count(int reset);

/*
 * Benchmark support (no counterpart in the reference). While enabled on the calling thread, every
 * launch of the tensor-core attention kernel is bracketed by a CUDA event pair recorded on its stream
 * (the bf16 V staging pass is outside the pair). enable = 1 also discards earlier records.
 * phantom_attn_kernel_timing_read() waits for the recorded events and returns the summed kernel time
 * in milliseconds and the number of bracketed launches.
 */
int phantom_attn_kernel_timing(int enable);
int phantom_attn_kernel_timing_read(double* total_ms, long long* launches);

/*
 * Launch-shape override of the tensor-core kernel (fused_tc, fused_tuned, fused_tc_noalloc) for the
 * calling thread; the tile sweep's knobs. No counterpart in the reference: its tuning knobs were the
 * compiled (br, bc) tiles and double buffering (reference bench/sweep_tiles.py:22-63), which on sm_100a
 * are fixed by the tcgen05 instruction shape. 0 selects the automatic value.
 *   l2_group_kib  K and V bytes (4 * N * head_dim per head) of one scheduling group of heads, in KiB;
 *                 the persistent CTAs take all query blocks of a group before the next group, so a group
 *                 within L2 streams its K/V from DRAM once. Automatic: 16384 (16 MiB). At least one head.
 *   max_ctas      cap on the persistent grid (automatic: one CTA per SM), e.g. to leave SMs to work on
 *                 another stream.
 * Results do not depend on either value. Returns PHANTOM_ATTN_ERR_INVALID for a negative value or
 * l2_group_kib above 2^40.
 */
int phantom_attn_set_launch_shape(long long l2_group_kib, int max_ctas);
int phantom_attn_get_launch_shape(long long* l2_group_kib, int* max_ctas);

/*
 * Tail balancing of the tensor-core kernel (fused_tc, fused_tuned) for the calling thread. No
 * counterpart in the reference. The persistent CTAs run the query blocks in waves; when the last wave
 * would leave more than half of the CTAs idle at its end and is too large for one-tile units, its blocks
 * (non-causal only) are cut into 2-8 parts of their K/V range: each part leaves an unnormalised partial
 * result in the launch's scratch, and the last part of each row to finish merges them (results within the
 * usual tolerance of the whole-range computation, not bit-identical to it). allow = 1 (default) lets the
 * library choose this; allow = 0 keeps every block whole, so the results of a call are bit-identical for
 * every launch shape and GPU count. phantom_attn_fused_tc_noalloc never cuts K/V ranges.
 * Returns PHANTOM_ATTN_ERR_INVALID for a value other than 0 or 1; the getter returns the current value.
 */
int phantom_attn_set_kv_parts(int allow);
int phantom_attn_get_kv_parts(void);

#ifdef __cplusplus
}
#endif

#endif /* PHANTOM_ATTN_H_ */
