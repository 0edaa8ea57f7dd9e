// Fused attention forward on B200 5th-generation tensor cores (sm_100a).
//
//   O = softmax(Q K^T / sqrt(d)) V,   online softmax in the log2 domain
//
// Algorithm (same arithmetic contract as the reference's v4 kernel, csrc/kernels/fused_tc.cuh:45-179,
// and its NumPy model cuda_attn/online_softmax_ref.py:27-63 with p_fp16=True): scores in fp32, a
// running row max m and row sum l in fp32, P = exp2(S*log2e/sqrt(d) - m) rounded to fp16 for the P.V
// product while l sums the unrounded fp32 values, O accumulated in fp32 and divided by l at the end.
// bf16 inputs: Q K^T runs in bf16; V is first staged as fp16 by stage_v_f16 (exact for every bf16
// value inside the fp16 range) so that P.V also runs with fp16 P - rounding P to bf16 instead would
// alone give a relative-L2 error of ~2.4e-3, above the 1e-3 parity bound. A head whose V holds a
// finite value beyond the fp16 range falls back to bf16 P and the original bf16 V for that head; the
// call's main launch skips such heads and a second launch (OVF_HEADS) computes them.
//
// B200 mapping (not a translation of the WMMA kernel):
//   * Work unit: two 128-row Q tiles (A, B) of one (batch, head), streaming K/V tiles of 128 keys.
//     Persistent CTAs (one per SM) take units one after another from an atomic counter, heaviest
//     first (causal) within groups of heads whose K/V fit in L2; the K/V ring, the S sequence and all
//     barrier phases run on across units, so the next unit's Q load and first S overlap the current
//     unit's last tiles and output.
//   * Warp 9 (one thread) is the TMA producer: Q tiles once, then K_0, V_0, K_1, V_1, ... into a ring
//     of STAGES shared-memory slots (128-byte swizzle), completion tracked by mbarrier tx bytes.
//   * Warp 8 (one thread) issues the S_g = Q_g K_j^T products (both operands in shared memory, fp32
//     accumulator in TMEM, 128 lanes x 128 columns); warp 10 (one thread) issues O_g += P_g V_j
//     (P read from TMEM, V from shared memory as an MN-major operand, accumulator in TMEM). Commits
//     go to mbarriers. Two issuers because an issuing thread blocks while the tensor core's
//     instruction queue is full: with one, an S product waiting behind a P.V product (or the
//     reverse) stalled the other chain.
//   * Warps 0-3 / 4-7 are the softmax warpgroups of tiles A / B: thread t owns query row t = TMEM
//     lane t, so the row max and row sum need no shuffles. Each thread loads its S row from TMEM and
//     releases the S columns at once, masks, takes the max, rescales its O row in TMEM only when the
//     max grew by more than 2^8 (exact: every P and l of a row use the same reference max), computes
//     P with ex2 and writes it into its tile's P columns as packed 16-bit pairs (the A operand of
//     the P.V product), then arrives.
//   * P never shares columns with S, so the next S product runs while the softmax of the current K/V
//     tile still computes; each softmax warpgroup then goes from tile to tile without waiting for
//     its own P.V product (only for the previous one, before it overwrites P and rescales O).
//   * TMEM (512 columns): d = 128: S [0,128) used by tiles A and B in turn, P_A [128,192),
//     P_B [192,256), O_A [256,384), O_B [384,512); d = 64: O_A, O_B, then S_A, S_B, P_A, P_B.
//   * O leaves through shared memory: each softmax warp writes its 32 rows into a swizzled staging block
//     and one lane issues a TMA store.
//   * Every mbarrier wait is bounded; on expiry the CTA drains its in-flight copies and MMAs,
//     frees TMEM, records the failure in the device status word and exits.
#include <cuda.h>
#include <math_constants.h>

#include <algorithm>
#include <atomic>
#include <mutex>

#include "launchers.h"
#include "sm100_ptx.cuh"
#include "../../include/phantom_attn.h"

namespace phantom {
namespace tc {

constexpr int BM = 128;  // query rows per Q tile = TMEM lanes
constexpr int MMA_WARP = 8;          // issues the Q.K^T products
constexpr int TMA_WARP = 9;
constexpr int PV_WARP = 10;          // issues the P.V products; warp 11 completes the producer warpgroup
constexpr int NUM_THREADS = 384;
// Register split (setmaxnreg): the kernel launches at 168 registers/thread (384 threads, 1 CTA/SM).
// The producer warpgroup drops to 72 and the two softmax warpgroups rise to 216:
// 128*(168-72) = 2*128*(216-168), so the increase is exactly covered by the release.
constexpr int kRegsProducer = 72;
constexpr int kRegsSoftmax = 216;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale O only when the max grows by > 2^8

// Status-word bits (which wait expired).
constexpr int kErrTmaWait = 1, kErrMmaWait = 2, kErrSoftmaxWait = 4, kErrEpilogueWait = 8;
constexpr int kUnitRing = 4;  // published work units (shared memory, 32 bytes each)

// TMEM plan per head dimension (K/V tiles of BN = 128 keys). P (the probabilities as packed 16-bit
// pairs, the A operand of O += P V) never shares columns with S (fp32 scores), so a Q.K^T product is
// issued as soon as the softmax has read the previous S into registers, while O += P V of the
// previous tile still reads P:
//   d = 128: one S region that Q tiles A and B use in turn (A, B, A, B, ...):
//            S [0,128)  P_A [128,192)  P_B [192,256)  O_A [256,384)  O_B [384,512)
//   d =  64: an S region per Q tile:
//            O_A [0,64)  O_B [64,128)  S_A [128,256)  S_B [256,384)  P_A [384,448)  P_B [448,512)
template <int D>
struct Cfg {
  static constexpr bool SHARED_S = D == 128;
  static constexpr int BN = 128;                     // keys per K/V tile
  static constexpr int KBLK = D / 64;                // 64-element (128-byte) swizzle blocks across d
  static constexpr int Q_SUB = BM * 128;             // one 64-column block of a Q tile
  static constexpr int KV_SUB = BN * 128;            // one 64-column block of a K or V tile
  static constexpr int Q_TILE = BM * D * 2;
  static constexpr int KV_TILE = BN * D * 2;
  static constexpr int STAGES = D == 128 ? 4 : 8;    // K/V ring slots
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_KV = 2 * Q_TILE;
  static constexpr int OFF_BAR = OFF_KV + STAGES * KV_TILE;
  // barriers: q_full[0], kv_full[STAGES], kv_empty[STAGES], s_full[2], s_free[2], p_ready[2], o_done[2],
  // drain (S issuer), drain (P.V issuer), q_free, o_free[2], q_full[1]
  static constexpr int NUM_BARS = 1 + 2 * STAGES + 14;
  static constexpr int OFF_MISC = (OFF_BAR + NUM_BARS * 8 + 15) / 16 * 16;  // TMEM base address, abort flag, unit ring
  // O staging for the TMA-store epilogue: per softmax warp one 32-row x 64-column 16-bit block (4 KB) in the
  // 128-byte swizzled layout of the output tensor map (1024-byte aligned)
  static constexpr int OST_WARP = 32 * 128;
  static constexpr int OFF_OST = (OFF_MISC + 16 + 32 * kUnitRing + 1023) / 1024 * 1024;
  static constexpr int SMEM_BYTES = OFF_OST + 8 * OST_WARP + 1024;  // + slack to align the base to 1024
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory plan exceeds 227 KB");
  static_assert((OFF_MISC + 16) % 16 == 0, "unit ring must be 16-byte aligned");
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t T_S0 = SHARED_S ? 0 : 2 * D, T_S1 = SHARED_S ? 0 : 2 * D + BN;
  static constexpr uint32_t T_P0 = SHARED_S ? BN : 2 * D + 2 * BN, T_P1 = T_P0 + BN / 2;
  static constexpr uint32_t T_O0 = SHARED_S ? 2 * BN : 0, T_O1 = T_O0 + D;
  static_assert(T_P1 + BN / 2 <= TMEM_COLS, "TMEM plan exceeds 512 columns");
};

template <int N>
__device__ __forceinline__ void ld_row(uint32_t taddr, float (&s)[N]) {
  if constexpr (N == 64) {
    uint32_t r[64];
    tmem_ld64_wait(taddr, r);
#pragma unroll
    for (int i = 0; i < 64; ++i) s[i] = __uint_as_float(r[i]);
  } else {
    uint32_t r[128];
    tmem_ld128_wait(taddr, r);
#pragma unroll
    for (int i = 0; i < 128; ++i) s[i] = __uint_as_float(r[i]);
  }
}

// Maximum of N values: eight running 3-input maxima and a short final tree.
template <int N>
__device__ __forceinline__ float row_max(const float (&s)[N]) {
  float a[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) a[k] = fmaxf(s[k], s[k + 8]);
#pragma unroll
  for (int i = 16; i < N; i += 16)
#pragma unroll
    for (int k = 0; k < 8; ++k) a[k] = max3(a[k], s[i + k], s[i + 8 + k]);
  return fmaxf(max3(a[0], a[1], a[2]), max3(a[3], a[4], max3(a[5], a[6], a[7])));
}

// V staging for bf16 inputs: Vh = fp16(V), per (head, chunk) flag = 1 if a finite V value of the
// chunk lies outside the fp16 range (it would become inf). Grid (n_chunks, BH), 16-byte vectors; n_chunks =
// v_chunks(BH), a multiple of 32, so that few heads still give every SM several blocks (with 32 chunks per
// head a 4-head call ran 128 blocks: 14-16 us for 32 MiB, latency-bound). Block (0, 0) also zeroes the two
// attention launches' work counters ctr[0], ctr[1], which they read only after this kernel completes, and a
// block that finds an overflow writes the call's generation `gen` into *any_ovf (the second launch runs only
// if it finds it there; a stale or arbitrary value merely costs that launch a scan).
// Launched with programmatic stream serialization: it waits for the previous work on the stream before
// touching memory (its scratch may be memory the previous call on the stream released).
__host__ __device__ constexpr int v_chunks(int BH) {
  return 32 * (BH >= 20 ? 1 : ((640 + 32 * BH - 1) / (32 * BH) < 16 ? (640 + 32 * BH - 1) / (32 * BH) : 16));
}

__global__ void __launch_bounds__(256)
stage_v_f16(const uint4* __restrict__ V, uint4* __restrict__ Vh, int* __restrict__ flags, long long vec_per_head,
            int n_chunks, int* __restrict__ ctr, unsigned long long* __restrict__ any_ovf, unsigned long long gen) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int bh = blockIdx.y;
  if (blockIdx.x == 0 && bh == 0 && threadIdx.x == 0) {
    ctr[0] = 0;
    ctr[1] = 0;
  }
  const long long per_chunk = (vec_per_head + n_chunks - 1) / n_chunks;
  const long long b = (long long)blockIdx.x * per_chunk;
  const long long e = min(vec_per_head, b + per_chunk);
  const uint4* src = V + (long long)bh * vec_per_head;
  uint4* dst = Vh + (long long)bh * vec_per_head;
  int ovf = 0;
  // four 16-byte loads in flight per thread (one at a time left small calls latency-bound)
  constexpr int kU = 4;
  for (long long i0 = b + threadIdx.x; i0 < e; i0 += kU * (long long)blockDim.x) {
    uint4 w[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const long long i = i0 + (long long)u * blockDim.x;
      if (i < e) w[u] = src[i];
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const long long i = i0 + (long long)u * blockDim.x;
      if (i >= e) continue;
      uint32_t in[4] = {w[u].x, w[u].y, w[u].z, w[u].w}, out[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float lo = __uint_as_float(in[j] << 16), hi = __uint_as_float(in[j] & 0xFFFF0000u);
        ovf |= (fabsf(lo) >= 65520.f && fabsf(lo) != CUDART_INF_F) | (fabsf(hi) >= 65520.f && fabsf(hi) != CUDART_INF_F);
        out[j] = pack2<false>(lo, hi);
      }
      dst[i] = make_uint4(out[0], out[1], out[2], out[3]);
    }
  }
  ovf = __syncthreads_or(ovf);
  if (threadIdx.x == 0) {
    flags[bh * n_chunks + blockIdx.x] = ovf;
    if (ovf) *any_ovf = gen;
  }
}

// p = exp2(s*scale - m_sub) for 64 scores of a row (s[OFF .. OFF+63]), packed as 16-bit pairs into p[32];
// returns the sum of the unrounded fp32 values. Column pairs c with c % 8 in {0, 3} take the
// polynomial exp2 on the FMA pipe, the others the MUFU ex2 unit (16 results per clock per SM). Measured
// on configs 2-4 against 0, 1, 3 and 4 of every 8 pairs (and other placements of 2): 2 of 8 at {0, 3}
// was fastest (+1.5% to +3.5% over 3 of 8).
// The polynomial clamps its argument at -125, so a masked score (-inf) or one more than 125 below the
// reference max gives 2^-125 instead of 0. In fp16 that rounds to 0, and in the row sum (>= 1) it is
// absorbed, so only bf16 P (heads whose V exceeds the fp16 range, where |V| may reach 1e38) needs the
// exact zero, which it gets here.
template <bool P_BF16, int OFF, int N>
__device__ __forceinline__ float softmax64(const float (&s)[N], float scale_log2, float m_sub, uint32_t (&p)[32]) {
  const float2 sc = make_float2(scale_log2, scale_log2), nm = make_float2(-m_sub, -m_sub);
  float2 acc[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
  for (int c = 0; c < 32; ++c) {
    float2 x = fma2(make_float2(s[OFF + 2 * c], s[OFF + 2 * c + 1]), sc, nm);
    if ((0x09 >> (c & 7)) & 1) {
      const float2 arg = x;
      x = exp2_fma2(x);
      if constexpr (P_BF16) {
        x.x = arg.x < -125.f ? 0.f : x.x;
        x.y = arg.y < -125.f ? 0.f : x.y;
      }
    } else {
      x.x = ex2(x.x);
      x.y = ex2(x.y);
    }
    acc[c & 1] = add2(acc[c & 1], x);
    p[c] = pack2<P_BF16>(x.x, x.y);
  }
  const float2 t = add2(acc[0], acc[1]);
  return t.x + t.y;
}

// BF16: input/output dtype. vflags (bf16 only): per-(head, chunk) fp16-overflow flags of V.
// Persistent: each CTA processes a sequence of work units (two 128-row Q tiles of one head); the K/V
// ring, the S sequence and every barrier phase run on across units, so the next unit's Q is loaded and
// its first S computed while the softmax warps still finish and write out the current unit.
// Last partial wave of a launch (host-chosen, see make_plan): query blocks from `from` on run as `pieces`
// units each - one-tile units (kv == 0: piece = Q tile of the block), or parts of the K/V range
// (kv == 1: piece p covers K/V tiles [p*n/P, (p+1)*n/P) of both Q tiles; each part leaves an unnormalised
// partial result, which merge_kv_parts combines after the launch). No tail: from = #blocks, pieces = 1.
struct Tail {
  int from;
  int pieces;
  int kv;
  float4* part_o;   // kv: per (tail block, Q tile, part) the partial O, [D/4][BM] float4 (lane-contiguous)
  float2* part_ml;  // kv: per (tail block, Q tile, part) the rows' (reference max, sum)
};

// (head, first query row) of query block `blk` in the unit order: heads in L2 groups of group_heads,
// inside a group the blocks from the last query block to the first (all heads of a group interleaved).
__device__ __forceinline__ void block_coords(int blk, int BH, int n_qblk, int group_heads, int* bh, int* qt0) {
  const int grp = blk / (group_heads * n_qblk);
  const int g_heads = min(group_heads, BH - grp * group_heads);
  const int r_in = blk - grp * group_heads * n_qblk;
  *bh = grp * group_heads + r_in % g_heads;
  *qt0 = 2 * (n_qblk - 1 - r_in / g_heads);
}

// KV_PARTS: the launch's tail is cut into K/V parts (Tail::kv = 1). A separate instantiation, so that every
// other launch runs a kernel without the parts' bookkeeping (measured: carrying it cost 2-5% per tile).
// OVF_HEADS (bf16 inputs): a bf16 call is two launches. The first (OVF_HEADS = false) computes P.V with fp16 P
// and the fp16 copy of V and skips every head whose V overflows fp16; the second (OVF_HEADS = true, launched
// after it) computes exactly those heads with bf16 P and the original V, and returns at once unless the
// staging kernel wrote this call's generation into *any_ovf. One kernel holding both P paths took 6-7% more
// cycles on every bf16 shape (ncu; the second exponential path costs code and registers in the hot loop).
template <int D, bool BF16, bool KV_PARTS, bool OVF_HEADS>
__global__ void __launch_bounds__(NUM_THREADS, 1)
attn_fwd_tc(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
            const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmVh,
            const __grid_constant__ CUtensorMap tmO, const int* __restrict__ vflags, int vchunks,
            const unsigned long long* __restrict__ any_ovf, unsigned long long gen,
            uint16_t* __restrict__ O, int BH, int N, float scale_log2, int causal,
            int group_heads, const Tail tail, int* __restrict__ status, int* __restrict__ work_ctr) {
  static_assert(BF16 || !OVF_HEADS, "only bf16 inputs have fp16-overflow heads");
  if constexpr (OVF_HEADS) {
    // before anything else (no barrier, no TMEM yet): wait for the work before this launch, then leave unless
    // some head of this call overflowed fp16 (the whole CTA takes the same branch)
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (*reinterpret_cast<const volatile unsigned long long*>(any_ovf) != gen) return;
  }
  using C = Cfg<D>;
  constexpr int BN = C::BN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + C::OFF_BAR;
  // q_full[u & 1]: unit u is published and its Q tiles have landed. Two barriers used by alternate units: a
  // consumer role may fall up to two units behind the producer (causal two-tile units of two K/V tiles, where
  // tile A runs one, let B and the issuers finish the next unit while A still writes its output), and
  // parity waits on a single barrier would then alias.
  auto q_full = [&](int u) { return (u & 1) ? bar0 + 8u * (14 + 2 * C::STAGES) : bar0; };
  auto kv_full = [&](int s) { return bar0 + 8u * (1 + s); };
  auto kv_empty = [&](int s) { return bar0 + 8u * (1 + C::STAGES + s); };
  auto s_full = [&](int g) { return bar0 + 8u * (1 + 2 * C::STAGES + g); };
  auto s_free = [&](int g) { return bar0 + 8u * (3 + 2 * C::STAGES + g); };
  auto p_ready = [&](int g) { return bar0 + 8u * (5 + 2 * C::STAGES + g); };
  auto o_done = [&](int g) { return bar0 + 8u * (7 + 2 * C::STAGES + g); };
  const uint32_t drain_bar = bar0 + 8u * (9 + 2 * C::STAGES);
  const uint32_t drain_pv_bar = bar0 + 8u * (10 + 2 * C::STAGES);
  auto q_free = [&]() { return bar0 + 8u * (11 + 2 * C::STAGES); };
  auto o_free = [&](int g) { return bar0 + 8u * (12 + 2 * C::STAGES + g); };
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);
  int4* unit_ring = reinterpret_cast<int4*>(smem + C::OFF_MISC + 16);  // [kUnitRing][2]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Work units: (head, query block of two 128-row Q tiles). Unit order: heads in groups of group_heads
  // whose K and V fit in L2 together; inside a group, the query blocks of all its heads from the
  // heaviest (causal: the most K/V tiles) to the lightest. CTA c starts with unit c; each further unit
  // is the next one in that order, taken with an atomic counter once the CTA has queued the copies of
  // its current unit, so SMs that run faster take more units (list scheduling, longest first). The
  // producer warp takes the units and publishes each (decoded) in a shared-memory ring before arriving
  // on q_full; the other roles read it after their wait on q_full (they are at most one unit behind, so
  // neither the phase nor the ring slot can be overtaken). A unit id of -1 ends every role's loop.
  // Query blocks from tail.from on (host-chosen, all two-tile) run as tail.pieces units each: one-tile
  // units, so that a last partial wave of r <= #CTAs/2 blocks becomes 2r short units, one per CTA; or
  // parts of the K/V range, so that a last wave of r > #CTAs/2 blocks spreads over all CTAs.
  const int n_qtiles = (N + BM - 1) / BM;
  const int n_qblk = (n_qtiles + 1) / 2;
  const int n_units = tail.from + (n_qblk * BH - tail.from) * tail.pieces;
  struct Unit {
    int bh, row0, kv0, n_kv;
    int part, tb;  // K/V part of a tail block (-1: the whole K/V range), tail block index
    int has_b;     // the unit has a second Q tile
    int id;        // unit index; -1 ends the roles' loops
  };
  auto unit_of = [&](int u) {
    Unit x;
    x.id = u;
    const bool in_tail = u >= tail.from;
    int blk, piece;
    if constexpr (KV_PARTS) {
      blk = in_tail ? tail.from + (u - tail.from) / tail.pieces : u;
      piece = in_tail ? (u - tail.from) % tail.pieces : 0;
    } else {  // the tail, if any, is one-tile units: two per block
      blk = in_tail ? tail.from + ((u - tail.from) >> 1) : u;
      piece = in_tail ? (u - tail.from) & 1 : 0;
    }
    const bool one_tile = !KV_PARTS && in_tail;
    int qt0;
    block_coords(blk, BH, n_qblk, group_heads, &x.bh, &qt0);
    qt0 += one_tile ? piece : 0;
    x.has_b = !one_tile && qt0 + 1 < n_qtiles;
    x.row0 = qt0 * BM;
    const int kv_end = causal ? min(N, x.row0 + (x.has_b ? 2 * BM : BM)) : N;
    const int n_kv = (kv_end + BN - 1) / BN;
    if constexpr (KV_PARTS) {
      x.part = in_tail ? piece : -1;
      x.tb = blk - tail.from;
      x.kv0 = in_tail ? piece * n_kv / tail.pieces : 0;
      x.n_kv = in_tail ? (piece + 1) * n_kv / tail.pieces - x.kv0 : n_kv;
    } else {
      x.part = -1;
      x.tb = 0;
      x.kv0 = 0;
      x.n_kv = n_kv;
    }
    return x;
  };
  // Whether a V value of head bh overflows fp16 (bf16 inputs; warp-wide: each lane ORs vchunks / 32 chunk
  // flags). Such heads belong to the OVF_HEADS launch, the others to the first one.
  auto head_overflows = [&](int bh) -> bool {
    if (!BF16) return false;
    int f = 0;
    for (int i = lane; i < vchunks; i += 32) f |= vflags[bh * vchunks + i];
    return __any_sync(0xffffffffu, f != 0);
  };

  if (threadIdx.x == 0) {
    mbar_init(q_full(0), 1);
    mbar_init(q_full(1), 1);
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(kv_full(s), 1);
      mbar_init(kv_empty(s), 1);
    }
    for (int g = 0; g < 2; ++g) {
      mbar_init(s_full(g), 1);
      mbar_init(s_free(g), 128);
      mbar_init(p_ready(g), 128);
      mbar_init(o_done(g), 1);
      mbar_init(o_free(g), 128);
    }
    mbar_init(drain_bar, 1);
    mbar_init(drain_pv_bar, 1);
    mbar_init(q_free(), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == MMA_WARP) {
    tmem_alloc(smem_u32(tmem_holder), C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  // Programmatic dependent launch (the launch sets programmaticStreamSerializationAllowed): let the next
  // kernel on this stream be scheduled now (its CTAs take SMs as ours exit), and wait here - before any
  // global memory access - until the work before this kernel has completed and its writes are visible, so
  // the prologue above (barriers, TMEM) overlaps the previous kernel's tail. Measured back to back, without
  // event records between the launches (an event in between orders them fully): config 5 N = 512 d = 64
  // +11%, N = 128 +2%, config 4 +0.5%, config 2 and N = 2048 d = 128 unchanged; bit-identical.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");

  // The producer decodes each unit once and publishes it (32 bytes) in the ring; the consumer roles read it
  // after their wait on q_full instead of decoding the id themselves (three integer divisions each).
  auto publish_unit = [&](int slot, const Unit& x) {
    unit_ring[2 * slot] = make_int4(x.bh, x.row0, x.kv0, x.n_kv);
    unit_ring[2 * slot + 1] = make_int4(x.part, x.tb, x.has_b, x.id);
  };
  auto read_unit = [&](int slot) {
    const int4 a = unit_ring[2 * slot], b = unit_ring[2 * slot + 1];
    Unit x;
    x.bh = a.x, x.row0 = a.y, x.kv0 = a.z, x.n_kv = a.w;
    x.part = b.x, x.tb = b.y, x.has_b = b.z, x.id = b.w;
    return x;
  };
  // Next unit of a consumer role: wait for the unit's q_full phase, read the published unit (id -1: none).
  auto next_unit = [&](int nu, bool& ok) -> Unit {
    ok = __all_sync(0xffffffffu, mbar_wait(q_full(nu), (nu >> 1) & 1, abort_flag, status, kErrMmaWait));
    if (ok) return read_unit(nu % kUnitRing);
    Unit x;
    x.id = -1;
    return x;
  };

  if (warp == TMA_WARP || warp == PV_WARP + 1) {
    setmaxnreg_dec<kRegsProducer>();
    if (warp == TMA_WARP) {
      // Producer, per unit: wait until the previous unit's last Q.K^T has read the Q buffer, publish the
      // unit, load its Q tiles, then K_0, V_0, K_1, V_1, ... into the ring (warp-uniform loop, one elected
      // lane issues copies), then reserve the next unit.
      int t = 0, nu = 0, nq_arrivals = 0;  // K/V copies, units issued, q_full phases started (+ end marker)
      int next_u = blockIdx.x;             // the unit this CTA runs next
      bool ok = true;
      auto take_unit = [&]() -> int {  // the next unit id from the work counter (one wave: none left)
        if (n_units <= (int)gridDim.x) return n_units;  // every unit was some CTA's first; no counter
        int got = 0;
        if (lane == 0) got = (int)gridDim.x + atomicAdd(work_ctr, 1);
        return __shfl_sync(0xffffffffu, got, 0);
      };
      // a unit of a head that the other launch of a bf16 call computes (OVF_HEADS)
      auto other_launch = [&](int u) -> bool {
        if constexpr (!BF16) return false;
        else return head_overflows(unit_of(u).bh) != OVF_HEADS;
      };
      if (elect_one()) {
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc((BF16 && !OVF_HEADS) ? &tmVh : &tmV);
        tma_prefetch_desc(&tmO);
      }
      __syncwarp();
      for (;;) {
        if (nu > 0 && !(ok = __all_sync(0xffffffffu, mbar_wait(q_free(), (nu - 1) & 1, abort_flag, status, kErrTmaWait))))
          break;
        int u = next_u;
        while (u < n_units && other_launch(u)) u = take_unit();
        if (u >= n_units) u = -1;
        if (u < 0) {
          if (elect_one()) {
            Unit end;
            end.bh = end.row0 = end.kv0 = end.n_kv = end.part = end.tb = end.has_b = 0;
            end.id = -1;
            publish_unit(nu % kUnitRing, end);
            mbar_arrive(q_full(nu));  // release semantics: the consumers' wait sees the unit
          }
          __syncwarp();
          ++nq_arrivals;
          break;
        }
        const Unit x = unit_of(u);
        const CUtensorMap* tm_v = (BF16 && !OVF_HEADS) ? &tmVh : &tmV;
        const int nq = x.has_b ? 2 : 1;
        if (elect_one()) {
          publish_unit(nu % kUnitRing, x);
          mbar_arrive_expect_tx(q_full(nu), nq * C::Q_TILE);
          for (int g = 0; g < nq; ++g)
            for (int c = 0; c < C::KBLK; ++c)
              tma_load_3d(sbase + C::OFF_Q + g * C::Q_TILE + c * C::Q_SUB, &tmQ, q_full(nu), c * 64, x.row0 + g * BM,
                          x.bh);
        }
        __syncwarp();
        ++nu;
        ++nq_arrivals;
        for (int jt = 0; jt < 2 * x.n_kv; ++jt, ++t) {
          const int s = t % C::STAGES, rr = t / C::STAGES;
          if (rr > 0 && !(ok = __all_sync(0xffffffffu, mbar_wait(kv_empty(s), (rr - 1) & 1, abort_flag, status, kErrTmaWait))))
            break;
          const CUtensorMap* m = (jt & 1) ? tm_v : &tmK;
          if (elect_one()) {
            mbar_arrive_expect_tx(kv_full(s), C::KV_TILE);
            for (int c = 0; c < C::KBLK; ++c)
              tma_load_3d(sbase + C::OFF_KV + s * C::KV_TILE + c * C::KV_SUB, m, kv_full(s), c * 64,
                          ((KV_PARTS ? x.kv0 : 0) + (jt >> 1)) * BN, x.bh);
          }
          __syncwarp();
        }
        if (!ok) break;
        // Reserve the next unit now that this unit's copies are all queued. Its Q load waits for q_free,
        // which follows this unit's last Q.K^T a few tiles later, so the counter's round trip (~1000 cycles)
        // no longer delays it (it did when the unit was taken after q_free). Reserving at the start of a
        // unit instead weakened the longest-first balance (measured 0.5-8% slower). One wave (units <= CTAs):
        // every unit was some CTA's first and the counter is not used.
        next_u = take_unit();
      }
      // Drain: every issued copy must land before this CTA's shared memory can be released.
      // (phases of a barrier complete in order: the last phase started on each q_full barrier covers its Q copies)
      for (int a = nq_arrivals - 2; a < nq_arrivals; ++a)
        if (a >= 0) mbar_wait_drain(q_full(a), (a >> 1) & 1);
      if (!ok) *abort_flag = 1;  // consumers waiting for a unit id stop at once
      for (int i = (t > C::STAGES ? t - C::STAGES : 0); i < t; ++i) mbar_wait_drain(kv_full(i % C::STAGES), (i / C::STAGES) & 1);
    }
  } else if (warp == MMA_WARP || warp == PV_WARP) {
    setmaxnreg_dec<kRegsProducer>();
    // Two MMA issuers, each a warp-uniform loop in which one elected lane (the same one every time, as
    // tcgen05.commit tracks the issuing thread's MMAs) issues tcgen05.mma and tcgen05.commit: warp 8
    // the S = Q K^T products, warp 10 the O += P V products. An issuer blocks while the tensor core's
    // instruction queue is full, so separate issuers keep the two dependency chains from waiting on
    // each other; they touch disjoint TMEM columns (S / P, O), and every cross dependency goes through
    // the softmax warps and the barriers below.
    {
      constexpr uint32_t idesc_qk = idesc_f16(BF16, BM, BN, false);
      // Descriptors are formed as (region base descriptor) + (byte offset >> 4): the start-address
      // field is the low 14 bits and every operand lies below 256 KB of shared memory, so the addition
      // never carries out of the field.
      const uint64_t dq = smem_desc_sw128(sbase + C::OFF_Q, 16, 1024);
      const uint64_t dk = smem_desc_sw128(sbase + C::OFF_KV, 16, 1024);
      const uint64_t dv = smem_desc_sw128(sbase + C::OFF_KV, C::KV_SUB, 1024);
      auto wait = [&](uint32_t bar, int parity) {
        return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, status, kErrMmaWait));
      };
      auto kv_wait = [&](int t) { return wait(kv_full(t % C::STAGES), (t / C::STAGES) & 1); };
      if (warp == MMA_WARP) {
        // S_g = Q_g K^T: K-major operands, 16 of d per instruction.
        auto issue_qk = [&](int g, int stage) {
          const uint32_t a_off = (uint32_t)(g * C::Q_TILE) >> 4, b_off = (uint32_t)(stage * C::KV_TILE) >> 4;
          const uint32_t d_t = tmem + (g ? C::T_S1 : C::T_S0);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t oa = ((kk >> 2) * C::Q_SUB + (kk & 3) * 32) >> 4;
            const uint32_t ob = ((kk >> 2) * C::KV_SUB + (kk & 3) * 32) >> 4;
            mma_ss(d_t, dq + (a_off + oa), dk + (b_off + ob), idesc_qk, kk > 0 ? 1u : 0u);
          }
        };
        // Per K tile, Q tile A then B. Shared S region (d = 128): one sequence of products over all units,
        // each issued once the softmax has read the previous one (s_free). One S region per Q tile
        // (d = 64): each product issued once that tile's softmax has read its previous S. After a unit's
        // last product, q_free lets the producer load the next unit's Q. Causal two-tile units: the last K
        // tile (keys row0 + 128 ... row0 + 255) lies entirely after tile A's rows, so only B runs it.
        int tb = 0, nu = 0, ks = 0;  // first K/V copy of the unit, units done, S products (shared S)
        int qc[2] = {0, 0};          // S products per Q tile (separate S)
        bool ok = true;
        for (;;) {
          const Unit x = next_unit(nu, ok);
          if (x.id < 0) break;
          const int ng = x.has_b ? 2 : 1;
          const bool skip_a = causal && x.has_b;  // tile A skips the unit's last K tile
          for (int q = 0; ok && q < x.n_kv; ++q) {
            const int tk = tb + 2 * q, sk = tk % C::STAGES;
            if (!(ok = kv_wait(tk))) break;
            // Unrolled over the two Q tiles. As a loop over [first, ng) the fp16 d = 128 instantiation took 13% more
            // cycles than the bf16 one (5.72 M against 5.06 M on B = 1, H = 32, N = 16384, ncu); unrolled, 4.73 M
            // (bf16 1% fewer, d = 64 unchanged).
#pragma unroll
            for (int g = 0; g < 2; ++g) {
              if (g >= ng || (g == 0 && skip_a && q == x.n_kv - 1)) continue;
              const int n_prev = C::SHARED_S ? ks : qc[g];
              if (n_prev > 0 && !(ok = wait(s_free(C::SHARED_S ? 0 : g), (n_prev - 1) & 1))) break;
              tc_fence_after();
              if (elect_one()) {
                issue_qk(g, sk);
                mma_commit(s_full(g));
                if (g == ng - 1) mma_commit(kv_empty(sk));
              }
              __syncwarp();
              if (C::SHARED_S) ++ks; else ++qc[g];
            }
          }
          if (!ok) break;
          if (elect_one()) mma_commit(q_free());
          __syncwarp();
          tb += 2 * x.n_kv;
          ++nu;
        }
        if (elect_one()) mma_commit(drain_bar);
        __syncwarp();
        mbar_wait_drain(drain_bar, 0);
      } else {
        // O_g += P_g V: P from TMEM (8 columns per 16 keys), V as an MN-major operand, 16 keys per
        // instruction; Q tile A then B for each V tile. A unit's first product overwrites O_g, so it
        // waits until the softmax has read the previous unit's O_g out (o_free).
        int tb = 0, nu = 0;
        int pc[2] = {0, 0}, uc[2] = {0, 0};  // P.V products and units per Q tile
        bool ok = true;
        for (;; ++nu) {
          const Unit x = next_unit(nu, ok);
          if (x.id < 0) break;
          const int ng = x.has_b ? 2 : 1;
          constexpr uint32_t idesc_pv = idesc_f16(OVF_HEADS, BM, D, true);  // bf16 P and V only in that launch
          auto issue_pv = [&](int g, int stage, bool acc) {
            const uint32_t b_off = (uint32_t)(stage * C::KV_TILE) >> 4;
            const uint32_t d_t = tmem + (g ? C::T_O1 : C::T_O0);
            const uint32_t p_t = tmem + (g ? C::T_P1 : C::T_P0);
#pragma unroll
            for (int kk = 0; kk < BN / 16; ++kk)
              mma_ts(d_t, p_t + kk * 8, dv + (b_off + kk * (2048 >> 4)), idesc_pv, (acc || kk > 0) ? 1u : 0u);
          };
          const bool skip_a = causal && x.has_b;  // tile A skips the unit's last V tile (all its keys masked)
          for (int p = 0; ok && p < x.n_kv; ++p) {
            const int tv = tb + 2 * p + 1, sv = tv % C::STAGES;
            if (!(ok = kv_wait(tv))) break;
            // (left as a loop: unrolled like the S products above, with pc[] and uc[] in registers, config 4 took
            // 4.8% more cycles)
            for (int g = (skip_a && p == x.n_kv - 1) ? 1 : 0; g < ng; ++g) {
              if (p == 0 && uc[g] > 0 && !(ok = wait(o_free(g), (uc[g] - 1) & 1))) break;
              if (!(ok = wait(p_ready(g), pc[g] & 1))) break;
              tc_fence_after();
              if (elect_one()) {
                issue_pv(g, sv, p > 0);
                mma_commit(o_done(g));
                if (g == ng - 1) mma_commit(kv_empty(sv));
              }
              __syncwarp();
              ++pc[g];
            }
          }
          if (!ok) break;
          for (int g = 0; g < ng; ++g) ++uc[g];
          tb += 2 * x.n_kv;
        }
        if (elect_one()) mma_commit(drain_pv_bar);
        __syncwarp();
        mbar_wait_drain(drain_pv_bar, 0);
      }
    }
  } else {
    // Softmax warpgroups: warps 0-3 own Q tile A, warps 4-7 Q tile B of every unit; thread t owns
    // query row t = TMEM lane t, so the row max and row sum need no shuffles. Per K/V tile: load S,
    // release the S columns, mask, take the max, wait for the previous P.V product (it reads P and
    // writes O), rescale O only when the max grew by more than 2^8 (exact: every P and l of a row use
    // the same reference max), write P = exp2(S*scale - m) as packed 16-bit pairs into the P columns,
    // then arrive. After a unit's last tile: O / l to global memory, then release O (o_free).
    setmaxnreg_inc<kRegsSoftmax>();
    const int g = warp >> 2;
    const int r_local = threadIdx.x & 127;  // row within the Q tile = TMEM lane
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t t_s = tmem + lane_off + (g ? C::T_S1 : C::T_S0);
    const uint32_t t_p = tmem + lane_off + (g ? C::T_P1 : C::T_P0);
    const uint32_t t_o = tmem + lane_off + (g ? C::T_O1 : C::T_O0);
    const uint32_t o_stage = sbase + C::OFF_OST + (uint32_t)warp * C::OST_WARP;  // this warp's O staging block
    int sc = 0, oc = 0;  // S products read and P.V products waited for, this Q tile, all units
    bool ok = true;
    for (int nu = 0;; ++nu) {
      Unit x = next_unit(nu, ok);
      if (x.id < 0) break;
      if (g == 1 && !x.has_b) continue;
      // causal two-tile unit: the last K/V tile lies entirely after tile A's rows, and A skips it
      const int n_kv = x.n_kv - ((causal && x.has_b && g == 0) ? 1 : 0);
      const int tile_row0 = x.row0 + g * BM;
      const int row = tile_row0 + r_local;
      float m_used = -CUDART_INF_F, l = 0.f;
      // d = 64 (one S region per Q tile): the next tile's S is normally complete long before its wait,
      // whose shared-memory probe runs at ~90-cycle latency while Q.K^T reads shared memory. So the
      // probe is issued mid-tile (non-blocking) and the wait skipped if it saw the phase complete; the
      // phase cannot advance again before this warp releases S. Measured +1.7% on config 2; at d = 128
      // the next S is usually not ready mid-tile and the probe did not pay.
      bool s_ready = false;
      for (int j = 0; j < n_kv; ++j) {
        if (!s_ready) {
          ok = __all_sync(0xffffffffu, mbar_wait(s_full(g), sc & 1, abort_flag, status, kErrSoftmaxWait));
          if (!ok) break;
        }
        ++sc;
        tc_fence_after();
        float s[BN];
        ld_row<BN>(t_s, s);
        tc_fence_before();
        mbar_arrive(s_free(C::SHARED_S ? 0 : g));  // the next Q.K^T may overwrite S now
        const int j0 = ((KV_PARTS ? x.kv0 : 0) + j) * BN;  // first key of this K/V tile
        if (j0 + BN > N || (causal && j0 + BN - 1 > tile_row0)) {
          // columns c >= lim lie past N or (causal) after this row
          const int lim = min(N, causal ? row + 1 : N) - j0;
#pragma unroll
          for (int c = 0; c < BN; ++c) s[c] = c < lim ? s[c] : -CUDART_INF_F;
        }
        const float m_new = row_max<BN>(s) * scale_log2;
        float alpha = 1.f;
        bool need = false;
        if (j == 0) {
          m_used = m_new;
        } else {
          need = m_new > m_used + kRescaleThreshold;
          if (need) {
            alpha = ex2(m_used - m_new);
            m_used = m_new;
          }
          // O += P_{j-1} V_{j-1} must be complete: it reads the P columns and writes O.
          ok = __all_sync(0xffffffffu, mbar_wait(o_done(g), oc & 1, abort_flag, status, kErrSoftmaxWait));
          if (!ok) break;
          ++oc;
          tc_fence_after();
          if (__any_sync(0xffffffffu, need)) {
            const float2 a2 = make_float2(alpha, alpha);  // 1 in rows that keep their reference max
#pragma unroll
            for (int c = 0; c < D / 32; ++c) {
              uint32_t rr[32];
              tmem_ld32_wait(t_o + c * 32, rr);
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const float2 x = mul2(make_float2(__uint_as_float(rr[2 * i]), __uint_as_float(rr[2 * i + 1])), a2);
                rr[2 * i] = __float_as_uint(x.x);
                rr[2 * i + 1] = __float_as_uint(x.y);
              }
              tmem_st32(t_o + c * 32, rr);
            }
          }
        }
        const float m_sub = m_used == -CUDART_INF_F ? 0.f : m_used;
        uint32_t p[32];
        float psum = softmax64<OVF_HEADS, 0>(s, scale_log2, m_sub, p);
        tmem_st32(t_p, p);
        bool next_test = false;
        if constexpr (!C::SHARED_S) next_test = j + 1 < n_kv && mbar_test(s_full(g), sc & 1);
        if constexpr (BN == 128) {
          psum += softmax64<OVF_HEADS, 64>(s, scale_log2, m_sub, p);
          tmem_st32(t_p + 32, p);
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(p_ready(g));
        if constexpr (!C::SHARED_S) s_ready = __all_sync(0xffffffffu, next_test);
        l = l * alpha + psum;
      }
      if (!ok) break;
      ok = __all_sync(0xffffffffu, mbar_wait(o_done(g), oc & 1, abort_flag, status, kErrEpilogueWait));
      if (!ok) break;
      ++oc;
      tc_fence_after();
      x = read_unit(nu % kUnitRing);  // read again: fewer registers live across the tile loop
      if (!KV_PARTS || x.part < 0) {
        // O / l through shared memory to a TMA store: each warp writes its 32 rows, 64 columns at a time, into
        // its staging block in the output map's 128-byte swizzled layout (16-byte chunk k of a row at chunk
        // k ^ (row % 8): conflict-free) and lane 0 stores the block; the store runs asynchronously, clipped at
        // row N. Storing each thread's row straight to global memory (32 rows per warp instruction) took
        // 1-3 K cycles per unit and held up the warp's next shared-memory accesses while the stores drained.
        const float inv_l = 1.f / l;
        const int wrow0 = tile_row0 + (warp & 3) * 32;  // first row of this warp's 32-row slab
#pragma unroll
        for (int cb = 0; cb < D / 64; ++cb) {
          if (lane == 0) bulk_wait_read_all();  // the previous store from this block has read it
          __syncwarp();
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint32_t rr[32];
            tmem_ld32_wait(t_o + cb * 64 + h * 32, rr);
            uint32_t w[16];
#pragma unroll
            for (int i = 0; i < 16; ++i)
              w[i] = pack2<BF16>(__uint_as_float(rr[2 * i]) * inv_l, __uint_as_float(rr[2 * i + 1]) * inv_l);
#pragma unroll
            for (int k = 0; k < 4; ++k)
              st_shared_v4(o_stage + lane * 128 + (uint32_t)(((4 * h + k) ^ (lane & 7)) * 16), w[4 * k], w[4 * k + 1],
                           w[4 * k + 2], w[4 * k + 3]);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && wrow0 < N) {
            tma_store_3d(&tmO, o_stage, cb * 64, wrow0, x.bh);
            bulk_commit();
          }
        }
      } else if constexpr (KV_PARTS) {
        // K/V part of a tail block: leave this row's unnormalised O, reference max and sum; merge_kv_parts,
        // launched after this kernel on the same stream, combines the parts and writes the row of O.
        float4* po = tail.part_o + ((((size_t)x.tb * 2 + g) * tail.pieces + x.part) * (D / 4)) * BM + r_local;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t rr[32];
          tmem_ld32_wait(t_o + c * 32, rr);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            po[(size_t)(c * 8 + i) * BM] = make_float4(__uint_as_float(rr[4 * i]), __uint_as_float(rr[4 * i + 1]),
                                                       __uint_as_float(rr[4 * i + 2]), __uint_as_float(rr[4 * i + 3]));
        }
        tail.part_ml[(((size_t)x.tb * 2 + g) * tail.pieces + x.part) * BM + r_local] = make_float2(m_used, l);
      }
      tc_fence_before();
      mbar_arrive(o_free(g));  // the next unit's first P.V may overwrite O now
    }
    if (lane == 0) bulk_wait_all();  // this warp's O stores have completed (and read its staging block)
  }

  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// Merge of the K/V parts of a launch's tail blocks. Block (tail block, Q tile, 16-column chunk); thread =
// query row. m = max_p m_p, O = sum_p 2^(m_p - m) O_p / sum_p 2^(m_p - m) l_p, summed over the parts in
// their fixed order (results do not depend on which part ran first or where). All of a thread's loads (the
// parts' (max, sum) pairs and their 16 columns of O, up to kMaxParts parts) are issued before any is used:
// with a 32-column chunk and the parts read one after another the merge of the 4-head config-4 shard was
// latency-bound (14.6 us for 57 MB, mostly from L2). bf16 inputs: blocks of heads whose V overflows fp16
// were not cut into parts (the second launch computes them whole) and are skipped.
constexpr int kMergeCols = 16;
template <int D, bool BF16>
__global__ void __launch_bounds__(BM)
merge_kv_parts(const float4* __restrict__ part_o, const float2* __restrict__ part_ml, uint16_t* __restrict__ O,
               int BH, int N, int n_qblk, int group_heads, int tail_from, int P, const int* __restrict__ vflags,
               int vchunks) {
  constexpr int kMaxP = 8;  // = kMaxParts (host side)
  asm volatile("griddepcontrol.wait;" ::: "memory");  // launched as a programmatic dependent of the attention kernel
  const int tb = blockIdx.x, g = blockIdx.y, c = blockIdx.z, r = threadIdx.x;
  int bh, qt0;
  block_coords(tail_from + tb, BH, n_qblk, group_heads, &bh, &qt0);
  if constexpr (BF16) {
    int f = 0;
    for (int i = r; i < vchunks; i += BM) f |= vflags[bh * vchunks + i];
    if (__syncthreads_or(f)) return;  // whole block: the head belongs to the second launch
  }
  const int row = (qt0 + g) * BM + r;
  if (qt0 + g >= (N + BM - 1) / BM || row >= N) return;  // no second Q tile / past the end
  const size_t slot0 = ((size_t)tb * 2 + g) * P;
  float2 ml[kMaxP];
  float4 v[kMaxP][kMergeCols / 4];
#pragma unroll
  for (int q = 0; q < kMaxP; ++q) {
    if (q < P) {
      ml[q] = part_ml[(slot0 + q) * BM + r];
      const float4* po = part_o + (slot0 + q) * (D / 4) * BM + r;
#pragma unroll
      for (int i = 0; i < kMergeCols / 4; ++i) v[q][i] = po[(size_t)(c * (kMergeCols / 4) + i) * BM];
    }
  }
  float m = -CUDART_INF_F;
#pragma unroll
  for (int q = 0; q < kMaxP; ++q)
    if (q < P) m = fmaxf(m, ml[q].x);
  float acc[kMergeCols], lt = 0.f;
#pragma unroll
  for (int i = 0; i < kMergeCols; ++i) acc[i] = 0.f;
#pragma unroll
  for (int q = 0; q < kMaxP; ++q) {
    if (q < P) {
      const float w = ex2(ml[q].x - m);
      lt = fmaf(w, ml[q].y, lt);
#pragma unroll
      for (int i = 0; i < kMergeCols / 4; ++i) {
        acc[4 * i] = fmaf(w, v[q][i].x, acc[4 * i]);
        acc[4 * i + 1] = fmaf(w, v[q][i].y, acc[4 * i + 1]);
        acc[4 * i + 2] = fmaf(w, v[q][i].z, acc[4 * i + 2]);
        acc[4 * i + 3] = fmaf(w, v[q][i].w, acc[4 * i + 3]);
      }
    }
  }
  const float inv_l = 1.f / lt;
  uint32_t w[kMergeCols / 2];
#pragma unroll
  for (int i = 0; i < kMergeCols / 2; ++i) w[i] = pack2<BF16>(acc[2 * i] * inv_l, acc[2 * i + 1] * inv_l);
  uint16_t* dst = O + ((size_t)bh * N + row) * D + c * kMergeCols;
  if ((reinterpret_cast<uintptr_t>(O) & 31) == 0) {
    st_global_v8(dst, w);
  } else {
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int i = 0; i < kMergeCols / 8; ++i) d4[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
  }
}

// Failure-path probe: one warp waits, with the same bounded mbarrier wait the attention kernel uses,
// on a barrier that nothing arrives on. The wait gives up after kWaitLimitCycles, raises the abort
// flag and ORs kErrProbeWait into the status word; a second wait then returns at once on the flag.
// `status2` (may be null): a second status word that gets the same bit once the wait has expired (the
// allocation-free entry point's own word). Nothing is left in flight (no copies, no MMAs, no TMEM), so
// the context stays usable.
constexpr int kErrProbeWait = 16;

__global__ void __launch_bounds__(32, 1) wait_expiry_probe(int* __restrict__ status, int* __restrict__ status2) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncwarp();
  const bool first = mbar_wait(smem_u32(&bar), 0, &abort_flag, status, kErrProbeWait);
  const bool second = mbar_wait(smem_u32(&bar), 0, &abort_flag, status, kErrProbeWait);
  if (threadIdx.x == 0 && (first || second)) atomicOr(status, 1 << 30);  // a wait completed: impossible
  if (threadIdx.x == 0 && !first && status2 != nullptr) atomicOr(status2, kErrProbeWait);
}

// Zeroes the persistent CTAs' work counter of an fp16 call (bf16 calls have the staging kernel do it). A kernel
// rather than a memset, so that the stream's programmatic-launch chain stays unbroken: it waits for the work
// before it, and the attention kernel after it is scheduled as it exits and waits for it in turn.
__global__ void __launch_bounds__(32, 1) zero_counter(int* __restrict__ ctr) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (threadIdx.x == 0) ctr[0] = 0;
}

}  // namespace tc

// ------------------------------------------------------------------------------------ host side
namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// (d, N, BH) view of a contiguous (BH, N, d) 16-bit array; 64 x rows x 1 boxes, 128-byte swizzle.
// Rows past N read as zeros, per head.
bool encode_map(CUtensorMap* m, const void* base, int BH, int N, int d, bool bf16, int rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[3] = {(cuuint64_t)d, (cuuint64_t)N, (cuuint64_t)BH};
  const cuuint64_t strides[2] = {(cuuint64_t)d * 2, (cuuint64_t)N * d * 2};
  const cuuint32_t box[3] = {64, (cuuint32_t)rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Per-thread cache of encoded maps. A map is a pure function of (base, BH, N, d, dtype, rows), so a
// cached copy stays correct even after the caller frees and reuses an address; the cache only saves
// the host-side encoding on calls that repeat their buffers.
constexpr int kMapCache = 16;
struct MapEntry {
  CUtensorMap map;
  const void* base = nullptr;
  int BH = 0, N = 0, d = 0, rows = 0;
  bool bf16 = false, valid = false;
};
thread_local MapEntry g_maps[kMapCache];
thread_local int g_map_next = 0;

bool make_map(CUtensorMap* m, const void* base, int BH, int N, int d, bool bf16, int rows) {
  for (const MapEntry& e : g_maps)
    if (e.valid && e.base == base && e.BH == BH && e.N == N && e.d == d && e.rows == rows && e.bf16 == bf16) {
      *m = e.map;
      return true;
    }
  if (!encode_map(m, base, BH, N, d, bf16, rows)) return false;
  MapEntry& e = g_maps[g_map_next];
  g_map_next = (g_map_next + 1) % kMapCache;
  e.map = *m;
  e.base = base;
  e.BH = BH, e.N = N, e.d = d, e.rows = rows;
  e.bf16 = bf16;
  e.valid = true;
  return true;
}

// Stream-ordered scratch of each launch (its work counter and, for bf16 inputs, the staged V): one
// memory pool per device, owned by the library, that keeps freed blocks cached (release threshold =
// max) so repeated calls do not go back to the driver. Allocation and free are ordered on the caller's
// stream, so concurrent calls on different streams each get their own block.
constexpr int kMaxDevices = 64;
cudaMemPool_t g_pool[kMaxDevices] = {};
std::mutex g_pool_mu;

cudaError_t device_pool(int dev, cudaMemPool_t* out) {
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_pool_mu);
  if (g_pool[dev] == nullptr) {
    cudaMemPoolProps props = {};
    props.allocType = cudaMemAllocationTypePinned;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = dev;
    cudaMemPool_t pool;
    cudaError_t e = cudaMemPoolCreate(&pool, &props);
    if (e != cudaSuccess) return e;
    uint64_t keep = ~0ull;
    e = cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
    if (e != cudaSuccess) return e;
    g_pool[dev] = pool;
  }
  *out = g_pool[dev];
  return cudaSuccess;
}

// Launch shape of one call: persistent grid, L2 head groups, the last partial wave's split (tail), and
// whether the CTAs take units from a work counter (more units than CTAs).
struct Plan {
  unsigned grid = 0;
  int group_heads = 1;
  int tail_from = 0;    // first query block of the tail (= #blocks: no tail)
  int tail_pieces = 1;  // units per tail block
  bool tail_kv = false; // pieces are K/V parts (else one-tile units)
  int n_tail = 0;       // tail blocks
  bool uses_counter = false;
};

// K/V parts per tail block: the fewest parts P (2..8, at least kMinPartTiles K/V tiles each) that minimise
// the tail's length ceil(r*P/G)/P (in units of one block's time), used only if the launch's predicted length
// falls by at least kMinPartGain: waves + 1 -> waves + that length. The parts cost time of their own (each
// part restarts the pipeline and writes its partial result, merge_kv_parts reads them all), and units of
// earlier waves end at staggered times, so the last wave is less idle than this count says. Measured on a
// B200: config 4 (13 full waves + 124 of 148 blocks, predicted 1%) was 2.6% slower with 7 parts; config 4's
// 8-GPU shard (1 full wave + 108 blocks, predicted 12.5%) runs 3.6% faster with 4 parts; parts of 8 K/V tiles
// (config 3's 8-GPU shard) lost 24% with an in-kernel merge, hence at least 16 tiles per part.
constexpr int kMaxParts = 8;
static_assert(kMaxParts <= 8, "merge_kv_parts holds at most 8 parts' loads in registers");
constexpr int kMinPartTiles = 16;
constexpr double kMinPartGain = 0.08;
int kv_parts(long long waves, long long r, long long grid, int n_kv) {
  int best = 1;
  double best_len = 1.0;
  for (int P = 2; P <= kMaxParts && n_kv / P >= kMinPartTiles; ++P) {
    const double len = (double)((r * P + grid - 1) / grid) / P;
    if (len < best_len - 1e-9) {
      best_len = len;
      best = P;
    }
  }
  return (waves + 1.0) / (waves + best_len) >= 1.0 + kMinPartGain ? best : 1;
}

// Per-device launch facts, written once per device (std::atomic: several host threads may launch).
std::atomic<bool> g_attr_set[2][kMaxDevices];
std::atomic<int> g_sm_count[kMaxDevices];

template <int D>
cudaError_t make_plan(const LaunchArgs& a, int dev, bool allow_kv_parts, Plan* p) {
  const int n_qtiles = (a.N + tc::BM - 1) / tc::BM;
  const int n_qblk = (n_qtiles + 1) / 2;
  if ((long long)n_qblk * a.BH > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  // Persistent grid: one CTA per SM (at most one per work unit).
  int n_sm = g_sm_count[dev].load(std::memory_order_relaxed);
  if (n_sm == 0) {
    cudaError_t e = cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    g_sm_count[dev].store(n_sm, std::memory_order_relaxed);
  }
  const LaunchShape& shape = launch_shape();
  if (shape.max_ctas > 0) n_sm = std::min(n_sm, shape.max_ctas);
  const long long n_blk = (long long)n_qblk * a.BH;
  p->grid = (unsigned)std::min<long long>(n_blk, n_sm);
  // Heads per scheduling group: K and V of a group (4*N*d bytes per head) within ~16 MiB of L2. The
  // persistent CTAs drift apart in their K/V streams, so a group's whole K/V is live in L2 at once; with
  // 48 MiB groups config 4 read its K/V 2-2.3x from DRAM, with 16 MiB once (ncu), at equal speed.
  const long long kv_bytes = 4LL * a.N * D;
  const long long group_bytes = shape.l2_group_kib > 0 ? shape.l2_group_kib << 10 : 16LL << 20;
  p->group_heads = (int)std::max(1LL, std::min((long long)a.BH, group_bytes / kv_bytes));
  // Tail (non-causal): a last partial wave of r query blocks with 2r <= CTAs runs as 2r one-tile units,
  // one per CTA, instead of r two-tile units on r CTAs while the others idle. Only two-tile blocks are
  // split: with an odd tile count the one-tile blocks are the first of each head group. A larger last
  // wave (r > CTAs/2, e.g. config 4 on 8 GPUs: 256 blocks on 148 CTAs) has its blocks' K/V ranges cut
  // into P parts (kv_parts), so that its r*P shorter units spread over every CTA.
  p->tail_from = (int)n_blk;
  p->tail_pieces = 1;
  p->tail_kv = false;
  if (!a.causal && n_blk > p->grid) {
    const long long r = n_blk % p->grid;
    const long long n_groups = (a.BH + p->group_heads - 1) / p->group_heads;
    const long long last_group = (n_groups - 1) * p->group_heads * n_qblk;
    const long long last_heads = a.BH - (n_groups - 1) * p->group_heads;
    const bool odd_tiles = n_qtiles % 2 != 0;
    const bool two_tile_tail = !odd_tiles || n_blk - r >= last_group + last_heads;
    const int n_kv = (a.N + tc::Cfg<D>::BN - 1) / tc::Cfg<D>::BN;
    if (r > 0 && 2 * r <= p->grid && two_tile_tail && n_blk + r <= 0x7fffffffLL) {
      p->tail_from = (int)(n_blk - r);
      p->tail_pieces = 2;
    } else if (r > 0 && allow_kv_parts && launch_shape().kv_parts && two_tile_tail) {
      const int P = kv_parts(n_blk / p->grid, r, p->grid, n_kv);
      if (P > 1 && n_blk + r * (P - 1) <= 0x7fffffffLL) {
        p->tail_from = (int)(n_blk - r);
        p->tail_pieces = P;
        p->tail_kv = true;
      }
    }
  }
  p->n_tail = (int)n_blk - p->tail_from;
  // A launch of one wave (units <= CTAs) never reads the work counter.
  p->uses_counter = (long long)p->tail_from + (long long)p->n_tail * p->tail_pieces > (long long)p->grid;
  return cudaSuccess;
}

// Device memory one call works in besides its inputs and output. `ctr`: ctr[0] the persistent CTAs' work
// counter; bf16 inputs also ctr[1], the work counter of the launch for fp16-overflow heads, and at ctr + 2 a
// 64-bit word the staging kernel sets to the call's generation `gen` when some head overflows (16 bytes in all;
// the counters are zeroed on the call's stream before the attention kernels run). `part_o`, `part_ml`: the K/V
// parts' partial results. `vh`, `flags` (bf16 inputs only): the fp16 copy of V and its per-(head, chunk)
// fp16-overflow flags.
struct Scratch {
  int* ctr = nullptr;
  float4* part_o = nullptr;
  float2* part_ml = nullptr;
  void* vh = nullptr;
  int* flags = nullptr;
  unsigned long long gen = 0;
};

// A value unique to each bf16 call in this process (never 0): what the staging kernel writes into the call's
// overflow word, so the word needs no zeroing (a leftover value of another call can only differ).
unsigned long long next_generation() {
  static std::atomic<unsigned long long> count{0};
  return 0x9E3779B97F4A7C15ull * (count.fetch_add(1, std::memory_order_relaxed) + 1);
}

size_t round256(size_t b) { return (b + 255) & ~size_t(255); }
// Bytes of the work counter (zeroed before each launch) and of the K/V parts' partial results of a plan, 0
// when unused; counter_bytes() is the 256-byte-aligned room the counter takes in an allocation.
size_t counters_used(const Plan& p, bool bf16) { return bf16 ? 16 : (p.uses_counter ? sizeof(int) : 0); }
size_t counter_bytes(const Plan& p, bool bf16) { return round256(counters_used(p, bf16)); }
size_t part_o_bytes(const Plan& p, int d) {
  return p.tail_kv ? (size_t)p.n_tail * 2 * p.tail_pieces * tc::BM * d * sizeof(float) : 0;
}
size_t part_ml_bytes(const Plan& p) {
  return p.tail_kv ? round256((size_t)p.n_tail * 2 * p.tail_pieces * tc::BM * sizeof(float2)) : 0;
}

template <int D, bool BF16>
cudaError_t launch_t(const LaunchArgs& a, const Plan& p, const CUtensorMap& mq, const CUtensorMap& mk,
                     const CUtensorMap& mv, const CUtensorMap& mvh, const Scratch& s, int dev) {
  auto kern = p.tail_kv ? tc::attn_fwd_tc<D, BF16, true, false> : tc::attn_fwd_tc<D, BF16, false, false>;
  constexpr int smem = tc::Cfg<D>::SMEM_BYTES;
  std::atomic<bool>& attr = g_attr_set[D == 128 ? 1 : 0][dev];
  if (!attr.load(std::memory_order_acquire)) {
    // Every instantiation of one head dimension has the same shared-memory size; setting it twice is
    // harmless, so two threads racing here need no lock.
    cudaError_t e = cudaSuccess;
    for (auto f : {tc::attn_fwd_tc<D, false, false, false>, tc::attn_fwd_tc<D, true, false, false>,
                   tc::attn_fwd_tc<D, false, true, false>, tc::attn_fwd_tc<D, true, true, false>,
                   tc::attn_fwd_tc<D, true, false, true>})
      if (e == cudaSuccess) e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    attr.store(true, std::memory_order_release);
  }
  if (((p.uses_counter || BF16) && s.ctr == nullptr) || (p.tail_kv && (s.part_o == nullptr || s.part_ml == nullptr)))
    return cudaErrorInvalidValue;
  const unsigned long long* any_ovf = BF16 ? reinterpret_cast<const unsigned long long*>(s.ctr + 2) : nullptr;
  const int vchunks = tc::v_chunks(a.BH);
  // O is written by TMA stores of 32-row x 64-column blocks (one per softmax warp), clipped at row N
  CUtensorMap mo;
  if (!make_map(&mo, a.o, a.BH, a.N, D, BF16, 32)) return cudaErrorInvalidValue;
  const float scale_log2 = 1.4426950408889634f / sqrtf((float)D);
  tc::Tail tail{p.tail_from, p.tail_pieces, p.tail_kv ? 1 : 0, s.part_o, s.part_ml};
  timing_begin(a.stream);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.grid);
  cfg.blockDim = dim3(tc::NUM_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = a.stream;
  cudaLaunchAttribute attr_pdl[1];
  attr_pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr_pdl[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr_pdl;
  cfg.numAttrs = 1;
  cudaError_t el = cudaLaunchKernelEx(&cfg, kern, mq, mk, mv, mvh, mo, (const int*)s.flags, vchunks, any_ovf, s.gen,
                                      static_cast<uint16_t*>(a.o), a.BH, a.N, scale_log2, a.causal ? 1 : 0,
                                      p.group_heads, tail, a.status, s.ctr);
  if (el != cudaSuccess) return el;
  note_launch();
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess && p.tail_kv) {
    // programmatic dependent launch: the merge's blocks are scheduled as the attention CTAs exit and wait in
    // the kernel (griddepcontrol.wait) for the whole attention grid, instead of for a launch after it
    const int n_qblk = ((a.N + tc::BM - 1) / tc::BM + 1) / 2;
    cudaLaunchConfig_t mcfg = {};
    mcfg.gridDim = dim3(p.n_tail, 2, D / tc::kMergeCols);
    mcfg.blockDim = dim3(tc::BM);
    mcfg.stream = a.stream;
    mcfg.attrs = attr_pdl;
    mcfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&mcfg, tc::merge_kv_parts<D, BF16>, (const float4*)s.part_o, (const float2*)s.part_ml,
                           static_cast<uint16_t*>(a.o), a.BH, a.N, n_qblk, p.group_heads, p.tail_from, p.tail_pieces,
                           (const int*)s.flags, vchunks);
    if (e == cudaSuccess) {
      note_launch();
      e = cudaGetLastError();
    }
  }
  if constexpr (BF16) {
    // The launch for heads whose V overflows fp16: every query block whole (no tail split), its own work counter;
    // it returns at once when the staging kernel found no overflow in this call.
    if (e == cudaSuccess) {
      const long long n_blk = (long long)(((a.N + tc::BM - 1) / tc::BM + 1) / 2) * a.BH;
      tc::Tail whole{(int)n_blk, 1, 0, nullptr, nullptr};
      cudaLaunchConfig_t ocfg = cfg;  // same persistent grid, block, shared memory, stream, programmatic launch
      e = cudaLaunchKernelEx(&ocfg, tc::attn_fwd_tc<D, true, false, true>, mq, mk, mv, mvh, mo, (const int*)s.flags,
                             vchunks, any_ovf, s.gen, static_cast<uint16_t*>(a.o), a.BH, a.N, scale_log2,
                             a.causal ? 1 : 0, p.group_heads, whole, a.status, s.ctr + 1);
      if (e == cudaSuccess) {
        note_launch();
        e = cudaGetLastError();
      }
    }
  }
  timing_end(a.stream);
  return e;
}

// One call in the scratch `s`: zero the work counter (fp16: zero_counter; bf16: the staging kernel does it), stage
// V as fp16 (bf16), run the attention kernel.
template <int D>
cudaError_t run_d(const LaunchArgs& a, const Plan& p, const CUtensorMap& mq, const CUtensorMap& mk,
                  const CUtensorMap& mv, const Scratch& s, int dev) {
  const bool bf16 = a.dtype == PHANTOM_ATTN_BF16;
  if (counters_used(p, bf16) && !bf16) {
    cudaLaunchConfig_t zcfg = {};
    zcfg.gridDim = dim3(1);
    zcfg.blockDim = dim3(32);
    zcfg.stream = a.stream;
    cudaLaunchAttribute zpdl[1];
    zpdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    zpdl[0].val.programmaticStreamSerializationAllowed = 1;
    zcfg.attrs = zpdl;
    zcfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&zcfg, tc::zero_counter, s.ctr);
    if (e != cudaSuccess) return e;
    note_launch();
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  if (!bf16) return launch_t<D, false>(a, p, mq, mk, mv, mv, s, dev);
  const long long vec_per_head = (long long)a.N * D / 8;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tc::v_chunks(a.BH), a.BH);
  cfg.blockDim = dim3(256);
  cfg.stream = a.stream;
  cudaLaunchAttribute attr_pdl[1];
  attr_pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr_pdl[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr_pdl;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, tc::stage_v_f16, static_cast<const uint4*>(a.v), static_cast<uint4*>(s.vh),
                                     s.flags, vec_per_head, tc::v_chunks(a.BH), s.ctr,
                                     reinterpret_cast<unsigned long long*>(s.ctr + 2), s.gen);
  if (e != cudaSuccess) return e;
  note_launch();
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  CUtensorMap mvh;
  if (!make_map(&mvh, s.vh, a.BH, a.N, D, false, tc::Cfg<D>::BN)) return cudaErrorInvalidValue;
  return launch_t<D, true>(a, p, mq, mk, mv, mvh, s, dev);
}

size_t staged_v_bytes(int BH, int N, int d) { return (size_t)BH * N * d * 2; }
size_t flag_bytes(int BH) { return (size_t)BH * tc::v_chunks(BH) * sizeof(int); }

// Allocating path: the launch's scratch [counters | K/V-part partials | fp16 V | flags] is one block from
// the library's stream-ordered pool, taken and released on the caller's stream. Launches that overlap on
// the GPU (other streams, other threads) therefore never share a counter or a buffer.
template <int D>
cudaError_t launch_alloc(const LaunchArgs& a, const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                         int dev) {
  Plan p;
  cudaError_t e = make_plan<D>(a, dev, true, &p);
  if (e != cudaSuccess) return e;
  const bool bf16 = a.dtype == PHANTOM_ATTN_BF16;
  const size_t cb = counter_bytes(p, bf16), ob = part_o_bytes(p, D), mb = part_ml_bytes(p);
  const size_t need = cb + ob + mb + (bf16 ? staged_v_bytes(a.BH, a.N, D) + flag_bytes(a.BH) : 0);
  if (need == 0) return run_d<D>(a, p, mq, mk, mv, Scratch{}, dev);
  cudaMemPool_t pool;
  if ((e = device_pool(dev, &pool)) != cudaSuccess) return e;
  void* block = nullptr;
  if ((e = cudaMallocFromPoolAsync(&block, need, pool, a.stream)) != cudaSuccess) return e;
  char* base = static_cast<char*>(block);
  Scratch s;
  if (cb) s.ctr = reinterpret_cast<int*>(base);
  if (bf16) s.gen = next_generation();
  if (ob) {
    s.part_o = reinterpret_cast<float4*>(base + cb);
    s.part_ml = reinterpret_cast<float2*>(base + cb + ob);
  }
  if (bf16) {
    s.vh = base + cb + ob + mb;
    s.flags = reinterpret_cast<int*>(base + cb + ob + mb + staged_v_bytes(a.BH, a.N, D));
  }
  e = run_d<D>(a, p, mq, mk, mv, s, dev);
  const cudaError_t ef = cudaFreeAsync(block, a.stream);
  return e != cudaSuccess ? e : ef;
}

// Caller-supplied scratch (no allocation): the counters (and, for bf16, the overflow word; 16 bytes) at `ctr`,
// [fp16 V | flags] at `scratch`. The tail is never cut into K/V parts here (their partial results would need
// more scratch).
template <int D>
cudaError_t launch_given(const LaunchArgs& a, const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                         int dev, int* ctr, void* scratch) {
  Plan p;
  cudaError_t e = make_plan<D>(a, dev, false, &p);
  if (e != cudaSuccess) return e;
  Scratch s;
  s.ctr = ctr;
  if (a.dtype == PHANTOM_ATTN_BF16) s.gen = next_generation();
  if (a.dtype == PHANTOM_ATTN_BF16) {
    s.vh = scratch;
    s.flags = reinterpret_cast<int*>(static_cast<char*>(scratch) + staged_v_bytes(a.BH, a.N, D));
  }
  return run_d<D>(a, p, mq, mk, mv, s, dev);
}

bool input_maps(const LaunchArgs& a, CUtensorMap* mq, CUtensorMap* mk, CUtensorMap* mv) {
  const bool bf16 = a.dtype == PHANTOM_ATTN_BF16;
  const int bn = a.d == 64 ? tc::Cfg<64>::BN : tc::Cfg<128>::BN;
  return make_map(mq, a.q, a.BH, a.N, a.d, bf16, tc::BM) && make_map(mk, a.k, a.BH, a.N, a.d, bf16, bn) &&
         make_map(mv, a.v, a.BH, a.N, a.d, bf16, bn);
}

cudaError_t current_dev(int* dev) {
  cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return e;
  return (*dev < 0 || *dev >= kMaxDevices) ? cudaErrorInvalidDevice : cudaSuccess;
}

}  // namespace

size_t fused_tc_smem_bytes(int d) { return d == 64 ? tc::Cfg<64>::SMEM_BYTES : tc::Cfg<128>::SMEM_BYTES; }

size_t fused_tc_scratch_bytes(int BH, int N, int d, int dtype) {
  if (dtype != PHANTOM_ATTN_BF16) return 0;
  return staged_v_bytes(BH, N, d) + flag_bytes(BH);
}

cudaError_t launch_fused_tc_sm100_scratch(const LaunchArgs& a, int* work_ctr, void* scratch) {
  int dev = 0;
  cudaError_t e = current_dev(&dev);
  if (e != cudaSuccess) return e;
  CUtensorMap mq, mk, mv;
  if (!input_maps(a, &mq, &mk, &mv)) return cudaErrorInvalidValue;
  return a.d == 64 ? launch_given<64>(a, mq, mk, mv, dev, work_ctr, scratch)
                   : launch_given<128>(a, mq, mk, mv, dev, work_ctr, scratch);
}

cudaError_t launch_fused_tc_sm100(const LaunchArgs& a) {
  int dev = 0;
  cudaError_t e = current_dev(&dev);
  if (e != cudaSuccess) return e;
  CUtensorMap mq, mk, mv;
  if (!input_maps(a, &mq, &mk, &mv)) return cudaErrorInvalidValue;
  return a.d == 64 ? launch_alloc<64>(a, mq, mk, mv, dev) : launch_alloc<128>(a, mq, mk, mv, dev);
}

cudaError_t scratch_usage(int dev, long long* high_water, long long* reserved, bool reset) {
  *high_water = 0;
  *reserved = 0;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  cudaMemPool_t pool = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_pool_mu);
    pool = g_pool[dev];
  }
  if (pool == nullptr) return cudaSuccess;  // no call on this device has needed scratch yet
  uint64_t hw = 0, rs = 0;
  cudaError_t e = cudaMemPoolGetAttribute(pool, cudaMemPoolAttrUsedMemHigh, &hw);
  if (e == cudaSuccess) e = cudaMemPoolGetAttribute(pool, cudaMemPoolAttrReservedMemCurrent, &rs);
  if (e == cudaSuccess && reset) {
    uint64_t zero = 0;
    e = cudaMemPoolSetAttribute(pool, cudaMemPoolAttrUsedMemHigh, &zero);
  }
  *high_water = (long long)hw;
  *reserved = (long long)rs;
  return e;
}

cudaError_t launch_wait_expiry_probe(int* status, int* status2, cudaStream_t stream) {
  tc::wait_expiry_probe<<<1, 32, 0, stream>>>(status, status2);
  note_launch();
  return cudaGetLastError();
}

}  // namespace phantom
