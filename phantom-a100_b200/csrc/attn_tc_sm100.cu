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
// finite value beyond the fp16 range falls back to bf16 P and the original bf16 V for that head.
//
// B200 mapping (not a translation of the WMMA kernel):
//   * One CTA owns two 128-row Q tiles (A, B) of one (batch, head) and streams K/V tiles of 128 keys.
//   * Warp 9 (one thread) is the TMA producer: Q tiles once, then K_0, V_0, K_1, V_1, ... into a ring
//     of STAGES shared-memory slots (128-byte swizzle), completion tracked by mbarrier tx bytes.
//   * Warp 8 (one thread) issues every tcgen05.mma: S_g = Q_g K_j^T (both operands in shared memory,
//     fp32 accumulator in TMEM, 128 lanes x 128 columns) and O_g += P_g V_j (P read from TMEM,
//     V from shared memory as an MN-major operand, accumulator in TMEM). Commits go to mbarriers.
//   * Warps 0-3 / 4-7 are the softmax warpgroups of tiles A / B: thread t owns query row t = TMEM
//     lane t, so the row max and row sum need no shuffles. Each thread loads its S row from TMEM,
//     masks, takes the max, rescales its O row in TMEM only when the max grew by more than 2^8
//     (exact: every P and l of a row use the same reference max), computes P with ex2, writes it
//     back into the S columns as packed 16-bit pairs (the A operand of the next MMA), then arrives.
//   * While one warpgroup runs its softmax the tensor core works on the other tile's MMAs.
//   * TMEM: S_A [0,128), S_B [128,256), O_A [256,256+d), O_B [256+d,256+2d); P_g aliases S_g.
//   * Every mbarrier wait is bounded; on expiry the CTA drains its in-flight copies and MMAs,
//     frees TMEM, records the failure in the device status word and exits.
#include <cuda.h>
#include <math_constants.h>

#include <mutex>

#include "launchers.h"
#include "sm100_ptx.cuh"
#include "../../include/phantom_attn.h"

namespace phantom {
namespace tc {

constexpr int BM = 128;  // query rows per Q tile = TMEM lanes
constexpr int BN = 128;  // keys per K/V tile
constexpr int MMA_WARP = 8;
constexpr int TMA_WARP = 9;          // warps 10-11 complete the producer warpgroup and idle
constexpr int NUM_THREADS = 384;
// Register split (setmaxnreg): the kernel launches at 168 registers/thread (384 threads, 1 CTA/SM).
// The producer warpgroup drops to 72 and the two softmax warpgroups rise to 216:
// 128*(168-72) = 2*128*(216-168), so the increase is exactly covered by the release.
constexpr int kRegsProducer = 72;
constexpr int kRegsSoftmax = 216;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale O only when the max grows by > 2^8

// Status-word bits (which wait expired).
constexpr int kErrTmaWait = 1, kErrMmaWait = 2, kErrSoftmaxWait = 4, kErrEpilogueWait = 8;

template <int D>
struct Cfg {
  static constexpr int KBLK = D / 64;                // 64-element (128-byte) swizzle blocks across d
  static constexpr int SUB_BYTES = BM * 128;         // one 64-column block of a 128-row tile
  static constexpr int TILE_BYTES = BM * D * 2;      // one Q, K or V tile
  static constexpr int STAGES = D == 128 ? 4 : 8;    // K/V ring slots
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_KV = 2 * TILE_BYTES;
  static constexpr int OFF_BAR = OFF_KV + STAGES * TILE_BYTES;
  // barriers: q_full, kv_full[STAGES], kv_empty[STAGES], s_full[2], p_ready[2], o_done[2], drain,
  // p_half[2]
  static constexpr int NUM_BARS = 1 + 2 * STAGES + 9;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;  // TMEM base address, abort flag
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;  // + slack to align the base to 1024
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t T_S0 = 0, T_S1 = 128, T_O0 = 256, T_O1 = 256 + D;
};

__device__ __forceinline__ void ld128(uint32_t taddr, float (&s)[128]) {
  uint32_t r[128];
  tmem_ld128_wait(taddr, r);
#pragma unroll
  for (int i = 0; i < 128; ++i) s[i] = __uint_as_float(r[i]);
}

// Maximum of 128 values: a 5-level tree of 3-input maxima (64 instructions, short dependency chain).
__device__ __forceinline__ float row_max128(const float (&s)[128]) {
  float x[43];
#pragma unroll
  for (int i = 0; i < 42; ++i) x[i] = max3(s[3 * i], s[3 * i + 1], s[3 * i + 2]);
  x[42] = fmaxf(s[126], s[127]);
  float y[15];
#pragma unroll
  for (int i = 0; i < 14; ++i) y[i] = max3(x[3 * i], x[3 * i + 1], x[3 * i + 2]);
  y[14] = x[42];
  float z[5];
#pragma unroll
  for (int i = 0; i < 5; ++i) z[i] = max3(y[3 * i], y[3 * i + 1], y[3 * i + 2]);
  return max3(max3(z[0], z[1], z[2]), z[3], z[4]);
}

// V staging for bf16 inputs: Vh = fp16(V), per (head, chunk) flag = 1 if a finite V value of the
// chunk lies outside the fp16 range (it would become inf). Grid (kVChunks, BH), 16-byte vectors.
constexpr int kVChunks = 32;

__global__ void __launch_bounds__(256)
stage_v_f16(const uint4* __restrict__ V, uint4* __restrict__ Vh, int* __restrict__ flags, long long vec_per_head) {
  const int bh = blockIdx.y;
  const long long per_chunk = (vec_per_head + kVChunks - 1) / kVChunks;
  const long long b = (long long)blockIdx.x * per_chunk;
  const long long e = min(vec_per_head, b + per_chunk);
  const uint4* src = V + (long long)bh * vec_per_head;
  uint4* dst = Vh + (long long)bh * vec_per_head;
  int ovf = 0;
  for (long long i = b + threadIdx.x; i < e; i += blockDim.x) {
    const uint4 w = src[i];
    uint32_t in[4] = {w.x, w.y, w.z, w.w}, out[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float lo = __uint_as_float(in[j] << 16), hi = __uint_as_float(in[j] & 0xFFFF0000u);
      ovf |= (fabsf(lo) >= 65520.f && fabsf(lo) != CUDART_INF_F) | (fabsf(hi) >= 65520.f && fabsf(hi) != CUDART_INF_F);
      out[j] = pack2<false>(lo, hi);
    }
    dst[i] = make_uint4(out[0], out[1], out[2], out[3]);
  }
  ovf = __syncthreads_or(ovf);
  if (threadIdx.x == 0) flags[bh * kVChunks + blockIdx.x] = ovf;
}

// Half a row of the softmax (columns H*64 .. H*64+63 of an S row held in registers): replaces each
// score by p = exp2(s*scale - m_sub) in place (fp32, unrounded, kept for the row sum) and packs the
// 64 values as 16-bit pairs into p[32]. Scale-and-subtract uses packed two-lane fp32 instructions; the
// MUFU ex2 unit (16 results per clock per SM) would otherwise bound this loop, so 3 of every 8 column
// pairs take the polynomial exp2 on the FMA pipe instead (exp2_fma2).
template <bool P_BF16, int H>
__device__ __forceinline__ void softmax_half(float (&s)[128], float scale_log2, float m_sub, uint32_t (&p)[32]) {
  const float2 sc = make_float2(scale_log2, scale_log2), nm = make_float2(-m_sub, -m_sub);
#pragma unroll
  for (int c = 0; c < 32; ++c) {
    const int i = H * 64 + 2 * c;
    float2 x = fma2(make_float2(s[i], s[i + 1]), sc, nm);
    if ((c & 7) < 3) {
      x = exp2_fma2(x);
    } else {
      x.x = ex2(x.x);
      x.y = ex2(x.y);
    }
    s[i] = x.x;
    s[i + 1] = x.y;
    p[c] = pack2<P_BF16>(x.x, x.y);
  }
}

// Sum of the 128 unrounded p values of a row (packed two-lane adds, four independent chains).
__device__ __forceinline__ float row_sum128(const float (&s)[128]) {
  float2 acc[4] = {make_float2(s[0], s[1]), make_float2(s[2], s[3]), make_float2(s[4], s[5]), make_float2(s[6], s[7])};
#pragma unroll
  for (int c = 4; c < 64; ++c) acc[c & 3] = add2(acc[c & 3], make_float2(s[2 * c], s[2 * c + 1]));
  const float2 t = add2(add2(acc[0], acc[1]), add2(acc[2], acc[3]));
  return t.x + t.y;
}

// BF16: input/output dtype. vflags (bf16 only): per-(head, chunk) fp16-overflow flags of V.
template <int D, bool BF16>
__global__ void __launch_bounds__(NUM_THREADS, 1)
attn_fwd_tc(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
            const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmVh,
            const int* __restrict__ vflags, uint16_t* __restrict__ O, int N, float scale_log2, int causal,
            int* __restrict__ status) {
  using C = Cfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + C::OFF_BAR;
  auto q_full = [&]() { return bar0; };
  auto kv_full = [&](int s) { return bar0 + 8u * (1 + s); };
  auto kv_empty = [&](int s) { return bar0 + 8u * (1 + C::STAGES + s); };
  auto s_full = [&](int g) { return bar0 + 8u * (1 + 2 * C::STAGES + g); };
  auto p_ready = [&](int g) { return bar0 + 8u * (3 + 2 * C::STAGES + g); };
  auto o_done = [&](int g) { return bar0 + 8u * (5 + 2 * C::STAGES + g); };
  const uint32_t drain_bar = bar0 + 8u * (7 + 2 * C::STAGES);
  auto p_half = [&](int g) { return bar0 + 8u * (8 + 2 * C::STAGES + g); };
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);
  int* pv_bf16_flag = reinterpret_cast<int*>(smem + C::OFF_MISC + 8);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.y;
  const int n_qtiles = (N + BM - 1) / BM;
  const int qblk = gridDim.x - 1 - blockIdx.x;  // heaviest (causal) blocks first
  const int qt0 = 2 * qblk;
  const bool has_b = qt0 + 1 < n_qtiles;
  const int row0 = qt0 * BM;
  const int kv_end = causal ? min(N, row0 + (has_b ? 2 * BM : BM)) : N;
  const int n_kv = (kv_end + BN - 1) / BN;

  if (threadIdx.x == 0) {
    mbar_init(q_full(), 1);
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(kv_full(s), 1);
      mbar_init(kv_empty(s), 1);
    }
    for (int g = 0; g < 2; ++g) {
      mbar_init(s_full(g), 1);
      mbar_init(p_ready(g), 128);
      mbar_init(p_half(g), 128);
      mbar_init(o_done(g), 1);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == MMA_WARP) {
    tmem_alloc(smem_u32(tmem_holder), C::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == MMA_WARP + 2) {
    // P.V precision of this head: fp16 unless a V value of the head overflows fp16 (bf16 inputs).
    int ovf = 0;
    if (BF16) ovf = vflags[bh * kVChunks + lane] != 0;
    ovf = __any_sync(0xffffffffu, ovf);
    if (lane == 0) *pv_bf16_flag = ovf;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const bool pv_bf16 = BF16 && *pv_bf16_flag != 0;  // CTA-uniform

  if (warp == TMA_WARP || warp >= MMA_WARP + 2) {
    setmaxnreg_dec<kRegsProducer>();
    if (warp == TMA_WARP) {
      // Producer: warp-uniform loop, one elected lane issues the copies.
      const CUtensorMap* tm_v = (BF16 && !pv_bf16) ? &tmVh : &tmV;
      const int nq = has_b ? 2 : 1;
      if (elect_one()) {
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(tm_v);
        mbar_arrive_expect_tx(q_full(), nq * C::TILE_BYTES);
        for (int g = 0; g < nq; ++g)
          for (int c = 0; c < C::KBLK; ++c)
            tma_load_3d(sbase + C::OFF_Q + g * C::TILE_BYTES + c * C::SUB_BYTES, &tmQ, q_full(), c * 64,
                        row0 + g * BM, bh);
      }
      __syncwarp();
      int issued = 0;
      for (int t = 0; t < 2 * n_kv; ++t) {
        const int s = t % C::STAGES, r = t / C::STAGES;
        if (r > 0) {
          const bool ok = __all_sync(0xffffffffu, mbar_wait(kv_empty(s), (r - 1) & 1, abort_flag, status, kErrTmaWait));
          if (!ok) break;
        }
        const CUtensorMap* m = (t & 1) ? tm_v : &tmK;
        const int j = t >> 1;
        if (elect_one()) {
          mbar_arrive_expect_tx(kv_full(s), C::TILE_BYTES);
          for (int c = 0; c < C::KBLK; ++c)
            tma_load_3d(sbase + C::OFF_KV + s * C::TILE_BYTES + c * C::SUB_BYTES, m, kv_full(s), c * 64, j * BN, bh);
        }
        __syncwarp();
        issued = t + 1;
      }
      // Drain: every issued copy must land before this CTA's shared memory can be released.
      mbar_wait_drain(q_full(), 0);
      for (int t = (issued > C::STAGES ? issued - C::STAGES : 0); t < issued; ++t)
        mbar_wait_drain(kv_full(t % C::STAGES), (t / C::STAGES) & 1);
    }
  } else if (warp == MMA_WARP) {
    setmaxnreg_dec<kRegsProducer>();
    // MMA issuer: the whole warp runs this warp-uniform loop and waits on the barriers; one elected
    // lane (the same one every time, as tcgen05.commit tracks the issuing thread's MMAs) issues the
    // tcgen05.mma and tcgen05.commit instructions.
    {
      constexpr uint32_t idesc_qk = idesc_f16(BF16, BM, BN, false);
      const uint32_t idesc_pv = idesc_f16(pv_bf16, BM, D, true);
      // Descriptors are formed as (region base descriptor) + (byte offset >> 4): the start-address
      // field is the low 14 bits and every operand lies below 256 KB of shared memory, so the addition
      // never carries out of the field.
      const uint64_t dq = smem_desc_sw128(sbase + C::OFF_Q, 16, 1024);
      const uint64_t dk = smem_desc_sw128(sbase + C::OFF_KV, 16, 1024);
      const uint64_t dv = smem_desc_sw128(sbase + C::OFF_KV, C::SUB_BYTES, 1024);
      auto issue_qk = [&](int g, int stage) {
        const uint32_t a_off = (uint32_t)(g * C::TILE_BYTES) >> 4, b_off = (uint32_t)(stage * C::TILE_BYTES) >> 4;
        const uint32_t d_t = tmem + (g ? C::T_S1 : C::T_S0);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = ((kk >> 2) * C::SUB_BYTES + (kk & 3) * 32) >> 4;
          mma_ss(d_t, dq + (a_off + off), dk + (b_off + off), idesc_qk, kk > 0 ? 1u : 0u);
        }
      };
      // P.V in two halves of 64 keys each (k steps 0-3 and 4-7), issued as each half of P lands.
      auto issue_pv = [&](int g, int stage, bool acc, int half) {
        const uint32_t b_off = (uint32_t)(stage * C::TILE_BYTES) >> 4;
        const uint32_t d_t = tmem + (g ? C::T_O1 : C::T_O0);
        const uint32_t p_t = tmem + (g ? C::T_S1 : C::T_S0);
#pragma unroll
        for (int k = 0; k < BN / 32; ++k) {
          const int kk = half * (BN / 32) + k;
          mma_ts(d_t, p_t + kk * 8, dv + (b_off + kk * (2048 >> 4)), idesc_pv, (acc || kk > 0) ? 1u : 0u);
        }
      };
      auto wait = [&](uint32_t bar, int parity) {
        return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, status, kErrMmaWait));
      };
      auto kv_wait = [&](int t) { return wait(kv_full(t % C::STAGES), (t / C::STAGES) & 1); };
      // Issue order (ping-pong): tile A's P.V and its next Q.K^T go out as soon as softmax A hands P
      // over, independently of tile B, so each softmax warpgroup overlaps the other tile's MMAs. The
      // next S_g = Q_g K^T is issued right behind O_g += P_g V, although S_g's columns hold P_g: the
      // tensor pipe executes one CTA's MMAs in issue order, so the P.V product has read P_g before the
      // Q.K^T product writes there (the published FlashAttention-4 Blackwell kernel relies on the same
      // ordering; the parity tests check the results bit for bit across reruns).
      bool ok = wait(q_full(), 0) && kv_wait(0);
      if (ok) {
        tc_fence_after();
        if (elect_one()) {
          issue_qk(0, 0);
          mma_commit(s_full(0));
          if (has_b) {
            issue_qk(1, 0);
            mma_commit(s_full(1));
          }
          mma_commit(kv_empty(0));
        }
        __syncwarp();
      }
      for (int j = 0; ok && j < n_kv; ++j) {
        const int tv = 2 * j + 1, tk = 2 * j + 2;  // positions of V_j and K_{j+1} in the load sequence
        const int sv = tv % C::STAGES, sk = tk % C::STAGES;
        const bool more = j + 1 < n_kv;
        if (!(ok = kv_wait(tv))) break;
        // ---- tile A: O_A += P_A V_j, then S_A = Q_A K_{j+1}^T
        if (!(ok = wait(p_half(0), j & 1))) break;
        tc_fence_after();
        if (elect_one()) issue_pv(0, sv, j > 0, 0);
        __syncwarp();
        if (!(ok = wait(p_ready(0), j & 1))) break;
        tc_fence_after();
        if (elect_one()) {
          issue_pv(0, sv, j > 0, 1);
          mma_commit(o_done(0));
        }
        __syncwarp();
        if (more) {
          if (!(ok = kv_wait(tk))) break;
          tc_fence_after();
          if (elect_one()) {
            issue_qk(0, sk);
            mma_commit(s_full(0));
          }
          __syncwarp();
        }
        // ---- tile B
        if (has_b) {
          if (!(ok = wait(p_half(1), j & 1))) break;
          tc_fence_after();
          if (elect_one()) issue_pv(1, sv, j > 0, 0);
          __syncwarp();
          if (!(ok = wait(p_ready(1), j & 1))) break;
          tc_fence_after();
          if (elect_one()) {
            issue_pv(1, sv, j > 0, 1);
            mma_commit(o_done(1));
            mma_commit(kv_empty(sv));
          }
          __syncwarp();
          if (more) {
            if (elect_one()) {
              issue_qk(1, sk);
              mma_commit(s_full(1));
              mma_commit(kv_empty(sk));
            }
            __syncwarp();
          }
        } else {
          if (elect_one()) {
            mma_commit(kv_empty(sv));
            if (more) mma_commit(kv_empty(sk));
          }
          __syncwarp();
        }
      }
      // Drain: all MMAs issued by the elected lane complete before TMEM is released.
      if (elect_one()) mma_commit(drain_bar);
      __syncwarp();
      mbar_wait_drain(drain_bar, 0);
    }
  } else {
    // Softmax warpgroups.
    setmaxnreg_inc<kRegsSoftmax>();
    const int g = warp >> 2;
    const int r_local = threadIdx.x & 127;  // row within the Q tile = TMEM lane
    if (g == 0 || has_b) {
      const int tile_row0 = row0 + g * BM;
      const int row = tile_row0 + r_local;
      const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
      const uint32_t t_s = tmem + lane_off + (g ? C::T_S1 : C::T_S0);
      const uint32_t t_o = tmem + lane_off + (g ? C::T_O1 : C::T_O0);
      float m_used = -CUDART_INF_F, l = 0.f;
      bool ok = true;
      for (int j = 0; j < n_kv; ++j) {
        ok = mbar_wait(s_full(g), j & 1, abort_flag, status, kErrSoftmaxWait);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        float s[128];
        ld128(t_s, s);
        const int j0 = j * BN;
        if (j0 + BN > N || (causal && j0 + BN - 1 > tile_row0)) {
#pragma unroll
          for (int c = 0; c < BN; ++c) {
            const int col = j0 + c;
            if (col >= N || (causal && col > row)) s[c] = -CUDART_INF_F;
          }
        }
        const float m_new = row_max128(s) * scale_log2;
        if (j == 0) {
          m_used = m_new;
        } else {
          const bool need = m_new > m_used + kRescaleThreshold;
          if (__any_sync(0xffffffffu, need)) {
            float alpha = 1.f;
            if (need) {
              alpha = ex2(m_used - m_new);
              m_used = m_new;
            }
            l *= alpha;
#pragma unroll
            for (int c = 0; c < D / 32; ++c) {
              uint32_t r[32];
              tmem_ld32_wait(t_o + c * 32, r);
#pragma unroll
              for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
              tmem_st32(t_o + c * 32, r);
            }
          }
        }
        const float m_sub = m_used == -CUDART_INF_F ? 0.f : m_used;
        // P for keys 0-63 goes out first: the MMA warp starts the P.V product on it while keys 64-127
        // are still being exponentiated; the row sum comes after both halves are handed over.
        uint32_t p[32];
        if (pv_bf16)
          softmax_half<true, 0>(s, scale_log2, m_sub, p);
        else
          softmax_half<false, 0>(s, scale_log2, m_sub, p);
        tmem_st32(t_s, p);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(p_half(g));
        if (pv_bf16)
          softmax_half<true, 1>(s, scale_log2, m_sub, p);
        else
          softmax_half<false, 1>(s, scale_log2, m_sub, p);
        tmem_st32(t_s + 32, p);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(p_ready(g));
        l += row_sum128(s);
      }
      if (ok) {
        ok = mbar_wait(o_done(g), (n_kv - 1) & 1, abort_flag, status, kErrEpilogueWait);
        ok = __all_sync(0xffffffffu, ok);
      }
      if (ok) {
        tc_fence_after();
        const float inv_l = 1.f / l;
        uint16_t* out = O + ((size_t)bh * N + row) * D;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t r[32];
          tmem_ld32_wait(t_o + c * 32, r);
          uint32_t w[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            w[i] = pack2<BF16>(__uint_as_float(r[2 * i]) * inv_l, __uint_as_float(r[2 * i + 1]) * inv_l);
          if (row < N) {
            uint4* dst = reinterpret_cast<uint4*>(out + c * 32);
#pragma unroll
            for (int i = 0; i < 4; ++i) dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
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

// (d, N, BH) view of a contiguous (BH, N, d) 16-bit array; 64 x 128 x 1 boxes, 128-byte swizzle.
// Rows past N read as zeros, per head.
bool make_map(CUtensorMap* m, const void* base, int BH, int N, int d, bool bf16) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[3] = {(cuuint64_t)d, (cuuint64_t)N, (cuuint64_t)BH};
  const cuuint64_t strides[2] = {(cuuint64_t)d * 2, (cuuint64_t)N * d * 2};
  const cuuint32_t box[3] = {64, (cuuint32_t)tc::BM, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Stream-ordered scratch for the bf16 V staging: one memory pool per device, owned by the library,
// that keeps freed blocks cached (release threshold = max) so repeated calls do not go back to the
// driver. Allocation and free are ordered on the caller's stream, so concurrent calls on different
// streams each get their own block.
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

template <int D, bool BF16>
cudaError_t launch_t(const LaunchArgs& a, const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                     const CUtensorMap& mvh, const int* vflags) {
  auto kern = tc::attn_fwd_tc<D, BF16>;
  constexpr int smem = tc::Cfg<D>::SMEM_BYTES;
  static bool attr_set[kMaxDevices] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < kMaxDevices && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  const int n_qtiles = (a.N + tc::BM - 1) / tc::BM;
  const dim3 grid((n_qtiles + 1) / 2, a.BH);
  const float scale_log2 = 1.4426950408889634f / sqrtf((float)D);
  timing_begin(a.stream);
  kern<<<grid, tc::NUM_THREADS, smem, a.stream>>>(mq, mk, mv, mvh, vflags, static_cast<uint16_t*>(a.o), a.N,
                                                   scale_log2, a.causal ? 1 : 0, a.status);
  timing_end(a.stream);
  note_launch();
  return cudaGetLastError();
}

template <int D>
cudaError_t launch_d(const LaunchArgs& a, const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv) {
  if (a.dtype != PHANTOM_ATTN_BF16) return launch_t<D, false>(a, mq, mk, mv, mv, nullptr);
  // bf16: stage V as fp16 in stream-ordered scratch [Vh | flags], run, release.
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  cudaMemPool_t pool;
  if ((e = device_pool(dev, &pool)) != cudaSuccess) return e;
  const size_t vh_bytes = (size_t)a.BH * a.N * D * 2;
  const size_t flag_bytes = (size_t)a.BH * tc::kVChunks * sizeof(int);
  void* scratch = nullptr;
  if ((e = cudaMallocFromPoolAsync(&scratch, vh_bytes + flag_bytes, pool, a.stream)) != cudaSuccess) return e;
  void* vh = scratch;
  int* flags = reinterpret_cast<int*>(static_cast<char*>(scratch) + vh_bytes);
  const long long vec_per_head = (long long)a.N * D / 8;
  tc::stage_v_f16<<<dim3(tc::kVChunks, a.BH), 256, 0, a.stream>>>(
      static_cast<const uint4*>(a.v), static_cast<uint4*>(vh), flags, vec_per_head);
  note_launch();
  e = cudaGetLastError();
  CUtensorMap mvh;
  if (e == cudaSuccess && !make_map(&mvh, vh, a.BH, a.N, D, false)) e = cudaErrorInvalidValue;
  if (e == cudaSuccess) e = launch_t<D, true>(a, mq, mk, mv, mvh, flags);
  const cudaError_t ef = cudaFreeAsync(scratch, a.stream);
  return e != cudaSuccess ? e : ef;
}

// Same as launch_d, with the bf16 staging buffer [Vh | flags] supplied by the caller (no allocation).
template <int D>
cudaError_t launch_d_scratch(const LaunchArgs& a, const CUtensorMap& mq, const CUtensorMap& mk,
                             const CUtensorMap& mv, void* scratch) {
  if (a.dtype != PHANTOM_ATTN_BF16) return launch_t<D, false>(a, mq, mk, mv, mv, nullptr);
  const size_t vh_bytes = (size_t)a.BH * a.N * D * 2;
  void* vh = scratch;
  int* flags = reinterpret_cast<int*>(static_cast<char*>(scratch) + vh_bytes);
  const long long vec_per_head = (long long)a.N * D / 8;
  tc::stage_v_f16<<<dim3(tc::kVChunks, a.BH), 256, 0, a.stream>>>(
      static_cast<const uint4*>(a.v), static_cast<uint4*>(vh), flags, vec_per_head);
  note_launch();
  cudaError_t e = cudaGetLastError();
  CUtensorMap mvh;
  if (e == cudaSuccess && !make_map(&mvh, vh, a.BH, a.N, D, false)) e = cudaErrorInvalidValue;
  if (e == cudaSuccess) e = launch_t<D, true>(a, mq, mk, mv, mvh, flags);
  return e;
}

}  // namespace

size_t fused_tc_smem_bytes(int d) { return d == 64 ? tc::Cfg<64>::SMEM_BYTES : tc::Cfg<128>::SMEM_BYTES; }

size_t fused_tc_scratch_bytes(int BH, int N, int d, int dtype) {
  if (dtype != PHANTOM_ATTN_BF16) return 0;
  return (size_t)BH * N * d * 2 + (size_t)BH * tc::kVChunks * sizeof(int);
}

cudaError_t launch_fused_tc_sm100_scratch(const LaunchArgs& a, void* scratch) {
  const bool bf16 = a.dtype == PHANTOM_ATTN_BF16;
  CUtensorMap mq, mk, mv;
  if (!make_map(&mq, a.q, a.BH, a.N, a.d, bf16) || !make_map(&mk, a.k, a.BH, a.N, a.d, bf16) ||
      !make_map(&mv, a.v, a.BH, a.N, a.d, bf16))
    return cudaErrorInvalidValue;
  return a.d == 64 ? launch_d_scratch<64>(a, mq, mk, mv, scratch) : launch_d_scratch<128>(a, mq, mk, mv, scratch);
}

cudaError_t launch_fused_tc_sm100(const LaunchArgs& a) {
  const bool bf16 = a.dtype == PHANTOM_ATTN_BF16;
  CUtensorMap mq, mk, mv;
  if (!make_map(&mq, a.q, a.BH, a.N, a.d, bf16) || !make_map(&mk, a.k, a.BH, a.N, a.d, bf16) ||
      !make_map(&mv, a.v, a.BH, a.N, a.d, bf16))
    return cudaErrorInvalidValue;
  return a.d == 64 ? launch_d<64>(a, mq, mk, mv) : launch_d<128>(a, mq, mk, mv);
}

}  // namespace phantom
