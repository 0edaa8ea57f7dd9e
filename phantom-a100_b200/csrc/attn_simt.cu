// Fused attention forward on CUDA cores with fp32 arithmetic (any head dim up to 256; fp32, fp16 or
// bf16 storage). This is the exact-precision path behind the reference's v1/v2/v3 entry points
// (csrc/kernels/naive.cuh, tiled.cuh, fused.cuh), which the reference tests hold to 1e-4 in fp32
// (tests/test_correctness.py:12). Tensor cores would round Q/K/V (TF32) and miss that tolerance.
//
// Same algorithm as the reference's v3 (fused.cuh:26-102): Q pre-scaled by log2(e)/sqrt(d), scores
// in the log2 domain, per-row running max m and sum l, O rescaled by exp2(m_old - m_new) per tile,
// divided by l at the end. The thread mapping is new:
//   * block = 64 query rows x 4 threads ("quad") per row = 256 threads;
//   * each thread keeps d/4 elements of its row's Q and O in registers, columns c = lane4 + 4 i;
//   * K/V tiles of 32 keys are staged in shared memory as fp32 (coalesced loads, one conversion);
//   * a score is a quad-partial dot product reduced with two shuffles, so every thread of the quad
//     holds all 32 scores of its row and the online softmax needs no shared-memory score tile;
//   * K/V reads are conflict-free: a quad reads 4 consecutive floats, the 8 quads of a warp share them.
#include <math_constants.h>

#include "launchers.h"
#include "sm100_ptx.cuh"
#include "../../include/phantom_attn.h"

namespace phantom {
namespace simt {

constexpr int BR = 64;   // query rows per block
constexpr int BC = 32;   // keys per K/V tile
constexpr int THREADS = BR * 4;

template <typename T> __device__ __forceinline__ float to_f(T x);
template <> __device__ __forceinline__ float to_f<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <typename T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

// DMAX: compile-time upper bound of d (multiple of 4); d itself is a runtime value <= DMAX.
template <typename T, int DMAX>
__global__ void __launch_bounds__(THREADS)
attn_fwd_simt(const T* __restrict__ Q, const T* __restrict__ K, const T* __restrict__ V, T* __restrict__ O,
              int N, int d, float scale_log2, int causal) {
  constexpr int PER = DMAX / 4;  // columns per thread
  extern __shared__ float smem_f[];
  float* Ks = smem_f;            // [BC][DMAX]
  float* Vs = Ks + BC * DMAX;    // [BC][DMAX]

  const int tid = threadIdx.x;
  const int r = tid >> 2, q4 = tid & 3;
  const int bh = blockIdx.y;
  const int i0 = blockIdx.x * BR;
  const int row = i0 + r;
  const size_t base = (size_t)bh * N * d;

  float q[PER], o[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int c = q4 + 4 * i;
    q[i] = (row < N && c < d) ? to_f(Q[base + (size_t)row * d + c]) * scale_log2 : 0.f;
    o[i] = 0.f;
  }
  float m = -CUDART_INF_F, l = 0.f;

  const int kv_end = causal ? min(N, i0 + BR) : N;
  for (int j0 = 0; j0 < kv_end; j0 += BC) {
    __syncthreads();  // previous tile consumed
    for (int idx = tid; idx < BC * DMAX; idx += THREADS) {
      const int kk = idx / DMAX, c = idx % DMAX, j = j0 + kk;
      const bool in = j < N && c < d;
      Ks[idx] = in ? to_f(K[base + (size_t)j * d + c]) : 0.f;
      Vs[idx] = in ? to_f(V[base + (size_t)j * d + c]) : 0.f;
    }
    __syncthreads();

    float s[BC];
    float mt = -CUDART_INF_F;
#pragma unroll
    for (int kk = 0; kk < BC; ++kk) {
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < PER; ++i) acc = fmaf(q[i], Ks[kk * DMAX + q4 + 4 * i], acc);
      acc += __shfl_xor_sync(0xffffffffu, acc, 1);
      acc += __shfl_xor_sync(0xffffffffu, acc, 2);
      const int col = j0 + kk;
      if (col >= N || (causal && col > row)) acc = -CUDART_INF_F;
      s[kk] = acc;
      mt = fmaxf(mt, acc);
    }
    const float m_new = fmaxf(m, mt);
    // A row with every key masked so far (never a real row: key 0 is always visible) keeps
    // m = -inf; subtracting 0 instead keeps its p = 0 and alpha = 0 free of inf - inf.
    const float m_sub = m_new == -CUDART_INF_F ? 0.f : m_new;
    const float alpha = ex2(m - m_sub);  // m = -inf on the first tile -> 0
    float ps = 0.f;
#pragma unroll
    for (int kk = 0; kk < BC; ++kk) {
      s[kk] = ex2(s[kk] - m_sub);
      ps += s[kk];
    }
    l = l * alpha + ps;
    m = m_new;
#pragma unroll
    for (int i = 0; i < PER; ++i) o[i] *= alpha;
#pragma unroll
    for (int kk = 0; kk < BC; ++kk) {
#pragma unroll
      for (int i = 0; i < PER; ++i) o[i] = fmaf(s[kk], Vs[kk * DMAX + q4 + 4 * i], o[i]);
    }
  }

  if (row < N) {
    const float inv = 1.f / l;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int c = q4 + 4 * i;
      if (c < d) O[base + (size_t)row * d + c] = from_f<T>(o[i] * inv);
    }
  }
}

template <typename T, int DMAX>
cudaError_t launch_t(const LaunchArgs& a) {
  auto kern = attn_fwd_simt<T, DMAX>;
  const size_t smem = 2 * BC * DMAX * sizeof(float);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  const float scale_log2 = 1.4426950408889634f / sqrtf((float)a.d);
  const dim3 grid((a.N + BR - 1) / BR, a.BH);
  kern<<<grid, THREADS, smem, a.stream>>>(static_cast<const T*>(a.q), static_cast<const T*>(a.k),
                                          static_cast<const T*>(a.v), static_cast<T*>(a.o), a.N, a.d, scale_log2,
                                          a.causal ? 1 : 0);
  note_launch();
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_dtype(const LaunchArgs& a) {
  if (a.d <= 64) return launch_t<T, 64>(a);
  if (a.d <= 128) return launch_t<T, 128>(a);
  return launch_t<T, 256>(a);
}

}  // namespace simt

size_t fused_simt_smem_bytes(int d) {
  const int dmax = d <= 64 ? 64 : d <= 128 ? 128 : 256;
  return 2 * simt::BC * dmax * sizeof(float);
}

cudaError_t launch_fused_simt(const LaunchArgs& a) {
  switch (a.dtype) {
    case PHANTOM_ATTN_F32: return simt::launch_dtype<float>(a);
    case PHANTOM_ATTN_F16: return simt::launch_dtype<__half>(a);
    case PHANTOM_ATTN_BF16: return simt::launch_dtype<__nv_bfloat16>(a);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace phantom
