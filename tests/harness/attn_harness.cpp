// Torch-free driver of the C ABI (include/phantom_attn.h): the role of b4batunde/Phantom-A100's
// sim/harness.cu for this library. Seeded inputs, one call, a float64 CPU check (oracle/ref64.c), one
// machine-readable RESULT line; with HARNESS_ITERS=<n>, n CUDA-event-timed launches and a TIME line.
//
//   attn_harness <kernel> <BH> <N> [d=64] [dtype=f16|bf16|f32] [causal=0] [seed=1]
//   kernel: fused_tc | fused_tc_noalloc | fused_tuned:<br>:<bc>:<db> | fused | naive | tiled
//
//   RESULT kernel=... BH=... N=... d=... dtype=... causal=... max_abs_err=... rel_l2=... status=PASS|FAIL
//   TIME kernel=... BH=... N=... d=... median_ms=... min_ms=... tflops=...
//
// Pass criteria: fp32 max |err| <= 1e-4; fp16/bf16 relative L2 <= 1e-3 and max |err| <= 2e-3 beyond one
// output ulp, both against the float64 result rounded to the output dtype.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <string>
#include <vector>

#include "phantom_attn.h"
#include "ref64.h"

#define CK(x)                                                                                   \
  do {                                                                                          \
    cudaError_t e_ = (x);                                                                       \
    if (e_ != cudaSuccess) {                                                                    \
      std::printf("RESULT status=CUDA_ERROR where=%s err=%s\n", #x, cudaGetErrorString(e_));    \
      return 2;                                                                                 \
    }                                                                                           \
  } while (0)

namespace {

// Round a float to the storage dtype and back; `bits` receives the 16- or 32-bit pattern.
float round_to(float x, int dtype, uint32_t* bits) {
  if (dtype == PHANTOM_ATTN_F16) {
    __half h = __float2half_rn(x);
    uint16_t b;
    std::memcpy(&b, &h, 2);
    *bits = b;
    return __half2float(h);
  }
  if (dtype == PHANTOM_ATTN_BF16) {
    __nv_bfloat16 h = __float2bfloat16_rn(x);
    uint16_t b;
    std::memcpy(&b, &h, 2);
    *bits = b;
    return __bfloat162float(h);
  }
  std::memcpy(bits, &x, 4);
  return x;
}

float from_bits(uint32_t b, int dtype) {
  if (dtype == PHANTOM_ATTN_F16) {
    uint16_t s = (uint16_t)b;
    __half h;
    std::memcpy(&h, &s, 2);
    return __half2float(h);
  }
  if (dtype == PHANTOM_ATTN_BF16) {
    uint16_t s = (uint16_t)b;
    __nv_bfloat16 h;
    std::memcpy(&h, &s, 2);
    return __bfloat162float(h);
  }
  float f;
  std::memcpy(&f, &b, 4);
  return f;
}

double ulp16(double x, int dtype) {
  const int mant = dtype == PHANTOM_ATTN_F16 ? 10 : 7;
  const double ax = std::max(std::fabs(x), std::ldexp(1.0, -14));
  return std::ldexp(1.0, (int)std::floor(std::log2(ax)) - mant);
}

}  // namespace

int main(int argc, char** argv) {
  if (argc < 4) {
    std::fprintf(stderr, "usage: %s <kernel> <BH> <N> [d=64] [dtype=f16|bf16|f32] [causal=0] [seed=1]\n", argv[0]);
    return 1;
  }
  const std::string name = argv[1];
  const int BH = std::atoi(argv[2]), N = std::atoi(argv[3]);
  const int d = argc > 4 ? std::atoi(argv[4]) : 64;
  const std::string dts = argc > 5 ? argv[5] : "f16";
  const int causal = argc > 6 ? std::atoi(argv[6]) : 0;
  const unsigned seed = argc > 7 ? (unsigned)std::atoi(argv[7]) : 1u;
  const int dtype = dts == "f32" ? PHANTOM_ATTN_F32 : dts == "bf16" ? PHANTOM_ATTN_BF16 : PHANTOM_ATTN_F16;
  const size_t esz = dtype == PHANTOM_ATTN_F32 ? 4 : 2;
  const size_t n = (size_t)BH * N * d;

  // Inputs: mt19937 N(0,1) rounded to the dtype (the reference harness's generator, harness.cu:78-86).
  std::mt19937 rng(seed);
  std::normal_distribution<float> dist(0.f, 1.f);
  std::vector<float> fq(n), fk(n), fv(n);
  std::vector<unsigned char> hq(n * esz), hk(n * esz), hv(n * esz), ho(n * esz);
  for (size_t i = 0; i < n; ++i) {
    uint32_t b;
    fq[i] = round_to(dist(rng), dtype, &b);
    std::memcpy(&hq[i * esz], &b, esz);
    fk[i] = round_to(dist(rng), dtype, &b);
    std::memcpy(&hk[i * esz], &b, esz);
    fv[i] = round_to(dist(rng), dtype, &b);
    std::memcpy(&hv[i * esz], &b, esz);
  }

  void *q, *k, *v, *o;
  CK(cudaMalloc(&q, n * esz));
  CK(cudaMalloc(&k, n * esz));
  CK(cudaMalloc(&v, n * esz));
  CK(cudaMalloc(&o, n * esz));
  CK(cudaMemcpy(q, hq.data(), n * esz, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(k, hk.data(), n * esz, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(v, hv.data(), n * esz, cudaMemcpyHostToDevice));
  CK(cudaMemset(o, 0xFF, n * esz));  // NaN canary: every element must be written

  auto launch = [&]() -> int {
    if (name == "fused_tc") return phantom_attn_fused_tc(q, k, v, o, BH, N, d, dtype, causal, nullptr);
    if (name == "fused_tc_noalloc") return phantom_attn_fused_tc_noalloc(q, k, v, o, BH, N, d, dtype, causal, nullptr);
    if (name == "fused") return phantom_attn_fused(q, k, v, o, BH, N, d, dtype, causal, nullptr);
    if (name == "naive") return phantom_attn_naive(q, k, v, o, BH, N, d, dtype, causal, nullptr);
    if (name == "tiled") return phantom_attn_tiled(q, k, v, o, BH, N, d, dtype, causal, nullptr);
    if (name.rfind("fused_tuned:", 0) == 0) {
      int br = 64, bc = 32, db = 1;
      std::sscanf(name.c_str(), "fused_tuned:%d:%d:%d", &br, &bc, &db);
      return phantom_attn_fused_tuned(q, k, v, o, BH, N, d, dtype, causal, db, br, bc, nullptr);
    }
    std::fprintf(stderr, "unknown kernel %s\n", name.c_str());
    return -1;
  };

  const int rc = launch();
  if (rc != PHANTOM_ATTN_OK) {
    std::printf("RESULT kernel=%s status=API_ERROR code=%d msg=\"%s\"\n", name.c_str(), rc, phantom_attn_last_error());
    return 3;
  }
  CK(cudaDeviceSynchronize());
  int status = 0;
  phantom_attn_device_status(&status);
  CK(cudaMemcpy(ho.data(), o, n * esz, cudaMemcpyDeviceToHost));

  std::vector<double> ref(n);
  phantom_ref64_attention(fq.data(), fk.data(), fv.data(), ref.data(), BH, N, d, causal);
  double max_abs = 0, max_excess = -1e30, num = 0, den = 0;
  bool finite = true;
  for (size_t i = 0; i < n; ++i) {
    uint32_t b = 0;
    std::memcpy(&b, &ho[i * esz], esz);
    const double out = from_bits(b, dtype);
    if (!std::isfinite(out)) finite = false;
    uint32_t rb;
    const double r = dtype == PHANTOM_ATTN_F32 ? ref[i] : (double)round_to((float)ref[i], dtype, &rb);
    const double e = std::fabs(out - r);
    max_abs = std::max(max_abs, e);
    if (dtype != PHANTOM_ATTN_F32) max_excess = std::max(max_excess, e - ulp16(r, dtype));
    num += (out - r) * (out - r);
    den += r * r;
  }
  const double rel = den > 0 ? std::sqrt(num / den) : std::sqrt(num);
  const bool pass = finite && status == 0 &&
                    (dtype == PHANTOM_ATTN_F32 ? max_abs <= 1e-4 : (rel <= 1e-3 && max_excess <= 2e-3));
  std::printf("RESULT kernel=%s BH=%d N=%d d=%d dtype=%s causal=%d max_abs_err=%.3e rel_l2=%.3e status=%s\n",
              name.c_str(), BH, N, d, dts.c_str(), causal, max_abs, rel, pass ? "PASS" : "FAIL");

  const char* iters_env = std::getenv("HARNESS_ITERS");
  const int iters = iters_env ? std::atoi(iters_env) : 0;
  if (iters > 0 && pass) {
    for (int w = 0; w < 5; ++w) launch();
    CK(cudaDeviceSynchronize());
    cudaEvent_t e0, e1;
    CK(cudaEventCreate(&e0));
    CK(cudaEventCreate(&e1));
    std::vector<float> ms(iters);
    for (int it = 0; it < iters; ++it) {
      CK(cudaEventRecord(e0));
      launch();
      CK(cudaEventRecord(e1));
      CK(cudaEventSynchronize(e1));
      CK(cudaEventElapsedTime(&ms[it], e0, e1));
    }
    std::sort(ms.begin(), ms.end());
    const double flops = 4.0 * BH * (double)N * N * d * (causal ? 0.5 : 1.0);
    std::printf("TIME kernel=%s BH=%d N=%d d=%d causal=%d median_ms=%.5f min_ms=%.5f tflops=%.1f iters=%d\n",
                name.c_str(), BH, N, d, causal, ms[iters / 2], ms[0], flops / (ms[iters / 2] * 1e-3) / 1e12, iters);
  }
  cudaFree(q);
  cudaFree(k);
  cudaFree(v);
  cudaFree(o);
  return pass ? 0 : 4;
}
