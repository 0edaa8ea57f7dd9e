#pragma once
// Internal launcher interface between the C ABI (capi.cu) and the kernels. Torch-free.
#include <cuda_runtime.h>

namespace phantom {

struct LaunchArgs {
  const void* q;
  const void* k;
  const void* v;
  void* o;
  int BH;
  int N;
  int d;
  int dtype;   // PHANTOM_ATTN_F32 / F16 / BF16
  bool causal;
  cudaStream_t stream;
  int* status;  // device status word (bounded-wait expiry bits), may be null for kernels without waits
};

// Tensor-core kernel (sm_100a tcgen05). d in {64, 128}, dtype F16/BF16.
cudaError_t launch_fused_tc_sm100(const LaunchArgs& a);
// Dynamic shared memory the tensor-core kernel needs for head dim d.
size_t fused_tc_smem_bytes(int d);
// Tensor-core kernel with caller-supplied scratch (no allocation inside): `work_ctr` is 16 bytes, 8-byte
// aligned: the persistent CTAs' work counters (two ints, zeroed on the call's stream) and, for bf16 inputs, the
// call's fp16-overflow word; calls that overlap on the GPU must not share it. `scratch` is the bf16 V staging
// buffer of fused_tc_scratch_bytes() bytes (0 for fp16 inputs).
cudaError_t launch_fused_tc_sm100_scratch(const LaunchArgs& a, int* work_ctr, void* scratch);
size_t fused_tc_scratch_bytes(int BH, int N, int d, int dtype);

// CUDA-core fp32-arithmetic kernel. Any d in [1, 256], dtype F32/F16/BF16.
cudaError_t launch_fused_simt(const LaunchArgs& a);
// One-warp kernel whose bounded mbarrier wait must expire (nothing arrives on the barrier); sets bit 16
// of *status, and of *status2 when that is not null (attn_tc_sm100.cu).
cudaError_t launch_wait_expiry_probe(int* status, int* status2, cudaStream_t stream);
size_t fused_simt_smem_bytes(int d);

// High-water mark of the scratch taken from device `dev`'s memory pool since the last reset, and the bytes
// the pool holds now (both 0 before any call needed scratch); reset = true restarts the high-water mark.
cudaError_t scratch_usage(int dev, long long* high_water, long long* reserved, bool reset);

// Number of kernel launches the library has made on this thread (benchmark accounting).
void note_launch();

// Benchmark event brackets around the main attention kernel (no-ops unless enabled on this thread).
void timing_begin(cudaStream_t s);
void timing_end(cudaStream_t s);

// Launch-shape override of the tensor-core kernel for the calling thread (0 = automatic): K/V bytes per
// L2 head group in KiB, a cap on the persistent grid, and whether a last partial wave may be cut into
// K/V parts (1, the default) or not (0: every query block then runs over its whole K/V range, so results
// are bit-identical for every launch shape).
struct LaunchShape {
  long long l2_group_kib = 0;
  int max_ctas = 0;
  int kv_parts = 1;
};
const LaunchShape& launch_shape();

}  // namespace phantom
