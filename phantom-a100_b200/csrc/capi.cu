// C ABI of the attention library (declared in include/phantom_attn.h). Validates arguments the way
// the reference's torch glue did (csrc/common.cuh:27-40, attn_fused_tc.cu:5-19,
// attn_fused_tuned.cu:5-21), keeps its error substrings, and dispatches to the sm_100a kernels.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

#include "launchers.h"
#include "../../include/phantom_attn.h"

namespace phantom {
namespace {

thread_local std::string g_last_error;
thread_local long long g_launches = 0;

// Benchmark event brackets: a reusable pool of event pairs per thread.
struct Timing {
  bool enabled = false;
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> pairs;
  size_t used = 0;
  int device = -1;
};
thread_local Timing g_timing;
thread_local LaunchShape g_shape;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(const char* name, cudaError_t e) {
  return fail(PHANTOM_ATTN_ERR_CUDA, "%s: CUDA error: %s", name, cudaGetErrorString(e));
}

constexpr int kMaxDevices = 64;
std::mutex g_mu;
int* g_status[kMaxDevices] = {};   // per-device status word (bounded-wait expiry bits)
int g_cc[kMaxDevices] = {};        // per-device compute capability (major * 10 + minor), 0 = unknown
int g_optin[kMaxDevices] = {};     // per-device opt-in shared memory per block

struct Device {
  int id = 0;
  int cc = 0;
  int optin = 0;
  int* status = nullptr;
};

// Current device, its properties and its 256-byte status region (allocated once per device, zeroed):
// the status word at byte 0.
int current_device(const char* name, Device* out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(name, e);
  if (dev < 0 || dev >= kMaxDevices) return fail(PHANTOM_ATTN_ERR_INVALID, "%s: device %d out of range", name, dev);
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_cc[dev] == 0) {
    int major = 0, minor = 0, optin = 0;
    if ((e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) != cudaSuccess)
      return cuda_fail(name, e);
    g_cc[dev] = major * 10 + minor;
    g_optin[dev] = optin;
  }
  if (g_status[dev] == nullptr) {
    int* p = nullptr;
    if ((e = cudaMalloc(&p, 256)) != cudaSuccess) return cuda_fail(name, e);
    if ((e = cudaMemset(p, 0, 256)) != cudaSuccess) return cuda_fail(name, e);
    g_status[dev] = p;
  }
  out->id = dev;
  out->cc = g_cc[dev];
  out->optin = g_optin[dev];
  out->status = g_status[dev];
  return PHANTOM_ATTN_OK;
}

// Device-pointer check: each of q, k, v, o must be device (or managed) memory of device `dev`.
int check_pointers(const char* name, const void* const* ptrs, int dev) {
  for (int i = 0; i < 4; ++i) {
    if (ptrs[i] == nullptr) return fail(PHANTOM_ATTN_ERR_INVALID, "%s: inputs must be CUDA tensors (null pointer)", name);
    cudaPointerAttributes attr;
    cudaError_t e = cudaPointerGetAttributes(&attr, ptrs[i]);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return fail(PHANTOM_ATTN_ERR_INVALID, "%s: inputs must be CUDA tensors", name);
    }
    if (attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged)
      return fail(PHANTOM_ATTN_ERR_INVALID, "%s: inputs must be CUDA tensors", name);
    if (attr.type == cudaMemoryTypeDevice && attr.device != dev)
      return fail(PHANTOM_ATTN_ERR_INVALID, "%s: q, k, v must be on the same device (current device %d)", name, dev);
  }
  return PHANTOM_ATTN_OK;
}

int check_common(const char* name, const void* q, const void* k, const void* v, void* o, int BH, int N, int d,
                 int dtype, Device* dev) {
  if (BH <= 0 || N <= 0 || d <= 0) return fail(PHANTOM_ATTN_ERR_INVALID, "%s: inputs must be non-empty", name);
  if (dtype != PHANTOM_ATTN_F32 && dtype != PHANTOM_ATTN_F16 && dtype != PHANTOM_ATTN_BF16)
    return fail(PHANTOM_ATTN_ERR_INVALID, "%s: unknown dtype code %d", name, dtype);
  if ((long long)BH > 65535) return fail(PHANTOM_ATTN_ERR_UNSUPPORTED, "%s: batch*heads = %d exceeds 65535", name, BH);
  int rc = current_device(name, dev);
  if (rc != PHANTOM_ATTN_OK) return rc;
  const void* ptrs[4] = {q, k, v, o};
  return check_pointers(name, ptrs, dev->id);
}

int run(const char* name, cudaError_t (*launch)(const LaunchArgs&), const void* q, const void* k, const void* v,
        void* o, int BH, int N, int d, int dtype, int causal, void* stream, const Device& dev) {
  LaunchArgs a{q, k, v, o, BH, N, d, dtype, causal != 0, static_cast<cudaStream_t>(stream), dev.status};
  cudaError_t e = launch(a);
  if (e != cudaSuccess) return cuda_fail(name, e);
  g_last_error.clear();
  return PHANTOM_ATTN_OK;
}

int tc_entry(const char* name, const void* q, const void* k, const void* v, void* o, int BH, int N, int d, int dtype,
             int causal, void* stream) {
  Device dev;
  int rc = check_common(name, q, k, v, o, BH, N, d, dtype, &dev);
  if (rc != PHANTOM_ATTN_OK) return rc;
  if (dtype == PHANTOM_ATTN_F32)
    return fail(PHANTOM_ATTN_ERR_UNSUPPORTED, "%s: float16 or bfloat16 only (tensor cores)", name);
  if (d != 64 && d != 128)
    return fail(PHANTOM_ATTN_ERR_UNSUPPORTED, "%s: only head dimension 64 and 128 are compiled (got %d)", name, d);
  for (const void* p : {q, k, v, static_cast<const void*>(o)})
    if (reinterpret_cast<uintptr_t>(p) % 16 != 0)
      return fail(PHANTOM_ATTN_ERR_INVALID, "%s: inputs must be 16-byte aligned", name);
  if (dev.cc != 100)
    return fail(PHANTOM_ATTN_ERR_UNSUPPORTED,
                "%s: the tcgen05 kernel is compiled for sm_100a (B200); this GPU is sm_%d", name, dev.cc);
  const size_t smem = fused_tc_smem_bytes(d);
  if (smem > (size_t)dev.optin)
    return fail(PHANTOM_ATTN_ERR_UNSUPPORTED, "%s: needs %zu bytes of shared memory, GPU allows %d", name, smem,
                dev.optin);
  return run(name, launch_fused_tc_sm100, q, k, v, o, BH, N, d, dtype, causal, stream, dev);
}

int simt_entry(const char* name, const void* q, const void* k, const void* v, void* o, int BH, int N, int d,
               int dtype, int causal, void* stream) {
  Device dev;
  int rc = check_common(name, q, k, v, o, BH, N, d, dtype, &dev);
  if (rc != PHANTOM_ATTN_OK) return rc;
  if (d > 256)
    return fail(PHANTOM_ATTN_ERR_UNSUPPORTED, "%s: head dimension up to 256 is compiled (got %d)", name, d);
  const size_t smem = fused_simt_smem_bytes(d);
  if (smem > (size_t)dev.optin)
    return fail(PHANTOM_ATTN_ERR_UNSUPPORTED, "%s: needs %zu bytes of shared memory, GPU allows %d", name, smem,
                dev.optin);
  return run(name, launch_fused_simt, q, k, v, o, BH, N, d, dtype, causal, stream, dev);
}

// ------------------------------------------------------------------ entry point without allocation
// Scratch of phantom_attn_fused_tc_noalloc, laid out as [status region (256 B: status word; at byte 128 the
// persistent CTAs' work counters and the call's fp16-overflow word, 16 bytes) | fp16 copy of V | V overflow
// flags]. A file-scope device array: every GPU that loads this library holds these 64 MiB until the process
// exits. All calls on a device share it, the counters included (each call resets them on its stream before
// its attention kernels run).
constexpr size_t kNoAllocScratchBytes = size_t(64) << 20;
constexpr size_t kNoAllocStatusBytes = 256;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
unsigned char* g_noalloc_ptr[kMaxDevices] = {};  // device address of g_noalloc_scratch, per device
int g_noalloc_cc[kMaxDevices] = {};
int g_noalloc_optin[kMaxDevices] = {};

// Per-device set-up, once, with `dev` current: the device address of the static scratch (host code
// only sees a stand-in for the array's name), the compute capability and the shared-memory limit,
// and a zeroed status word. Nothing here allocates.
int noalloc_setup(const char* name, int dev, unsigned char** scratch, int* cc, int* optin) {
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    int major = 0, minor = 0, opt = 0;
    cudaError_t e;
    if ((e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&opt, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) != cudaSuccess)
      return cuda_fail(name, e);
    void* p = nullptr;
    if ((e = cudaGetSymbolAddress(&p, g_noalloc_scratch)) != cudaSuccess) return cuda_fail(name, e);
    if ((e = cudaMemset(p, 0, kNoAllocStatusBytes)) != cudaSuccess) return cuda_fail(name, e);
    g_noalloc_cc[dev] = major * 10 + minor;
    g_noalloc_optin[dev] = opt;
    g_noalloc_ptr[dev] = static_cast<unsigned char*>(p);
  }
  *scratch = g_noalloc_ptr[dev];
  *cc = g_noalloc_cc[dev];
  *optin = g_noalloc_optin[dev];
  return PHANTOM_ATTN_OK;
}

// Reads and clears one status word (the device is already synchronised). Returns the CUDA error.
cudaError_t take_status_word(int* word, int* out) {
  *out = 0;
  if (word == nullptr) return cudaSuccess;
  cudaError_t e = cudaMemcpy(out, word, sizeof(int), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && *out != 0) e = cudaMemset(word, 0, sizeof(int));
  return e;
}

}  // namespace

void note_launch() { ++g_launches; }

const LaunchShape& launch_shape() { return g_shape; }

void timing_begin(cudaStream_t s) {
  Timing& t = g_timing;
  if (!t.enabled) return;
  if (t.used == t.pairs.size()) {
    std::pair<cudaEvent_t, cudaEvent_t> p;
    if (cudaEventCreate(&p.first) != cudaSuccess) return;
    if (cudaEventCreate(&p.second) != cudaSuccess) {
      cudaEventDestroy(p.first);
      return;
    }
    t.pairs.push_back(p);
  }
  cudaEventRecord(t.pairs[t.used].first, s);
}

void timing_end(cudaStream_t s) {
  Timing& t = g_timing;
  if (!t.enabled || t.used >= t.pairs.size()) return;
  cudaEventRecord(t.pairs[t.used].second, s);
  ++t.used;
}

}  // namespace phantom

using namespace phantom;

extern "C" {

int phantom_attn_version(void) { return 10000; }

const char* phantom_attn_last_error(void) { return g_last_error.c_str(); }

int phantom_attn_fused_tc(const void* q, const void* k, const void* v, void* o, int BH, int N, int head_dim,
                          int dtype, int causal, void* stream) {
  return tc_entry("fused_tc", q, k, v, o, BH, N, head_dim, dtype, causal, stream);
}

int phantom_attn_fused_tuned(const void* q, const void* k, const void* v, void* o, int BH, int N, int head_dim,
                             int dtype, int causal, int double_buffer, int br, int bc, void* stream) {
  (void)double_buffer;
  const bool compiled = (br == 64 || br == 128) && (bc == 32 || bc == 64);
  if (!compiled)
    return fail(PHANTOM_ATTN_ERR_UNSUPPORTED,
                "fused_tuned: (br, bc) = (%d, %d) not compiled; available: (64,32) (64,64) (128,32) (128,64)", br, bc);
  return tc_entry("fused_tuned", q, k, v, o, BH, N, head_dim, dtype, causal, stream);
}

int phantom_attn_fused(const void* q, const void* k, const void* v, void* o, int BH, int N, int head_dim, int dtype,
                       int causal, void* stream) {
  return simt_entry("fused", q, k, v, o, BH, N, head_dim, dtype, causal, stream);
}

int phantom_attn_naive(const void* q, const void* k, const void* v, void* o, int BH, int N, int head_dim, int dtype,
                       int causal, void* stream) {
  return simt_entry("naive", q, k, v, o, BH, N, head_dim, dtype, causal, stream);
}

int phantom_attn_tiled(const void* q, const void* k, const void* v, void* o, int BH, int N, int head_dim, int dtype,
                       int causal, void* stream) {
  return simt_entry("tiled", q, k, v, o, BH, N, head_dim, dtype, causal, stream);
}

int phantom_attn_fused_tc_noalloc(const void* q, const void* k, const void* v, void* o, int BH, int N,
                                  int head_dim, int dtype, int causal, void* stream) {
  const char* name = "fused_tc_noalloc";
  if (BH <= 0 || N <= 0 || head_dim <= 0) return fail(PHANTOM_ATTN_ERR_INVALID, "%s: inputs must be non-empty", name);
  if (dtype != PHANTOM_ATTN_F32 && dtype != PHANTOM_ATTN_F16 && dtype != PHANTOM_ATTN_BF16)
    return fail(PHANTOM_ATTN_ERR_INVALID, "%s: unknown dtype code %d", name, dtype);
  if (BH > 65535) return fail(PHANTOM_ATTN_ERR_UNSUPPORTED, "%s: batch*heads = %d exceeds 65535", name, BH);
  if (dtype == PHANTOM_ATTN_F32)
    return fail(PHANTOM_ATTN_ERR_UNSUPPORTED, "%s: float16 or bfloat16 only (tensor cores)", name);
  if (head_dim != 64 && head_dim != 128)
    return fail(PHANTOM_ATTN_ERR_UNSUPPORTED, "%s: only head dimension 64 and 128 are compiled (got %d)", name,
                head_dim);
  for (const void* p : {q, k, v, static_cast<const void*>(o)})
    if (reinterpret_cast<uintptr_t>(p) % 16 != 0)
      return fail(PHANTOM_ATTN_ERR_INVALID, "%s: inputs must be 16-byte aligned", name);
  const size_t need = kNoAllocStatusBytes + fused_tc_scratch_bytes(BH, N, head_dim, dtype);
  if (need > kNoAllocScratchBytes)
    return fail(PHANTOM_ATTN_ERR_UNSUPPORTED,
                "%s: bf16 inputs of B*H*N*d = %lld elements need %zu bytes of scratch; the static scratch holds "
                "%zu bytes (use phantom_attn_fused_tc, which allocates, for larger bf16 inputs)",
                name, (long long)BH * N * head_dim, need, kNoAllocScratchBytes);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(name, e);
  if (dev < 0 || dev >= kMaxDevices) return fail(PHANTOM_ATTN_ERR_INVALID, "%s: device %d out of range", name, dev);
  unsigned char* scratch = nullptr;
  int cc = 0, optin = 0;
  int rc = noalloc_setup(name, dev, &scratch, &cc, &optin);
  if (rc != PHANTOM_ATTN_OK) return rc;
  const void* ptrs[4] = {q, k, v, o};
  if ((rc = check_pointers(name, ptrs, dev)) != PHANTOM_ATTN_OK) return rc;
  if (cc != 100)
    return fail(PHANTOM_ATTN_ERR_UNSUPPORTED,
                "%s: the tcgen05 kernel is compiled for sm_100a (B200); this GPU is sm_%d", name, cc);
  if (fused_tc_smem_bytes(head_dim) > (size_t)optin)
    return fail(PHANTOM_ATTN_ERR_UNSUPPORTED, "%s: needs %zu bytes of shared memory, GPU allows %d", name,
                fused_tc_smem_bytes(head_dim), optin);
  int* status_word = reinterpret_cast<int*>(scratch);
  LaunchArgs a{q, k, v, o, BH, N, head_dim, dtype, causal != 0, static_cast<cudaStream_t>(stream), status_word};
  if ((e = launch_fused_tc_sm100_scratch(a, status_word + 32, scratch + kNoAllocStatusBytes)) != cudaSuccess)
    return cuda_fail(name, e);
  g_last_error.clear();
  return PHANTOM_ATTN_OK;
}

int phantom_attn_device_status(int* status) {
  if (status == nullptr) return fail(PHANTOM_ATTN_ERR_INVALID, "device_status: null output pointer");
  *status = 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail("device_status", e);
  if (dev < 0 || dev >= kMaxDevices) return fail(PHANTOM_ATTN_ERR_INVALID, "device_status: device %d out of range", dev);
  // Neither word is created here: a word that does not exist yet has recorded nothing, and a caller of
  // the allocation-free entry point can read its expiries without this call allocating.
  int* main_word = nullptr;
  int* noalloc_word = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    main_word = g_status[dev];
  }
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    noalloc_word = reinterpret_cast<int*>(g_noalloc_ptr[dev]);
  }
  if ((e = cudaDeviceSynchronize()) != cudaSuccess) return cuda_fail("device_status", e);
  int v_main = 0, v_noalloc = 0;
  if ((e = take_status_word(main_word, &v_main)) != cudaSuccess || (e = take_status_word(noalloc_word, &v_noalloc)) != cudaSuccess)
    return cuda_fail("device_status", e);
  const int v = v_main | (v_noalloc != 0 ? v_noalloc | PHANTOM_ATTN_STATUS_NOALLOC : 0);
  *status = v;
  g_last_error.clear();
  return v == 0 ? PHANTOM_ATTN_OK : fail(PHANTOM_ATTN_ERR_DEVICE, "device status 0x%x: a bounded wait expired", v);
}

int phantom_attn_wait_expiry_probe(void* stream) {
  Device dev;
  int rc = current_device("wait_expiry_probe", &dev);
  if (rc != PHANTOM_ATTN_OK) return rc;
  int* noalloc_word = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    noalloc_word = reinterpret_cast<int*>(g_noalloc_ptr[dev.id]);
  }
  const cudaError_t e = launch_wait_expiry_probe(dev.status, noalloc_word, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail("wait_expiry_probe", e);
  g_last_error.clear();
  return PHANTOM_ATTN_OK;
}

int phantom_attn_kernel_timing(int enable) {
  g_timing.enabled = enable != 0;
  g_timing.used = 0;
  return PHANTOM_ATTN_OK;
}

int phantom_attn_kernel_timing_read(double* total_ms, long long* launches) {
  if (!total_ms || !launches) return fail(PHANTOM_ATTN_ERR_INVALID, "kernel_timing_read: null output pointer");
  double sum = 0.0;
  for (size_t i = 0; i < g_timing.used; ++i) {
    cudaError_t e = cudaEventSynchronize(g_timing.pairs[i].second);
    if (e != cudaSuccess) return cuda_fail("kernel_timing_read", e);
    float ms = 0.f;
    if ((e = cudaEventElapsedTime(&ms, g_timing.pairs[i].first, g_timing.pairs[i].second)) != cudaSuccess)
      return cuda_fail("kernel_timing_read", e);
    sum += ms;
  }
  *total_ms = sum;
  *launches = (long long)g_timing.used;
  return PHANTOM_ATTN_OK;
}

int phantom_attn_set_launch_shape(long long l2_group_kib, int max_ctas) {
  if (l2_group_kib < 0 || l2_group_kib > (1LL << 40) || max_ctas < 0)
    return fail(PHANTOM_ATTN_ERR_INVALID, "set_launch_shape: l2_group_kib must be in [0, 2^40] and max_ctas >= 0 "
                "(got %lld, %d)", l2_group_kib, max_ctas);
  g_shape.l2_group_kib = l2_group_kib;
  g_shape.max_ctas = max_ctas;
  g_last_error.clear();
  return PHANTOM_ATTN_OK;
}

int phantom_attn_get_launch_shape(long long* l2_group_kib, int* max_ctas) {
  if (!l2_group_kib || !max_ctas) return fail(PHANTOM_ATTN_ERR_INVALID, "get_launch_shape: null output pointer");
  *l2_group_kib = g_shape.l2_group_kib;
  *max_ctas = g_shape.max_ctas;
  return PHANTOM_ATTN_OK;
}

int phantom_attn_set_kv_parts(int allow) {
  if (allow != 0 && allow != 1) return fail(PHANTOM_ATTN_ERR_INVALID, "set_kv_parts: allow must be 0 or 1 (got %d)", allow);
  g_shape.kv_parts = allow;
  g_last_error.clear();
  return PHANTOM_ATTN_OK;
}

int phantom_attn_get_kv_parts(void) { return g_shape.kv_parts; }

int phantom_attn_scratch_bytes(long long* high_water, long long* reserved, int reset) {
  if (!high_water || !reserved) return fail(PHANTOM_ATTN_ERR_INVALID, "scratch_bytes: null output pointer");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = scratch_usage(dev, high_water, reserved, reset != 0);
  if (e != cudaSuccess) return cuda_fail("scratch_bytes", e);
  g_last_error.clear();
  return PHANTOM_ATTN_OK;
}

long long phantom_attn_launch_count(int reset) {
  const long long n = g_launches;
  if (reset) g_launches = 0;
  return n;
}

}  // extern "C"
