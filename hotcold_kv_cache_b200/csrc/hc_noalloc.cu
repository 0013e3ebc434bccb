// Stand-alone decode attention that allocates nothing.
//
// Some callers cannot allocate device memory: a host runtime that binds this library over
// FFI and hands it only its input and output buffers, or a serving process whose device
// memory is fully reserved by its own pool after start-up. hc_attention_dense needs a
// caller-provided scratch area and counter array; this variant keeps both in static device
// arrays of this library instead. Every GPU that loads the library holds them until exit.
//
// Limits: the split-K partials (plus the evict_idx buffers) must fit kNoAllocScratchBytes
// (8 MiB) and B*Hk must not exceed kNoAllocCounters (4096); larger calls are rejected with
// HC_ERR_UNSUPPORTED. All calls share the arrays: calls that overlap on the GPU (two streams,
// two host threads) race and must not be issued concurrently. The arrays keep the last call's
// contents; the counters, which must start at zero, are cleared by every call.
//
// Set-up: every call resolves the arrays' device addresses on the current device with
// cudaGetSymbolAddress (cheap, and never stale: a device reset reloads the module and may move
// them). Under CUDA's lazy module loading (the 12.x default) the arrays are committed on a device
// when the first call there loads the module, so make that first call before the caller's own
// pool reserves the device's memory, and before any stream capture; or run the process with
// CUDA_MODULE_LOADING=EAGER, which commits them when the library is loaded.

#include <cstdio>

#include "hc_internal.cuh"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;
constexpr int kNoAllocCounters = 4096;

// In host code these names are host-side stand-ins, not device addresses: the address a
// kernel may use comes from cudaGetSymbolAddress, per device.
static __device__ __align__(256) unsigned char g_scratch[kNoAllocScratchBytes];
static __device__ __align__(256) int32_t g_counters[kNoAllocCounters];

struct DevicePtrs {
  void* scratch = nullptr;
  int32_t* counters = nullptr;
};

// The arrays' device addresses on the current device, resolved on every call.
cudaError_t device_ptrs(DevicePtrs& out) {
  void* s = nullptr;
  void* c = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&s, g_scratch);
  if (e != cudaSuccess) return e;
  e = cudaGetSymbolAddress(&c, g_counters);
  if (e != cudaSuccess) return e;
  out.scratch = s;
  out.counters = static_cast<int32_t*>(c);
  return cudaSuccess;
}

}  // namespace

extern "C" {

int hc_attention_dense_noalloc(const void* q, const void* k, const void* v, const uint8_t* mask, void* out,
                               int64_t* evict_idx, int B, int Hq, int Hk, int S, int D, int dtype, float scale,
                               int overflow_nan, void* stream) {
  char msg[256];
  if (B <= 0 || Hk <= 0 || Hq <= 0 || S <= 0) {
    hc::set_last_error("empty or negative shape");
    return HC_ERR_ARG;
  }
  const size_t need = hc_attention_dense_scratch_bytes(B, Hq, Hk, S, D);
  if (need > kNoAllocScratchBytes) {
    snprintf(msg, sizeof(msg), "needs %zu scratch bytes; the static area holds %zu", need, kNoAllocScratchBytes);
    hc::set_last_error(msg);
    return HC_ERR_UNSUPPORTED;
  }
  if ((long)B * Hk > kNoAllocCounters) {
    hc::set_last_error("B*Hk above the 4096 static counters");
    return HC_ERR_UNSUPPORTED;
  }
  DevicePtrs p;
  cudaError_t e = device_ptrs(p);
  if (e == cudaSuccess)
    e = cudaMemsetAsync(p.counters, 0, sizeof(int32_t) * (size_t)B * Hk, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    snprintf(msg, sizeof(msg), "static scratch set-up: %s", cudaGetErrorString(e));
    hc::set_last_error(msg);
    return HC_ERR_CUDA;
  }
  return hc_attention_dense(q, k, v, mask, out, evict_idx, B, Hq, Hk, S, D, dtype, scale, overflow_nan,
                            p.counters, p.scratch, kNoAllocScratchBytes, stream);
}

}  // extern "C"
