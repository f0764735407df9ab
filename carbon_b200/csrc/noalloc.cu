// Allocation-free variant of the absorbed-MLA sparse decode attention entry point (see noalloc.h).
// No counterpart in the reference.
#include <stdio.h>
#include <mutex>
#include "noalloc.h"
#include "small_ops.h"

namespace {

constexpr size_t kScratchBytes = size_t(32) << 20;          // 32 MiB per device, held until process exit
constexpr size_t kScratchFloats = kScratchBytes / sizeof(float);
constexpr int kMaxDevices = 64;

// Split-K partials (O then (m, l)) of the decode kernel. Host code must not pass this name to a kernel: on the host
// it is only a stand-in; the device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) float g_mla_scratch[kScratchFloats];

float* g_scratch_dev[kMaxDevices] = {};
int g_sm_count[kMaxDevices] = {};
std::mutex g_setup_mu;
thread_local char g_err[512] = "";

int fail(int code, const char* msg) {
  snprintf(g_err, sizeof(g_err), "%s", msg);
  return code;
}

// Same split rule as the allocating entry point (carbon_b200/ops/attention.py: mla_splits).
int splits_for(int T, int K, int sms) {
  int s = sms / (2 * (T > 0 ? T : 1));
  if (s < 1) s = 1;
  const int cap = (K + 127) / 128;
  if (s > cap) s = cap;
  return s < 1 ? 1 : s;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) size_t cb_noalloc_scratch_bytes(void) { return kScratchBytes; }

extern "C" __attribute__((visibility("default"))) const char* cb_noalloc_last_error(void) { return g_err; }

extern "C" __attribute__((visibility("default"))) int cb_sparse_mla_noalloc(const void* q, int T, int H,
                                                                              const void* kv, int S, const int* idx,
                                                                              int K, float scale, void* out,
                                                                              cudaStream_t stream) {
  g_err[0] = '\0';
  if (T < 0 || H <= 0 || H > 128 || S <= 0 || K < 0 || !q || !kv || !idx || !out)
    return fail(cudaErrorInvalidValue, "cb_sparse_mla_noalloc: bad arguments (need H in 1..128, non-null pointers)");
  if (T == 0) return cudaSuccess;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(e, "cb_sparse_mla_noalloc: cudaGetDevice failed");
  if (dev < 0 || dev >= kMaxDevices) return fail(cudaErrorInvalidDevice, "cb_sparse_mla_noalloc: device id too large");
  if (!g_scratch_dev[dev]) {
    std::lock_guard<std::mutex> g(g_setup_mu);
    if (!g_scratch_dev[dev]) {
      int sms = 0;
      e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      if (e != cudaSuccess) return fail(e, "cb_sparse_mla_noalloc: cannot query the SM count");
      float* ptr = nullptr;
      e = cudaGetSymbolAddress(reinterpret_cast<void**>(&ptr), g_mla_scratch);
      if (e != cudaSuccess || !ptr) return fail(e != cudaSuccess ? e : cudaErrorInvalidSymbol,
                                                "cb_sparse_mla_noalloc: cudaGetSymbolAddress of the scratch failed");
      g_sm_count[dev] = sms;
      g_scratch_dev[dev] = ptr;
    }
  }
  const int splits = splits_for(T, K, g_sm_count[dev]);
  if (splits > 1) {
    const size_t need = size_t(T) * splits * H * 514;
    if (need > kScratchFloats) {
      snprintf(g_err, sizeof(g_err),
               "cb_sparse_mla_noalloc: T=%d x splits=%d x H=%d needs %zu bytes of scratch, above the %zu-byte "
               "static array; use the allocating entry point or a smaller batch",
               T, splits, H, need * sizeof(float), kScratchBytes);
      return cudaErrorInvalidValue;
    }
  }
  float* part_o = g_scratch_dev[dev];
  float* part_ml = part_o + size_t(T) * splits * H * 512;
  e = cb::sparse_mla(q, T, H, kv, S, idx, K, scale, splits, splits > 1 ? part_o : nullptr,
                     splits > 1 ? part_ml : nullptr, out, nullptr, stream);
  if (e != cudaSuccess) return fail(e, "cb_sparse_mla_noalloc: kernel launch failed");
  return cudaSuccess;
}
