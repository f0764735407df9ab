// Allocation-free variant of the absorbed-MLA sparse decode attention entry point (see noalloc.h).
// No counterpart in the reference.
#include <stdio.h>
#include <mutex>
#include "noalloc.h"
#include "small_ops.h"

namespace {

constexpr size_t kScratchBytes = size_t(32) << 20;          // 32 MiB per device, held until process exit
constexpr size_t kStatusFloats = 64;                        // first 256 bytes: the kernel's status word
constexpr size_t kScratchFloats = kScratchBytes / sizeof(float) - kStatusFloats;
constexpr int kMaxDevices = 64;

// [status word, padding to 256 bytes][split-K partials: O, then (m, l)].  Host code must not pass this name to a
// kernel: on the host it is only a stand-in; the device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) float g_mla_scratch[kStatusFloats + kScratchFloats];

struct DeviceSetup {
  std::once_flag once;
  cudaError_t err = cudaSuccess;
  float* scratch = nullptr;      // device address of g_mla_scratch on this device
  int sms = 0;
};
DeviceSetup g_setup[kMaxDevices];
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

// Resolves this device's scratch address once (std::call_once: concurrent first calls from several host threads
// wait for the one that runs it, and every later reader sees its writes).  Must run with `dev` current.
DeviceSetup* setup_device(int dev) {
  DeviceSetup* d = &g_setup[dev];
  std::call_once(d->once, [d, dev] {
    int sms = 0;
    cudaError_t e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    float* ptr = nullptr;
    if (e == cudaSuccess) e = cudaGetSymbolAddress(reinterpret_cast<void**>(&ptr), g_mla_scratch);
    if (e == cudaSuccess && !ptr) e = cudaErrorInvalidSymbol;
    d->err = e;
    d->sms = sms;
    d->scratch = e == cudaSuccess ? ptr : nullptr;
  });
  return d;
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
  DeviceSetup* d = setup_device(dev);
  if (d->err != cudaSuccess)
    return fail(d->err, "cb_sparse_mla_noalloc: resolving the scratch array's device address failed");
  const int splits = splits_for(T, K, d->sms);
  if (splits > 1) {
    const size_t need = size_t(T) * splits * H * 514;
    if (need > kScratchFloats) {
      snprintf(g_err, sizeof(g_err),
               "cb_sparse_mla_noalloc: T=%d x splits=%d x H=%d needs %zu bytes of scratch, above the %zu bytes "
               "left after the status word; use the allocating entry point or a smaller batch",
               T, splits, H, need * sizeof(float), kScratchFloats * sizeof(float));
      return cudaErrorInvalidValue;
    }
  }
  int* status = reinterpret_cast<int*>(d->scratch);
  float* part_o = d->scratch + kStatusFloats;
  float* part_ml = part_o + size_t(T) * splits * H * 512;
  e = cudaMemsetAsync(status, 0, sizeof(int), stream);      // the status word starts at "no error" every call
  if (e != cudaSuccess) return fail(e, "cb_sparse_mla_noalloc: clearing the status word failed");
  e = cb::sparse_mla(q, T, H, kv, S, idx, K, scale, splits, splits > 1 ? part_o : nullptr,
                     splits > 1 ? part_ml : nullptr, out, status, stream);
  if (e != cudaSuccess) return fail(e, "cb_sparse_mla_noalloc: kernel launch failed");
  return cudaSuccess;
}

extern "C" __attribute__((visibility("default"))) int cb_noalloc_status(cudaStream_t stream, int* kernel_status) {
  g_err[0] = '\0';
  if (!kernel_status) return fail(cudaErrorInvalidValue, "cb_noalloc_status: null output pointer");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(e, "cb_noalloc_status: cudaGetDevice failed");
  if (dev < 0 || dev >= kMaxDevices) return fail(cudaErrorInvalidDevice, "cb_noalloc_status: device id too large");
  DeviceSetup* d = setup_device(dev);
  if (d->err != cudaSuccess) return fail(d->err, "cb_noalloc_status: resolving the scratch address failed");
  e = cudaMemcpyAsync(kernel_status, d->scratch, sizeof(int), cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return fail(e, "cb_noalloc_status: reading the status word failed");
  return cudaSuccess;
}
