// Common device helpers: types, warp reductions, launch checks, error flags.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <map>
#include <mutex>
#include <utility>

#define CB_DEVICE __device__ __forceinline__
#define CB_HOST_DEVICE __host__ __device__ __forceinline__

#define CB_CUDA_CHECK(expr)                                                                     \
  do {                                                                                          \
    cudaError_t _e = (expr);                                                                    \
    if (_e != cudaSuccess) {                                                                    \
      fprintf(stderr, "CUDA error %s at %s:%d: %s\n", #expr, __FILE__, __LINE__,                \
              cudaGetErrorString(_e));                                                          \
      return _e;                                                                                \
    }                                                                                           \
  } while (0)

namespace cb {

constexpr float kFp8Max = 448.0f;

// Error codes written to a device-side status word by kernels whose waits are bounded.
enum : int {
  kOk = 0,
  kErrTimeoutFull = 1,     // producer data never arrived
  kErrTimeoutEmpty = 2,    // consumer never released a stage
  kErrTimeoutTmem = 3,     // accumulator hand-off never happened
  kErrTimeoutPeer = 4,     // a peer rank's flag never arrived
  kErrBadArg = 5,
};

// Bounds-checked debug builds (compute-sanitizer is not available everywhere): building with
// CARBON_DEBUG_BOUNDS=1 defines CB_DEBUG_BOUNDS.  Index-driven kernels pass every row index they compute through
// cb_check_index() and skip the access when it fails; a debug build also prints the first failure of each
// translation unit (kernel site, index, limit, block, thread), so a wrong index shows up as one stderr line instead
// of a fault.  Release builds keep only the range test.
#ifdef CB_DEBUG_BOUNDS
static __device__ int cb_bounds_reported = 0;
__device__ __forceinline__ bool cb_check_index(long long idx, long long limit, const char* site) {
  if (idx >= 0 && idx < limit) return true;
  if (atomicCAS(&cb_bounds_reported, 0, 1) == 0)
    printf("[carbon bounds] %s: index %lld outside [0, %lld) (block %d thread %d)\n", site, idx, limit,
           int(blockIdx.x), int(threadIdx.x));
  return false;
}
#else
__device__ __forceinline__ bool cb_check_index(long long idx, long long limit, const char*) {
  return idx >= 0 && idx < limit;
}
#endif

CB_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
// Warp totals of NV per-lane values with NV/2 + NV/4 + ... + 1 (+ the remaining plain steps) shuffles instead of
// 5 NV: at each butterfly step a lane keeps one half of its values, receives its partner's partial of that half and
// sends the other.  Afterwards lane l holds the total of value  l >> (5 - log2 NV)  (NV = 8, 16 or 32).
template <int NV>
CB_DEVICE float warp_sum_many(float (&v)[NV], int lane) {
  static_assert(NV == 8 || NV == 16 || NV == 32, "warp_sum_many: NV in {8, 16, 32}");
  int n = NV;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    if (n > 1) {
      const int half = n >> 1;
      const bool up = (lane & off) != 0;
#pragma unroll
      for (int i = 0; i < NV / 2; ++i)
        if (i < half) {
          const float send = up ? v[i] : v[i + half];
          const float keep = up ? v[i + half] : v[i];
          v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
      n = half;
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], off);
    }
  }
  return v[0];
}
CB_DEVICE float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block reduction for blockDim.x a multiple of 32 and <= 1024. `smem` holds >= 32 floats.
CB_DEVICE float block_sum(float v, float* smem) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) smem[wid] = v;
  __syncthreads();
  float r = lane < nw ? smem[lane] : 0.f;
  r = warp_sum(r);
  return r;
}
CB_DEVICE float block_max(float v, float* smem) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) smem[wid] = v;
  __syncthreads();
  float r = lane < nw ? smem[lane] : -INFINITY;
  r = warp_max(r);
  return r;
}

// Power-of-two scale for an fp8 e4m3 block: smallest 2^e with amax / 2^e <= 448. Returns the biased UE8M0 byte
// (e + 127). Computed exactly from the fp32 exponent bits; no transcendental functions are involved.
CB_DEVICE uint32_t ue8m0_for_amax(float amax) {
  if (!(amax > 0.f)) return 127u;  // scale 1.0 for all-zero blocks
  float r = amax / kFp8Max;        // want smallest e with 2^e >= r
  uint32_t bits = __float_as_uint(r);
  int e = int((bits >> 23) & 0xff) - 127;
  if (bits & 0x7fffff) e += 1;     // not an exact power of two: round the exponent up
  int biased = e + 127;
  biased = biased < 1 ? 1 : (biased > 254 ? 254 : biased);
  return uint32_t(biased);
}
CB_DEVICE float ue8m0_to_float(uint32_t b) { return __uint_as_float(b << 23); }
// 1 / scale, exact for powers of two.
CB_DEVICE float ue8m0_inv(uint32_t b) { return __uint_as_float((254u - b) << 23); }

CB_DEVICE __nv_bfloat162 f2_to_bf2(float a, float b) { return __floats2bfloat162_rn(a, b); }

CB_DEVICE uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Pack 4 floats (already scaled into e4m3 range) into 4 fp8 e4m3 bytes (satfinite, round-to-nearest-even).
CB_DEVICE uint32_t pack_fp8x4(float a, float b, float c, float d) {
  __nv_fp8x2_e4m3 lo(make_float2(a, b));
  __nv_fp8x2_e4m3 hi(make_float2(c, d));
  return uint32_t(*reinterpret_cast<uint16_t*>(&lo)) | (uint32_t(*reinterpret_cast<uint16_t*>(&hi)) << 16);
}

CB_DEVICE float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
CB_DEVICE float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

// Raise a kernel's dynamic shared-memory limit to `bytes` on the CURRENT device.  cudaFuncSetAttribute acts on
// the current device's context only, so the opt-in is tracked per (device, kernel); the table is shared by every
// translation unit (inline function) and guarded by a mutex, so host threads driving different GPUs may call it.
inline cudaError_t smem_optin(const void* fn, int bytes) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  static std::mutex mu;
  static std::map<std::pair<int, const void*>, int> done;
  std::lock_guard<std::mutex> g(mu);
  int& have = done[std::make_pair(dev, fn)];
  if (have >= bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) have = bytes;
  return e;
}
template <typename F>
inline cudaError_t smem_optin(F* fn, int bytes) {
  return smem_optin(reinterpret_cast<const void*>(fn), bytes);
}

// End of a kernel that stored into peer GPUs' memory: one system-scope fence per CTA instead of one per thread.
// The block barrier orders every thread's stores before thread 0's fence (fences are cumulative over what the
// fencing thread has observed), and the kernel's completion orders that fence before the next kernel's barrier
// release that lets the peers read.  Every thread of the block must call it (it contains __syncthreads).
CB_DEVICE void publish_peer_stores() {
  __syncthreads();
  if (threadIdx.x == 0) __threadfence_system();
}

// Programmatic dependent launch.  Every kernel of this library starts with pdl_entry(): it waits until the kernel
// launched before it in the stream has completed and its memory is visible (a no-op when this launch carries no
// programmatic dependency), then lets the next kernel of the stream be launched early, so that its launch and
// prologue overlap this kernel's work.  Waiting first keeps the dependency transitive: a kernel can never finish
// before its predecessor has.
CB_DEVICE void pdl_entry() {
#if defined(__CUDA_ARCH__) && __CUDA_ARCH__ >= 900
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
#endif
}

// The two halves of pdl_entry(), for kernels that start work which does not depend on the previous kernel (weight
// loads) before waiting: every thread that reads the previous kernel's output must have executed pdl_wait() first.
CB_DEVICE void pdl_wait() {
#if defined(__CUDA_ARCH__) && __CUDA_ARCH__ >= 900
  asm volatile("griddepcontrol.wait;" ::: "memory");
#endif
}
CB_DEVICE void pdl_launch_dependents() {
#if defined(__CUDA_ARCH__) && __CUDA_ARCH__ >= 900
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
#endif
}

// Whether launches carry the programmatic-serialization attribute (CARBON_PDL=0 turns it off).
inline bool pdl_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("CARBON_PDL");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

#ifdef __CUDACC__
// Kernel launch with programmatic stream serialization (see pdl_entry); returns the launch's error code.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                            Args&&... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}
#endif

CB_HOST_DEVICE int ceil_div(int a, int b) { return (a + b - 1) / b; }
CB_HOST_DEVICE int64_t ceil_div64(int64_t a, int64_t b) { return (a + b - 1) / b; }

}  // namespace cb
