// Engram (hashed n-gram memory) kernels, sm_100a.
//
// engram_gather: out[t, c*dim : (c+1)*dim] = dequant(table row ids[t, c]).  The table holds fp8 e4m3 rows with one
//   UE8M0 scale byte (biased exponent) per 32 elements.  It may be split over ranks by row ranges (whole hash
//   columns per rank, in the symmetric heap): row r lives on the rank whose [bounds[k], bounds[k+1]) contains it and
//   is read straight from that rank's HBM over NVLink (plain loads; peer pointers).  One warp per (token, column);
//   each lane moves 8 elements (8 bytes) per step.
//   Reference: the Engram peer lookup, one CTA per row reading the owner's shard (dspd_w22/dspd/engram.py:165-170,
//   king_v10/bundle_v9/dec/peer_lookup.py:270).
//
// engram_gate: X[t, s, :] += sigmoid(clamp(<rms(X_s) * q_w, rms(k_s) * k_w> / sqrt(D), +-clamp)) * v for every mHC
//   stream s, with kv[t] = [k_0 .. k_{hc-1} | v]; writes the new sum of squares of X[t] (the mHC statistics input).
//   Tokens whose id is the image token (optional) are left unchanged.  One CTA per token.
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cstdint>
#include "common.cuh"

namespace cb {

__global__ void engram_gather_kernel(const int* __restrict__ ids, int T, int C, int dim,
                                     const uint64_t* __restrict__ data_ptrs, const uint64_t* __restrict__ sf_ptrs,
                                     const int* __restrict__ bounds, int world, __nv_bfloat16* __restrict__ out) {
  cb::pdl_entry();
  const int warps = blockDim.x >> 5;
  const int item = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (item >= T * C) return;
  const int t = item / C, c = item - t * C;
  const int id = ids[item];
  __nv_bfloat16* o = out + (size_t(t) * C + c) * dim;
  if (!cb_check_index(id, bounds[world], "engram_gather")) {       // bad row id: a zero row, no access
    for (int e0 = lane * 8; e0 < dim; e0 += 256) *reinterpret_cast<uint4*>(o + e0) = make_uint4(0, 0, 0, 0);
    return;
  }
  int r = 0;
  while (r + 1 < world && id >= bounds[r + 1]) ++r;
  const int local = id - bounds[r];
  const uint8_t* row = reinterpret_cast<const uint8_t*>(data_ptrs[r]) + size_t(local) * dim;
  const uint8_t* sf = reinterpret_cast<const uint8_t*>(sf_ptrs[r]) + size_t(local) * (dim / 32);
  for (int e0 = lane * 8; e0 < dim; e0 += 256) {
    const uint2 raw = *reinterpret_cast<const uint2*>(row + e0);
    const float scale = __uint_as_float(uint32_t(sf[e0 / 32]) << 23);        // 2^(sf - 127)
    const uint32_t w[2] = {raw.x, raw.y};
    uint32_t packed[4];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
#pragma unroll
      for (int b = 0; b < 4; b += 2) {
        __nv_fp8_e4m3 f0, f1;
        f0.__x = uint8_t(w[h] >> (8 * b));
        f1.__x = uint8_t(w[h] >> (8 * (b + 1)));
        packed[2 * h + b / 2] = pack_bf16x2(float(f0) * scale, float(f1) * scale);
      }
    }
    *reinterpret_cast<uint4*>(o + e0) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
  }
}

cudaError_t engram_gather(const int* ids, int T, int C, int dim, const uint64_t* data_ptrs, const uint64_t* sf_ptrs,
                          const int* bounds, int world, void* out, cudaStream_t s) {
  if (T == 0 || C == 0) return cudaSuccess;
  if (dim % 32) return cudaErrorInvalidValue;
  const int items = T * C;
  const int warps = 8;
  cb::launch_k(engram_gather_kernel, (items + warps - 1) / warps, 32 * warps, 0, s, 
      ids, T, C, dim, data_ptrs, sf_ptrs, bounds, world, reinterpret_cast<__nv_bfloat16*>(out));
  return cudaGetLastError();
}

__device__ __forceinline__ float block_sum_256(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
  if (threadIdx.x < 32) {
    s = l < int(blockDim.x >> 5) ? red[l] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (l == 0) red[32] = s;
  }
  __syncthreads();
  return red[32];
}

__global__ void engram_gate_kernel(__nv_bfloat16* __restrict__ X, const __nv_bfloat16* __restrict__ kv,
                                   const float* __restrict__ qw, const float* __restrict__ kw, int hc, int D,
                                   float eps, float clamp, float* __restrict__ sumsq, const int* __restrict__ tok,
                                   int img_id) {
  cb::pdl_entry();
  __shared__ float red[33];
  const int t = blockIdx.x;
  const bool skip = tok != nullptr && tok[t] == img_id;          // image tokens take no n-gram update
  const __nv_bfloat16* kvt = kv + size_t(t) * (hc + 1) * D;
  const __nv_bfloat16* v = kvt + size_t(hc) * D;
  float ss_new = 0.f;
  for (int s = 0; s < hc; ++s) {
    __nv_bfloat16* x = X + (size_t(t) * hc + s) * D;
    const __nv_bfloat16* k = kvt + size_t(s) * D;
    float sx = 0.f, sk = 0.f, dot = 0.f;
    for (int i = threadIdx.x; i < D; i += blockDim.x) {
      const float xi = __bfloat162float(x[i]), ki = __bfloat162float(k[i]);
      sx += xi * xi;
      sk += ki * ki;
      dot += (xi * qw[i]) * (ki * kw[i]);
    }
    sx = block_sum_256(sx, red);
    sk = block_sum_256(sk, red);
    dot = block_sum_256(dot, red);
    float z = dot * rsqrtf(sx / D + eps) * rsqrtf(sk / D + eps) * rsqrtf(float(D));
    z = fminf(fmaxf(z, -clamp), clamp);
    const float g = skip ? 0.f : 1.f / (1.f + __expf(-z));
    for (int i = threadIdx.x; i < D; i += blockDim.x) {
      const __nv_bfloat16 nx = __float2bfloat16_rn(__bfloat162float(x[i]) + g * __bfloat162float(v[i]));
      x[i] = nx;
      const float f = __bfloat162float(nx);
      ss_new += f * f;
    }
  }
  ss_new = block_sum_256(ss_new, red);
  if (threadIdx.x == 0 && sumsq) sumsq[t] = ss_new;
}

cudaError_t engram_gate(void* X, const void* kv, const float* qw, const float* kw, int T, int hc, int D, float eps,
                        float clamp, float* sumsq, cudaStream_t s, const int* tok, int img_id) {
  if (T == 0) return cudaSuccess;
  cb::launch_k(engram_gate_kernel, T, 256, 0, s, reinterpret_cast<__nv_bfloat16*>(X),
                                       reinterpret_cast<const __nv_bfloat16*>(kv), qw, kw, hc, D, eps, clamp, sumsq,
                                       tok, img_id);
  return cudaGetLastError();
}

}  // namespace cb
