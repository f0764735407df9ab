// Exact top-k over causal indexer logits (DSA): for query q the candidate keys are [0, q]; the k largest logits are
// selected, ties broken toward the lower key index (the order of a stable descending sort).  Output is the bit
// matrix the prefill attention kernel consumes: bit j of word w of row (row0 + q) = key 32w + j selected.
//
// One CTA per query row; the row lives in shared memory as order-preserving unsigned keys and a 4-pass 8-bit radix
// select finds the k-th largest value; equal-to-threshold keys are ranked with a block scan.  Reference: the exact
// top-k / paged top-k radix kernels (king_v10/bundle_v9/cuda_exact_topk.py:559, dec/cuda_paged_topk.py:559),
// written here from the algorithm.
#include "common.cuh"

namespace cb {

CB_DEVICE uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// inclusive scan of one int per thread over the block (blockDim.x multiple of 32, <= 1024)
CB_DEVICE int block_incl_scan(int v, int* sw) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += n;
  }
  if (lane == 31) sw[wid] = v;
  __syncthreads();
  if (wid == 0) {
    int w = lane < nw ? sw[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += n;
    }
    if (lane < nw) sw[lane] = w;
  }
  __syncthreads();
  const int r = v + (wid > 0 ? sw[wid - 1] : 0);
  __syncthreads();
  return r;
}

__global__ void topk_mask_kernel(const float* __restrict__ logits, int ldo, int Tq, int k, uint32_t* __restrict__ mask,
                                 int mask_words, int row0) {
  extern __shared__ uint32_t vals[];
  __shared__ int hist[256];
  __shared__ int sw[32];
  __shared__ uint32_t s_prefix;
  __shared__ int s_remaining;
  const int q = blockIdx.x;
  const int n = q + 1;                           // causal candidates
  uint32_t* out = mask + size_t(row0 + q) * mask_words;
  if (n <= k) {
    for (int w = threadIdx.x; w < mask_words; w += blockDim.x) {
      const int lo = w * 32;
      out[w] = lo + 32 <= n ? 0xffffffffu : (lo >= n ? 0u : ((1u << (n - lo)) - 1u));
    }
    return;
  }
  const float* row = logits + size_t(q) * ldo;
  for (int i = threadIdx.x; i < n; i += blockDim.x) vals[i] = order_key(row[i]);
  if (threadIdx.x == 0) { s_prefix = 0; s_remaining = k; }
  __syncthreads();
  uint32_t known = 0;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    const uint32_t prefix = s_prefix;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const uint32_t u = vals[i];
      if ((u & known) == prefix) atomicAdd(&hist[(u >> shift) & 255], 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int rem = s_remaining, c = 0, d = 255;
      for (; d > 0; --d) {
        if (c + hist[d] >= rem) break;
        c += hist[d];
      }
      s_remaining = rem - c;
      s_prefix = prefix | (uint32_t(d) << shift);
    }
    known |= 255u << shift;
    __syncthreads();
  }
  const uint32_t thr = s_prefix;
  const int take_eq = s_remaining;               // how many keys equal to thr are selected (lowest indices first)
  // rank the keys equal to thr in key order: each thread owns a contiguous range of words
  const int per = (mask_words + blockDim.x - 1) / blockDim.x;
  const int w0 = threadIdx.x * per, w1 = min(mask_words, w0 + per);
  int my_eq = 0;
  for (int w = w0; w < w1; ++w)
    for (int j = 0; j < 32; ++j) {
      const int key = w * 32 + j;
      if (key < n && vals[key] == thr) ++my_eq;
    }
  int before = block_incl_scan(my_eq, sw) - my_eq;
  for (int w = w0; w < w1; ++w) {
    uint32_t bits = 0;
    for (int j = 0; j < 32; ++j) {
      const int key = w * 32 + j;
      if (key >= n) break;
      const uint32_t u = vals[key];
      if (u > thr) bits |= 1u << j;
      else if (u == thr) { if (before < take_eq) bits |= 1u << j; ++before; }
    }
    out[w] = bits;
  }
}

cudaError_t topk_mask(const float* logits, int ldo, int Tq, int k, uint32_t* mask, int mask_words, int row0,
                      cudaStream_t s) {
  if (Tq <= 0) return cudaSuccess;
  const size_t smem = size_t(Tq) * 4;
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  static size_t attr = 0;
  if (smem > 48 * 1024 && smem > attr) {
    cudaError_t e = cudaFuncSetAttribute(topk_mask_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(200 * 1024));
    if (e != cudaSuccess) return e;
    attr = 200 * 1024;
  }
  topk_mask_kernel<<<Tq, 512, smem, s>>>(logits, ldo, Tq, k, mask, mask_words, row0);
  return cudaGetLastError();
}

}  // namespace cb
