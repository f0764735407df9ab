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

// All threads of the block: given the 256-bin histogram of this radix digit (over the keys that still match
// `prefix`), find the digit d such that the keys in bins above d number < rem <= those in bins >= d; record the
// extended prefix and how many keys of digit d remain to be taken.  A block scan over the bins in descending order
// replaces a 256-step serial walk.
CB_DEVICE void select_digit(const int* hist, int* sw, uint32_t* s_prefix, int* s_remaining, uint32_t prefix,
                            int shift) {
  const int t = threadIdx.x;
  const int rem = *s_remaining;                  // read by every thread before the scan's barriers
  const int c = t < 256 ? hist[255 - t] : 0;
  const int incl = block_incl_scan(c, sw);
  if (t < 256 && incl >= rem && incl - c < rem) {
    *s_remaining = rem - (incl - c);
    *s_prefix = prefix | (uint32_t(255 - t) << shift);
  }
  __syncthreads();
}

__global__ void topk_mask_kernel(const float* __restrict__ logits, int ldo, int Tq, int k, uint32_t* __restrict__ mask,
                                 int mask_words, int row0) {
  cb::pdl_entry();
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
    for (int i0 = 0; i0 < n; i0 += blockDim.x) {
      // warp-aggregated histogram update: lanes hitting the same bin add once (values of one row share most of
      // their high bits, so plain atomics would serialise on a few bins)
      const int i = i0 + threadIdx.x;
      int bin = -1;
      if (i < n) {
        const uint32_t u = vals[i];
        if ((u & known) == prefix) bin = int((u >> shift) & 255);
      }
      const unsigned grp = __match_any_sync(0xffffffffu, bin);
      if (bin >= 0 && (threadIdx.x & 31) == __ffs(grp) - 1) atomicAdd(&hist[bin], __popc(grp));
    }
    __syncthreads();
    select_digit(hist, sw, &s_prefix, &s_remaining, prefix, shift);
    known |= 255u << shift;
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

// ---------------------------------------------------------------------------------------------------------------
// Decode-side DSA top-k (the logits come from the tcgen05 kernel in indexer_decode.cu).
// ---------------------------------------------------------------------------------------------------------------
// Top-k slot indices of each row (keys in key order, -1 padded).  Row t's logits are logits[t * ldo + j] for its
// candidate keys j < n_t; slot of key j: slots[t * slot_stride + j] (slot_stride 0: one slot list shared by every
// row, e.g. the keys of one prefill sequence).  n_t = min(n_keys[t], Lmax), or with n_keys == nullptr the causal
// count row0 + t + 1 (row t of a sequence block starting at position row0).  Same radix select and lower-index tie
// rule as topk_mask_kernel; invalid keys carry -inf logits.
__global__ void topk_index_kernel(const float* __restrict__ logits, int ldo, const int* __restrict__ key_slots,
                                  int slot_stride, const int* __restrict__ n_keys, int row0, int Lmax, int k,
                                  int* __restrict__ out) {
  cb::pdl_entry();
  extern __shared__ uint32_t vals[];
  __shared__ int hist[256];
  __shared__ int sw[32];
  __shared__ uint32_t s_prefix;
  __shared__ int s_remaining;
  const int t = blockIdx.x;
  const int n = n_keys ? min(n_keys[t], Lmax) : min(row0 + t + 1, Lmax);
  const float* row = logits + size_t(t) * ldo;
  const int* slots = key_slots + size_t(t) * slot_stride;
  int* o = out + size_t(t) * k;
  if (n <= k) {
    for (int j = threadIdx.x; j < k; j += blockDim.x) o[j] = j < n ? slots[j] : -1;
    return;
  }
  for (int i = threadIdx.x; i < n; i += blockDim.x) vals[i] = order_key(row[i]);
  if (threadIdx.x == 0) { s_prefix = 0; s_remaining = k; }
  __syncthreads();
  uint32_t known = 0;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    const uint32_t prefix = s_prefix;
    for (int i0 = 0; i0 < n; i0 += blockDim.x) {
      // warp-aggregated histogram update: lanes hitting the same bin add once (values of one row share most of
      // their high bits, so plain atomics would serialise on a few bins)
      const int i = i0 + threadIdx.x;
      int bin = -1;
      if (i < n) {
        const uint32_t u = vals[i];
        if ((u & known) == prefix) bin = int((u >> shift) & 255);
      }
      const unsigned grp = __match_any_sync(0xffffffffu, bin);
      if (bin >= 0 && (threadIdx.x & 31) == __ffs(grp) - 1) atomicAdd(&hist[bin], __popc(grp));
    }
    __syncthreads();
    select_digit(hist, sw, &s_prefix, &s_remaining, prefix, shift);
    known |= 255u << shift;
  }
  const uint32_t thr = s_prefix;
  const int take_eq = s_remaining;
  // each thread owns a contiguous key range; selected keys are written in key order via a block scan of counts
  const int per = (n + blockDim.x - 1) / blockDim.x;
  const int j0 = threadIdx.x * per, j1 = min(n, j0 + per);
  int my_eq = 0, my_gt = 0;
  for (int j = j0; j < j1; ++j) { my_eq += vals[j] == thr; my_gt += vals[j] > thr; }
  const int eq_before = block_incl_scan(my_eq, sw) - my_eq;
  // selected in my range: all > thr, and == thr while the global equal rank < take_eq
  int my_sel = my_gt + max(0, min(my_eq, take_eq - eq_before));
  const int sel_before = block_incl_scan(my_sel, sw) - my_sel;
  int w = sel_before, eq = eq_before;
  for (int j = j0; j < j1; ++j) {
    const uint32_t u = vals[j];
    bool take = u > thr;
    if (u == thr) { take = eq < take_eq; ++eq; }
    if (take) o[w++] = slots[j];
  }
}

cudaError_t topk_slots(const float* logits, int ldo, const int* key_slots, int slot_stride, const int* n_keys,
                       int row0, int T, int Lmax, int k, int* out, cudaStream_t s);

cudaError_t topk_index(const float* logits, const int* key_slots, const int* n_keys, int T, int Lmax, int k,
                       int* out, cudaStream_t s) {
  return topk_slots(logits, Lmax, key_slots, Lmax, n_keys, 0, T, Lmax, k, out, s);
}

cudaError_t topk_slots(const float* logits, int ldo, const int* key_slots, int slot_stride, const int* n_keys,
                       int row0, int T, int Lmax, int k, int* out, cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  const size_t smem = size_t(Lmax) * 4;
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  if (smem > 48 * 1024) {
    cudaError_t e = smem_optin(topk_index_kernel, int(200 * 1024));
    if (e != cudaSuccess) return e;
  }
  cb::launch_k(topk_index_kernel, T, 512, smem, s, logits, ldo, key_slots, slot_stride, n_keys, row0, Lmax, k, out);
  return cudaGetLastError();
}

cudaError_t topk_mask(const float* logits, int ldo, int Tq, int k, uint32_t* mask, int mask_words, int row0,
                      cudaStream_t s) {
  if (Tq <= 0) return cudaSuccess;
  const size_t smem = size_t(Tq) * 4;
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  if (smem > 48 * 1024) {
    cudaError_t e = smem_optin(topk_mask_kernel, int(200 * 1024));
    if (e != cudaSuccess) return e;
  }
  cb::launch_k(topk_mask_kernel, Tq, 512, smem, s, logits, ldo, Tq, k, mask, mask_words, row0);
  return cudaGetLastError();
}

}  // namespace cb
