// CUDA-core kernels of the model: fp8 quantisers (UE8M0 1x128, SF-tile output), RMSNorm (+quant), RoPE,
// router top-k, MoE row layout / gather-quant / weighted combine, mHC coefficient / mix kernels, embedding.
//
// Reference parity: router = king_v10/bundle_v9/cuda_moe_front.py:262-346 (score, bias-only ranking, lower-id ties,
// renormalise, routed scale); quantisers = the pre-dispatch and q-norm quant of cuda_moe_prefill.py:3271-3452 and
// cuda_prefill_fuse.py:81; mHC = cuda_sinkhorn.py:150-190 and cuda_mhc_packed.py:60-170 (math restated in
// carbon_b200/ref/ops.py).  Every kernel here is written from that math; none reproduces another compiler's
// instruction sequence.
#include "common.cuh"
#include "small_ops.h"
#include "ptx.cuh"

namespace cb {

// SF tile word index for row r (within the whole matrix) and k-block kb: returns the byte offset.
CB_DEVICE size_t sf_byte_offset(int row, int kb, int row_blocks) {
  const int rb = row >> 7, r = row & 127;
  return ((size_t(kb >> 2) * row_blocks + rb) * 128 + (r & 31) * 4 + (r >> 5)) * 4 + (kb & 3);
}

// ---------------------------------------------------------------------------------------------------------------
// fp8 activation quantisation: one warp per (row, 512-column group); rows >= M (padding) get scale bytes 127.
// x: bf16 [M, K] with row stride ldx; q: fp8 [M, K] row stride ldq; src_rows (optional): gather map.
// ---------------------------------------------------------------------------------------------------------------
__global__ void act_quant_kernel(const __nv_bfloat16* __restrict__ x, int ldx, uint8_t* __restrict__ q, int ldq,
                                 uint32_t* __restrict__ sf, int M, int K, int row_blocks,
                                 const int* __restrict__ src_rows, int M_pad, const int* __restrict__ n_blocks,
                                 int x_rows) {
  cb::pdl_entry();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kg = blockIdx.x;
  const int rows_used = n_blocks ? min(M_pad, n_blocks[0] * 128) : M_pad;   // rows past the used blocks: never read
  // row groups stride over grid.y (at most 65535 groups of 8 rows per launch)
  for (int row = blockIdx.y * 8 + warp; row < rows_used; row += gridDim.y * 8) {
  int src = row < M ? row : -1;
  if (src >= 0 && src_rows) src = src_rows[row];
  if (src >= x_rows) src = -1;                   // anything but a valid source row quantises as a zero row
  uint32_t word = 0;
#pragma unroll
  for (int h = 0; h < 2; ++h) {                  // two halves of 256 columns = two k-blocks each
    const int kb = kg * 4 + h * 2 + (lane >> 4); // lanes 0-15 -> even k-block, 16-31 -> odd
    const int col = kb * 128 + (lane & 15) * 8;
    float v[8];
    bool in = src >= 0 && col < K;
    if (in && col + 8 <= K) {
      uint4 raw = *reinterpret_cast<const uint4*>(x + size_t(src) * ldx + col);
      v[0] = bf16_lo(raw.x); v[1] = bf16_hi(raw.x); v[2] = bf16_lo(raw.y); v[3] = bf16_hi(raw.y);
      v[4] = bf16_lo(raw.z); v[5] = bf16_hi(raw.z); v[6] = bf16_lo(raw.w); v[7] = bf16_hi(raw.w);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = (in && col + j < K) ? __bfloat162float(x[size_t(src) * ldx + col + j]) : 0.f;
    }
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[j]));
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const uint32_t sb = ue8m0_for_amax(amax);
    const float inv = ue8m0_inv(sb);
    if (row < M && col < K) {
      uint8_t* dst = q + size_t(row) * ldq + col;
      if (col + 8 <= K) {
        uint2 w;
        w.x = pack_fp8x4(v[0] * inv, v[1] * inv, v[2] * inv, v[3] * inv);
        w.y = pack_fp8x4(v[4] * inv, v[5] * inv, v[6] * inv, v[7] * inv);
        *reinterpret_cast<uint2*>(dst) = w;
      } else {
        for (int j = 0; j < 8 && col + j < K; ++j) {
          __nv_fp8_e4m3 f(v[j] * inv);
          dst[j] = *reinterpret_cast<uint8_t*>(&f);
        }
      }
    }
    // byte (h*2 + lane/16) of the SF word
    const uint32_t b = (kb * 128 < K) ? sb : 127u;
    const uint32_t b_other = __shfl_sync(0xffffffffu, b, lane ^ 16);
    if (lane == 0) word |= (b << (16 * h)) | (b_other << (16 * h + 8));
  }
  if (lane == 0) {
    const int rb = row >> 7, r = row & 127;
    sf[(size_t(kg) * row_blocks + rb) * 128 + (r & 31) * 4 + (r >> 5)] = word;
  }
  }
}

cudaError_t act_quant(const void* x, int ldx, void* q, int ldq, uint32_t* sf, int M, int K, const int* src_rows,
                      cudaStream_t s, const int* n_blocks, int x_rows) {
  if (x_rows < 0) x_rows = 0x7fffffff;
  const int row_blocks = ceil_div(M, 128), M_pad = row_blocks * 128;
  dim3 grid(ceil_div(K, 512), min(ceil_div(M_pad, 8), 65535));
  cb::launch_k(act_quant_kernel, grid, 256, 0, s, reinterpret_cast<const __nv_bfloat16*>(x), ldx,
                                        reinterpret_cast<uint8_t*>(q), ldq, sf, M, K, row_blocks, src_rows, M_pad,
                                        n_blocks, x_rows);
  return cudaGetLastError();
}

// Gather of already-quantised rows: dst row r = src row src_rows[r] (fp8 bytes and its SF words; -1 = a padding row,
// not written).  One warp per destination row; rows past n_blocks*128 are left alone.  Used by the MoE dispatch so
// that every token is quantised once instead of once per selected expert.
__global__ void gather_fp8_rows_kernel(const uint8_t* __restrict__ src, const uint32_t* __restrict__ src_sf,
                                       int src_rows_n, int K, const int* __restrict__ src_rows, int M,
                                       const int* __restrict__ n_blocks, uint8_t* __restrict__ dst,
                                       uint32_t* __restrict__ dst_sf) {
  cb::pdl_entry();
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  if (n_blocks && row >= n_blocks[0] * 128) return;
  int sr = src_rows[row];
  if (sr >= 0 && !cb_check_index(sr, src_rows_n, "gather_fp8_rows")) sr = -1;
  // padding rows of an expert segment are left as they are: every output row of the grouped GEMMs depends on its
  // own input row only, and no consumer reads a padding row's output (writing zeros cost ~150 MB per decode call)
  if (sr < 0) return;
  const uint4* s4 = reinterpret_cast<const uint4*>(src + size_t(sr) * K);
  uint4* d4 = reinterpret_cast<uint4*>(dst + size_t(row) * K);
  for (int c = lane; c < K / 16; c += 32) d4[c] = s4[c];
  const int kgroups = (K + 511) / 512;
  const int src_rb = (src_rows_n + 127) / 128, dst_rb = (M + 127) / 128;
  for (int kg = lane; kg < kgroups; kg += 32) {
    const uint32_t w = src_sf[(size_t(kg) * src_rb + (sr >> 7)) * 128 + (sr & 31) * 4 + ((sr & 127) >> 5)];
    dst_sf[(size_t(kg) * dst_rb + (row >> 7)) * 128 + (row & 31) * 4 + ((row & 127) >> 5)] = w;
  }
}

cudaError_t gather_fp8_rows(const void* src, const uint32_t* src_sf, int src_rows_n, int K, const int* src_rows,
                            int M, const int* n_blocks, void* dst, uint32_t* dst_sf, cudaStream_t s) {
  if (K % 16) return cudaErrorInvalidValue;
  cb::launch_k(gather_fp8_rows_kernel, ceil_div(M, 8), 256, 0, s, reinterpret_cast<const uint8_t*>(src), src_sf, src_rows_n,
                                                        K, src_rows, M, n_blocks, reinterpret_cast<uint8_t*>(dst),
                                                        dst_sf);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------------------------------
// RMSNorm over rows: y = x * rsqrt(mean(x^2) + eps) * w. Optional bf16 out and/or fp8 + SF out.
// One CTA (256 threads) per row; D % 8 == 0.
// ---------------------------------------------------------------------------------------------------------------
template <int MAXV>
__global__ void rms_norm_kernel(const __nv_bfloat16* __restrict__ x, int ldx, const float* __restrict__ w,
                                __nv_bfloat16* __restrict__ y, int ldy, uint8_t* __restrict__ q, uint32_t* sf,
                                int row_blocks, int D, float eps) {
  cb::pdl_entry();
  __shared__ float red[32];
  const int row = blockIdx.x;
  const __nv_bfloat16* xr = x + size_t(row) * ldx;
  float v[MAXV * 8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int col = (i * blockDim.x + threadIdx.x) * 8;
    if (col < D) {
      uint4 raw = *reinterpret_cast<const uint4*>(xr + col);
      v[i * 8 + 0] = bf16_lo(raw.x); v[i * 8 + 1] = bf16_hi(raw.x); v[i * 8 + 2] = bf16_lo(raw.y);
      v[i * 8 + 3] = bf16_hi(raw.y); v[i * 8 + 4] = bf16_lo(raw.z); v[i * 8 + 5] = bf16_hi(raw.z);
      v[i * 8 + 6] = bf16_lo(raw.w); v[i * 8 + 7] = bf16_hi(raw.w);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[i * 8 + j] * v[i * 8 + j];
    }
  }
  ss = block_sum(ss, red);
  const float r = rsqrtf(ss / D + eps);
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int col = (i * blockDim.x + threadIdx.x) * 8;
    if (col < D) {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i * 8 + j] = __bfloat162float(__float2bfloat16_rn(v[i * 8 + j] * r * w[col + j]));
      if (y) {
        uint4 o;
        o.x = pack_bf16x2(v[i * 8 + 0], v[i * 8 + 1]); o.y = pack_bf16x2(v[i * 8 + 2], v[i * 8 + 3]);
        o.z = pack_bf16x2(v[i * 8 + 4], v[i * 8 + 5]); o.w = pack_bf16x2(v[i * 8 + 6], v[i * 8 + 7]);
        *reinterpret_cast<uint4*>(y + size_t(row) * ldy + col) = o;
      }
    }
  }
  if (q) {
    // 16 threads own one 128-column block (8 values each): reduce amax across them.
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int col = (i * blockDim.x + threadIdx.x) * 8;
      float amax = 0.f;
      if (col < D)
#pragma unroll
        for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[i * 8 + j]));
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      const uint32_t sb = ue8m0_for_amax(amax);
      const float inv = ue8m0_inv(sb);
      if (col < D) {
        uint2 wq;
        wq.x = pack_fp8x4(v[i * 8 + 0] * inv, v[i * 8 + 1] * inv, v[i * 8 + 2] * inv, v[i * 8 + 3] * inv);
        wq.y = pack_fp8x4(v[i * 8 + 4] * inv, v[i * 8 + 5] * inv, v[i * 8 + 6] * inv, v[i * 8 + 7] * inv);
        *reinterpret_cast<uint2*>(q + size_t(row) * D + col) = wq;
        if ((threadIdx.x & 15) == 0)
          reinterpret_cast<uint8_t*>(sf)[sf_byte_offset(row, col / 128, row_blocks)] = uint8_t(sb);
      }
    }
  }
}

cudaError_t rms_norm(const void* x, int ldx, const float* w, void* y, int ldy, void* q, uint32_t* sf, int M, int D,
                     float eps, cudaStream_t s) {
  if (D % 8) return cudaErrorInvalidValue;
  const int per = ceil_div(D, 256 * 8);
  const int rb = ceil_div(M, 128);
  auto xx = reinterpret_cast<const __nv_bfloat16*>(x);
  auto yy = reinterpret_cast<__nv_bfloat16*>(y);
  auto qq = reinterpret_cast<uint8_t*>(q);
  if (q && D % 128) return cudaErrorInvalidValue;
  if (per <= 1) cb::launch_k(rms_norm_kernel<1>, M, 256, 0, s, xx, ldx, w, yy, ldy, qq, sf, rb, D, eps);
  else if (per <= 2) cb::launch_k(rms_norm_kernel<2>, M, 256, 0, s, xx, ldx, w, yy, ldy, qq, sf, rb, D, eps);
  else if (per <= 4) cb::launch_k(rms_norm_kernel<4>, M, 256, 0, s, xx, ldx, w, yy, ldy, qq, sf, rb, D, eps);
  else return cudaErrorInvalidValue;
  return cudaGetLastError();
}

// SF padding rows (>= M inside the last 128-row block) get scale bytes 127 so every SF tile is defined.
__global__ void sf_pad_kernel(uint32_t* sf, int M, int K, int row_blocks) {
  cb::pdl_entry();
  const int kg = blockIdx.x;
  const int r = (M & 127) + threadIdx.x;
  if ((M & 127) == 0 || r >= 128) return;
  const int row = (row_blocks - 1) * 128 + r;
  sf[(size_t(kg) * row_blocks + (row >> 7)) * 128 + (r & 31) * 4 + (r >> 5)] = 0x7f7f7f7fu;
}
cudaError_t sf_pad(uint32_t* sf, int M, int K, cudaStream_t s) {
  const int rb = ceil_div(M, 128);
  if ((M & 127) == 0) return cudaSuccess;
  cb::launch_k(sf_pad_kernel, ceil_div(K, 512), 128, 0, s, sf, M, K, rb);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------------------------------
// RoPE (interleaved pairs) in place on bf16 x[T, H, *] at column offset `off`, width `dim`.
// cos_sin: fp32 [max_pos, dim] laid out as (cos_0, sin_0, cos_1, sin_1, ...).
// ---------------------------------------------------------------------------------------------------------------
// RoPE in place on dims [off, off + dim) of every head (interleaved pairs).  Grid (T, ceil(H / 4)): a CTA rotates 4
// heads of one token, one pair per thread (dim <= 64), so decode-sized calls spread over many SMs.
__global__ void rope_kernel(__nv_bfloat16* x, int64_t stride_t, int64_t stride_h, int H, int off, int dim,
                            const float* __restrict__ cos_sin, const int* __restrict__ pos, int inverse) {
  cb::pdl_entry();
  const int t = blockIdx.x;
  const int p = pos[t];
  const int pairs = dim / 2;
  for (int i = threadIdx.x; i < 4 * pairs; i += blockDim.x) {
    const int h = blockIdx.y * 4 + i / pairs, j = i % pairs;
    if (h >= H) break;
    __nv_bfloat162* e = reinterpret_cast<__nv_bfloat162*>(x + t * stride_t + h * stride_h + off + 2 * j);
    const float2 cs = *reinterpret_cast<const float2*>(cos_sin + size_t(p) * dim + 2 * j);
    const float c = cs.x, sn = inverse ? -cs.y : cs.y;
    const float2 ab = __bfloat1622float2(*e);
    *e = __floats2bfloat162_rn(ab.x * c - ab.y * sn, ab.x * sn + ab.y * c);
  }
}
cudaError_t rope_inplace(void* x, int T, int64_t stride_t, int64_t stride_h, int H, int off, int dim,
                         const float* cos_sin, const int* pos, bool inverse, cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  if ((off | dim | stride_t | stride_h) & 1) return cudaErrorInvalidValue;     // bf16 pairs are 4-byte aligned
  cb::launch_k(rope_kernel, dim3(T, ceil_div(H, 4)), 128, 0, s, reinterpret_cast<__nv_bfloat16*>(x), stride_t,
               stride_h, H, off, dim, cos_sin, pos, inverse ? 1 : 0);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------------------------------
// Router: one warp per token. act = f(logit); key = act + bias; top-k by key (ties -> lower id);
// w = act[picked]; renormalise (optional); x route_scale.  E <= 1024, k <= 16.
// score: 0 sigmoid, 1 sqrt(softplus), 2 softmax.
// ---------------------------------------------------------------------------------------------------------------
// Multimodal: when `bias_img` is given, tokens whose id (tok[t]) equals img_id rank with bias_img instead of bias
// (the reference switches to a vision-language bias for image tokens; cuda_moe_front.py:265-269).
template <int EPL>  // experts per lane
__global__ void router_kernel(const float* __restrict__ logits, const float* __restrict__ bias, int T, int E, int k,
                              int score, int norm, float route_scale, float* __restrict__ w_out,
                              int* __restrict__ id_out, const float* __restrict__ bias_img,
                              const int* __restrict__ tok, int img_id, int n_groups, int topk_groups) {
  cb::pdl_entry();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= T) return;
  if (bias_img != nullptr && tok != nullptr && tok[warp] == img_id) bias = bias_img;
  const float* l = logits + size_t(warp) * E;
  float act[EPL], key[EPL];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = i * 32 + lane;
    act[i] = e < E ? l[e] : -INFINITY;
    mx = fmaxf(mx, act[i]);
  }
  if (score == 2) {
    mx = warp_max(mx);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < EPL; ++i) { act[i] = (i * 32 + lane) < E ? __expf(act[i] - mx) : 0.f; s += act[i]; }
    s = warp_sum(s);
#pragma unroll
    for (int i = 0; i < EPL; ++i) act[i] /= s;
  } else {
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const float z = act[i];
      if (score == 0) act[i] = 1.f / (1.f + expf(-z));
      else act[i] = sqrtf(z > 20.f ? z : log1pf(expf(z)));   // softplus from its definition
    }
  }
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = i * 32 + lane;
    key[i] = e < E ? act[i] + (bias ? bias[e] : 0.f) : -INFINITY;
  }
  if (n_groups > 1) {
    // group-limited routing: keep the experts of the topk_groups groups whose two best keys sum highest (ties ->
    // lower group id); group g holds experts [g*G, (g+1)*G)
    const int G = E / n_groups;
    float my_gs = -INFINITY;                 // lane g < n_groups: score of group g
    for (int g = 0; g < n_groups; ++g) {
      float b1 = -INFINITY, b2 = -INFINITY;  // this lane's two best keys in group g
#pragma unroll
      for (int i = 0; i < EPL; ++i) {
        const int e = i * 32 + lane;
        if (e < E && e / G == g) {
          if (key[i] > b1) { b2 = b1; b1 = key[i]; } else if (key[i] > b2) { b2 = key[i]; }
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float o1 = __shfl_xor_sync(0xffffffffu, b1, o), o2 = __shfl_xor_sync(0xffffffffu, b2, o);
        const float n1 = fmaxf(b1, o1);
        const float n2 = fmaxf(fminf(b1, o1), fmaxf(b2, o2));
        b1 = n1; b2 = n2;
      }
      if (lane == g) my_gs = b1 + b2;
    }
    uint32_t keep = 0;                       // bit g: group g selected
    for (int r = 0; r < topk_groups; ++r) {
      float bv = (lane < n_groups && !((keep >> lane) & 1u)) ? my_gs : -INFINITY;
      int bi = lane < n_groups ? lane : 0x7fffffff;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
      }
      if (bi < n_groups) keep |= 1u << bi;
    }
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const int e = i * 32 + lane;
      if (e < E && !((keep >> (e / G)) & 1u)) key[i] = -INFINITY;
    }
  }
  float wsum = 0.f, my_w = 0.f;
  int my_id = 0;
  for (int r = 0; r < k; ++r) {
    // local best (lowest id among equal keys: lower i first, strict >)
    float bv = -INFINITY; int bi = 0x7fffffff; float ba = 0.f;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const int e = i * 32 + lane;
      if (e < E && key[i] > bv) { bv = key[i]; bi = e; ba = act[i]; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      const float oa = __shfl_xor_sync(0xffffffffu, ba, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; ba = oa; }
    }
    if (lane == r) { my_w = ba; my_id = bi; }
    wsum += ba;
    if ((bi & 31) == lane) key[bi >> 5] = -INFINITY;
  }
  if (lane < k) {
    float wv = my_w;
    if (norm) wv = wv / (wsum + 1e-20f);
    w_out[size_t(warp) * k + lane] = wv * route_scale;
    id_out[size_t(warp) * k + lane] = my_id;
  }
}
cudaError_t router_topk(const float* logits, const float* bias, int T, int E, int k, int score, bool norm,
                        float route_scale, float* w, int* ids, cudaStream_t s, const float* bias_img,
                        const int* tok, int img_id, int n_groups, int topk_groups) {
  if (T == 0) return cudaSuccess;
  if (k > 32 || E > 1024) return cudaErrorInvalidValue;
  if (n_groups > 1 && (n_groups > 32 || E % n_groups || topk_groups < 1 || topk_groups > n_groups))
    return cudaErrorInvalidValue;
  const int blocks = ceil_div(T * 32, 256);
#define CB_ROUTER(N) cb::launch_k(router_kernel<N>, blocks, 256, 0, s, logits, bias, T, E, k, score, norm ? 1 : 0, route_scale, w, \
                                                            ids, bias_img, tok, img_id, n_groups, topk_groups)
  if (E <= 64) CB_ROUTER(2);
  else if (E <= 128) CB_ROUTER(4);
  else if (E <= 256) CB_ROUTER(8);
  else if (E <= 512) CB_ROUTER(16);
  else CB_ROUTER(32);
#undef CB_ROUTER
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------------------------------
// MoE layout: expert-sorted rows, every expert segment padded to `align` rows (128, or 256 for CTA-pair GEMM
// tiles), 128-row blocks tagged with their expert.  Three grid-wide steps: per-expert counts, segment offsets (one
// CTA scans the padded counts and tags the blocks), scatter of (token, slot) pairs.  Row order inside an expert
// segment is arbitrary (every row's GEMM result is independent of its position and the combine is per token).
__global__ void moe_count_local_kernel(const int* __restrict__ ids, int Tk, int E, int* __restrict__ cnt) {
  cb::pdl_entry();
  extern __shared__ int hcnt[];
  for (int e = threadIdx.x; e < E; e += blockDim.x) hcnt[e] = 0;
  __syncthreads();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < Tk; i += gridDim.x * blockDim.x) {
    const int e = ids[i];
    if (e >= 0 && e < E) atomicAdd(&hcnt[e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x)
    if (hcnt[e]) atomicAdd(&cnt[e], hcnt[e]);
}

__global__ void moe_offsets_kernel(const int* __restrict__ cnt, int E, int align, int max_blocks,
                                   int* __restrict__ start, int* __restrict__ fill, int* __restrict__ m_block_expert,
                                   int* __restrict__ num_blocks, int* __restrict__ row_src) {
  cb::pdl_entry();
  __shared__ int wsum[32];
  __shared__ int s_total;
  const int t = threadIdx.x, lane = t & 31, wid = t >> 5;
  const int c = t < E ? cnt[t] : 0;
  const int padded = (c + align - 1) / align * align;
  int v = padded;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += n;
  }
  if (lane == 31) wsum[wid] = v;
  __syncthreads();
  if (wid == 0) {
    int w = lane < int(blockDim.x >> 5) ? wsum[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += n;
    }
    wsum[lane] = w;
    if (lane == 31) s_total = w;
  }
  __syncthreads();
  const int incl = v + (wid > 0 ? wsum[wid - 1] : 0);
  const int st = incl - padded;
  const int max_rows = max_blocks * 128;
  __shared__ int st_s[1024], c_s[1024];
  if (t < E) {
    start[t] = st;
    fill[t] = 0;
    st_s[t] = st;
    c_s[t] = c;
    for (int b = st >> 7; b < (st + padded) >> 7 && b < max_blocks; ++b) m_block_expert[b] = t;
  }
  const int total_blocks = s_total >> 7;
  if (t == 0) num_blocks[0] = total_blocks;
  for (int b = total_blocks + t; b < max_blocks; b += blockDim.x) m_block_expert[b] = -1;
  __syncthreads();                              // the block -> expert map above is visible to the whole CTA
  // padding rows of each expert segment and every row past the used blocks -> -1, all threads over all rows
  for (int r = t; r < max_rows; r += blockDim.x) {
    const int b = r >> 7;
    const int e = b < total_blocks ? m_block_expert[b] : -1;
    if (e < 0 || r - st_s[e] >= c_s[e]) row_src[r] = -1;
  }
}

__global__ void moe_scatter_kernel(const int* __restrict__ ids, int Tk, int k, int E, const int* __restrict__ start,
                                   int* __restrict__ fill, int max_rows, int* __restrict__ slot_pos,
                                   int* __restrict__ row_src) {
  cb::pdl_entry();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < Tk; i += gridDim.x * blockDim.x) {
    const int e = ids[i];
    int pos = -1;
    if (e >= 0 && e < E) {
      pos = start[e] + atomicAdd(&fill[e], 1);
      if (pos < max_rows) row_src[pos] = i / k;
      else pos = -1;
    }
    slot_pos[i] = pos;
  }
}

// counts [E] (output), scratch [2E] (segment starts, fill counters)
cudaError_t moe_layout(const int* ids, int T, int k, int E, int max_blocks, int* slot_pos, int* row_src,
                       int* m_block_expert, int* num_blocks, int* counts, cudaStream_t s, int align, int* scratch) {
  if (E > 1024 || (align != 128 && align != 256) || !counts || !scratch) return cudaErrorInvalidValue;
  const int Tk = T * k;
  cudaError_t e = cudaMemsetAsync(counts, 0, sizeof(int) * E, s);
  if (e != cudaSuccess) return e;
  const int blocks = Tk / 1024 + 1 < 148 ? Tk / 1024 + 1 : 148;
  cb::launch_k(moe_count_local_kernel, blocks, 256, E * sizeof(int), s, ids, Tk, E, counts);
  cb::launch_k(moe_offsets_kernel, 1, 1024, 0, s, counts, E, align, max_blocks, scratch, scratch + E, m_block_expert,
                                        num_blocks, row_src);
  cb::launch_k(moe_scatter_kernel, blocks, 256, 0, s, ids, Tk, k, E, scratch, scratch + E, max_blocks * 128, slot_pos,
                                            row_src);
  return cudaGetLastError();
}

// Weighted combine: out[t] = sum_j w[t,j] * Y[slot_pos[t,j]] (+ add[t]); bf16 in/out, fp32 math. D % 8 == 0.
__global__ void moe_combine_kernel(const __nv_bfloat16* __restrict__ Y, int ldy, const float* __restrict__ w,
                                   const int* __restrict__ slot_pos, int k, const __nv_bfloat16* __restrict__ add,
                                   __nv_bfloat16* __restrict__ out, int D) {
  cb::pdl_entry();
  const int t = blockIdx.x;
  for (int c = (blockIdx.y * blockDim.x + threadIdx.x) * 8; c < D; c += gridDim.y * blockDim.x * 8) {
    float acc[8];
    if (add) {
      uint4 raw = *reinterpret_cast<const uint4*>(add + size_t(t) * D + c);
      acc[0] = bf16_lo(raw.x); acc[1] = bf16_hi(raw.x); acc[2] = bf16_lo(raw.y); acc[3] = bf16_hi(raw.y);
      acc[4] = bf16_lo(raw.z); acc[5] = bf16_hi(raw.z); acc[6] = bf16_lo(raw.w); acc[7] = bf16_hi(raw.w);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.f;
    }
    for (int j = 0; j < k; ++j) {
      const int pos = slot_pos[t * k + j];
      if (pos < 0) continue;
      const float wv = w[t * k + j];
      uint4 raw = *reinterpret_cast<const uint4*>(Y + size_t(pos) * ldy + c);
      acc[0] += wv * bf16_lo(raw.x); acc[1] += wv * bf16_hi(raw.x); acc[2] += wv * bf16_lo(raw.y);
      acc[3] += wv * bf16_hi(raw.y); acc[4] += wv * bf16_lo(raw.z); acc[5] += wv * bf16_hi(raw.z);
      acc[6] += wv * bf16_lo(raw.w); acc[7] += wv * bf16_hi(raw.w);
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]); o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]); o.w = pack_bf16x2(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(out + size_t(t) * D + c) = o;
  }
}
cudaError_t moe_combine(const void* Y, int ldy, const float* w, const int* slot_pos, int T, int k, const void* add,
                        void* out, int D, cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  if (D % 8) return cudaErrorInvalidValue;
  cb::launch_k(moe_combine_kernel, dim3(T, ceil_div(D, 128 * 8)), 128, 0, s, reinterpret_cast<const __nv_bfloat16*>(Y), ldy, w, slot_pos, k,
                                       reinterpret_cast<const __nv_bfloat16*>(add),
                                       reinterpret_cast<__nv_bfloat16*>(out), D);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------------------------------
// mHC
// ---------------------------------------------------------------------------------------------------------------
// Coefficients from the stats projection. mix: fp32 [T, ld_mix] holding m_hi (cols 0..nmix-1) and m_lo
// (cols nmix..2*nmix-1) of x_flat·fn^T (fn split into bf16 hi + lo parts); sumsq [T] = Σ x_flat².
// One thread per token (hc == 4).
__global__ void mhc_coeffs_kernel(const float* __restrict__ mix, int ld_mix, const float* __restrict__ sumsq,
                                  const float* __restrict__ base, const float* __restrict__ scale, int T, int flat_dim,
                                  int iters, float hc_eps, float rms_eps, float* __restrict__ pre,
                                  float* __restrict__ post, float* __restrict__ comb) {
  cb::pdl_entry();
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  constexpr int HC = 4, NMIX = 24;
  const float rsq = rsqrtf(sumsq[t] / flat_dim + rms_eps);
  const float* m = mix + size_t(t) * ld_mix;
  float mm[NMIX];
#pragma unroll
  for (int j = 0; j < NMIX; ++j) mm[j] = (m[j] + m[NMIX + j]) * rsq;
#pragma unroll
  for (int j = 0; j < HC; ++j) {
    pre[t * HC + j] = 1.f / (1.f + expf(-(mm[j] * scale[0] + base[j]))) + hc_eps;
    post[t * HC + j] = 2.f / (1.f + expf(-(mm[HC + j] * scale[1] + base[HC + j])));
  }
  float c[HC][HC];
#pragma unroll
  for (int i = 0; i < HC; ++i) {
    float mx = -INFINITY;
#pragma unroll
    for (int o = 0; o < HC; ++o) { c[i][o] = mm[2 * HC + i * HC + o] * scale[2] + base[2 * HC + i * HC + o]; mx = fmaxf(mx, c[i][o]); }
    float s = 0.f;
#pragma unroll
    for (int o = 0; o < HC; ++o) { c[i][o] = expf(c[i][o] - mx); s += c[i][o]; }
#pragma unroll
    for (int o = 0; o < HC; ++o) c[i][o] = c[i][o] / s + hc_eps;
  }
  // column normalise, then iters-1 (row, column) passes
#pragma unroll
  for (int o = 0; o < HC; ++o) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < HC; ++i) s += c[i][o];
#pragma unroll
    for (int i = 0; i < HC; ++i) c[i][o] /= (s + hc_eps);
  }
  for (int it = 1; it < iters; ++it) {
#pragma unroll
    for (int i = 0; i < HC; ++i) {
      float s = 0.f;
#pragma unroll
      for (int o = 0; o < HC; ++o) s += c[i][o];
#pragma unroll
      for (int o = 0; o < HC; ++o) c[i][o] /= (s + hc_eps);
    }
#pragma unroll
    for (int o = 0; o < HC; ++o) {
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < HC; ++i) s += c[i][o];
#pragma unroll
      for (int i = 0; i < HC; ++i) c[i][o] /= (s + hc_eps);
    }
  }
#pragma unroll
  for (int i = 0; i < HC; ++i)
#pragma unroll
    for (int o = 0; o < HC; ++o) comb[t * 16 + i * HC + o] = c[i][o];
}
// mHC mixing statistics for few tokens (decode): mix[t, r] = Σ_k X[t, k] · fn[r, k] for the fn rows r < R (bf16
// [hi; lo] parts of the fp32 projections), fp32 accumulation.  One CTA per (token, 8 fn rows): each thread walks
// 8-column chunks of the row (16-byte loads of X and of the 8 fn rows), then a block reduction per output.  The
// tensor-core GEMM would run a single 128-row tile split over K for a decode batch.
__global__ void __launch_bounds__(256) mhc_stats_small_kernel(const __nv_bfloat16* __restrict__ X, int ldx,
                                                               const __nv_bfloat16* __restrict__ fn, int K,
                                                               float* __restrict__ out, int ldo) {
  cb::pdl_entry();
  __shared__ float red[8][8];
  const int t = blockIdx.x, r0 = blockIdx.y * 8;
  const __nv_bfloat16* xr = X + size_t(t) * ldx;
  float acc[8];
#pragma unroll
  for (int r = 0; r < 8; ++r) acc[r] = 0.f;
  for (int c = threadIdx.x * 8; c < K; c += blockDim.x * 8) {
    const uint4 xv = *reinterpret_cast<const uint4*>(xr + c);
    const float x[8] = {bf16_lo(xv.x), bf16_hi(xv.x), bf16_lo(xv.y), bf16_hi(xv.y),
                        bf16_lo(xv.z), bf16_hi(xv.z), bf16_lo(xv.w), bf16_hi(xv.w)};
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const uint4 fv = __ldg(reinterpret_cast<const uint4*>(fn + size_t(r0 + r) * K + c));
      acc[r] += x[0] * bf16_lo(fv.x) + x[1] * bf16_hi(fv.x) + x[2] * bf16_lo(fv.y) + x[3] * bf16_hi(fv.y) +
                x[4] * bf16_lo(fv.z) + x[5] * bf16_hi(fv.z) + x[6] * bf16_lo(fv.w) + x[7] * bf16_hi(fv.w);
    }
  }
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    const float v = warp_sum(acc[r]);
    if (lane == 0) red[wid][r] = v;
  }
  __syncthreads();
  if (threadIdx.x < 8) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) v += red[w][threadIdx.x];
    out[size_t(t) * ldo + r0 + threadIdx.x] = v;
  }
}

cudaError_t mhc_stats_small(const void* X, int ldx, const void* fn, int R, int K, int T, float* out, int ldo,
                            cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  if (R % 8 || K % 8 || ldx % 8) return cudaErrorInvalidValue;
  cb::launch_k(mhc_stats_small_kernel, dim3(T, R / 8), 256, 0, s, reinterpret_cast<const __nv_bfloat16*>(X), ldx,
               reinterpret_cast<const __nv_bfloat16*>(fn), K, out, ldo);
  return cudaGetLastError();
}

cudaError_t mhc_coeffs(const float* mix, int ld_mix, const float* sumsq, const float* base, const float* scale, int T,
                       int flat_dim, int iters, float hc_eps, float rms_eps, float* pre, float* post, float* comb,
                       cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  cb::launch_k(mhc_coeffs_kernel, ceil_div(T, 128), 128, 0, s, mix, ld_mix, sumsq, base, scale, T, flat_dim, iters, hc_eps,
                                                     rms_eps, pre, post, comb);
  return cudaGetLastError();
}

// Head coefficients: pre_j = sigmoid(m_j*rsq*scale + base_j) + eps from a [T, 2*HC] hi/lo projection.
__global__ void mhc_head_coeffs_kernel(const float* __restrict__ mix, int ld_mix, const float* __restrict__ sumsq,
                                       const float* __restrict__ base, const float* __restrict__ scale, int T,
                                       int flat_dim, float hc_eps, float rms_eps, float* __restrict__ pre) {
  cb::pdl_entry();
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  const float rsq = rsqrtf(sumsq[t] / flat_dim + rms_eps);
  const float* m = mix + size_t(t) * ld_mix;
  for (int j = 0; j < 4; ++j)
    pre[t * 4 + j] = 1.f / (1.f + expf(-((m[j] + m[4 + j]) * rsq * scale[0] + base[j]))) + hc_eps;
}
cudaError_t mhc_head_coeffs(const float* mix, int ld_mix, const float* sumsq, const float* base, const float* scale,
                            int T, int flat_dim, float hc_eps, float rms_eps, float* pre, cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  cb::launch_k(mhc_head_coeffs_kernel, ceil_div(T, 128), 128, 0, s, mix, ld_mix, sumsq, base, scale, T, flat_dim, hc_eps,
                                                          rms_eps, pre);
  return cudaGetLastError();
}

// Pre-mix + RMSNorm (+ fp8 quant): y = RMSNorm(Σ_i pre_i X_i) * w.  X bf16 [T, 4, D]; one CTA per token.
// Writes bf16 y (optional) and fp8 q + SF tiles (optional). The mixed sum is rounded to bf16 before the norm.
template <int MAXV>
__global__ void mhc_pre_norm_kernel(const __nv_bfloat16* __restrict__ X, const float* __restrict__ pre,
                                    const float* __restrict__ w, int D, float eps, __nv_bfloat16* __restrict__ y,
                                    uint8_t* __restrict__ q, uint32_t* __restrict__ sf, int row_blocks,
                                    const int* __restrict__ rows) {
  cb::pdl_entry();
  __shared__ float red[32];
  const int t_out = blockIdx.x;
  const int t = rows ? rows[t_out] : t_out;
  const __nv_bfloat16* xr = X + size_t(t) * 4 * D;
  const float p0 = pre[t * 4 + 0], p1 = pre[t * 4 + 1], p2 = pre[t * 4 + 2], p3 = pre[t * 4 + 3];
  float v[MAXV * 8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int col = (i * blockDim.x + threadIdx.x) * 8;
    if (col < D) {
      float a[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) a[j] = 0.f;
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        const float ps = s == 0 ? p0 : s == 1 ? p1 : s == 2 ? p2 : p3;
        uint4 raw = *reinterpret_cast<const uint4*>(xr + size_t(s) * D + col);
        a[0] += ps * bf16_lo(raw.x); a[1] += ps * bf16_hi(raw.x); a[2] += ps * bf16_lo(raw.y);
        a[3] += ps * bf16_hi(raw.y); a[4] += ps * bf16_lo(raw.z); a[5] += ps * bf16_hi(raw.z);
        a[6] += ps * bf16_lo(raw.w); a[7] += ps * bf16_hi(raw.w);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v[i * 8 + j] = __bfloat162float(__float2bfloat16_rn(a[j]));
        ss += v[i * 8 + j] * v[i * 8 + j];
      }
    }
  }
  ss = block_sum(ss, red);
  const float r = rsqrtf(ss / D + eps);
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int col = (i * blockDim.x + threadIdx.x) * 8;
    float amax = 0.f;
    if (col < D) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v[i * 8 + j] = __bfloat162float(__float2bfloat16_rn(v[i * 8 + j] * r * w[col + j]));
        amax = fmaxf(amax, fabsf(v[i * 8 + j]));
      }
      if (y) {
        uint4 o;
        o.x = pack_bf16x2(v[i * 8 + 0], v[i * 8 + 1]); o.y = pack_bf16x2(v[i * 8 + 2], v[i * 8 + 3]);
        o.z = pack_bf16x2(v[i * 8 + 4], v[i * 8 + 5]); o.w = pack_bf16x2(v[i * 8 + 6], v[i * 8 + 7]);
        *reinterpret_cast<uint4*>(y + size_t(t_out) * D + col) = o;
      }
    }
    if (q) {
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      const uint32_t sb = ue8m0_for_amax(amax);
      const float inv = ue8m0_inv(sb);
      if (col < D) {
        uint2 wq;
        wq.x = pack_fp8x4(v[i * 8 + 0] * inv, v[i * 8 + 1] * inv, v[i * 8 + 2] * inv, v[i * 8 + 3] * inv);
        wq.y = pack_fp8x4(v[i * 8 + 4] * inv, v[i * 8 + 5] * inv, v[i * 8 + 6] * inv, v[i * 8 + 7] * inv);
        *reinterpret_cast<uint2*>(q + size_t(t_out) * D + col) = wq;
        if ((threadIdx.x & 15) == 0)
          reinterpret_cast<uint8_t*>(sf)[sf_byte_offset(t_out, col / 128, row_blocks)] = uint8_t(sb);
      }
    }
  }
}
cudaError_t mhc_pre_norm(const void* X, const float* pre, const float* w, int T, int D, float eps, void* y, void* q,
                         uint32_t* sf, const int* rows, cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  if (D % 128) return cudaErrorInvalidValue;
  const int per = ceil_div(D, 256 * 8), rb = ceil_div(T, 128);
  auto XX = reinterpret_cast<const __nv_bfloat16*>(X);
  auto yy = reinterpret_cast<__nv_bfloat16*>(y);
  auto qq = reinterpret_cast<uint8_t*>(q);
  if (per <= 1) cb::launch_k(mhc_pre_norm_kernel<1>, T, 256, 0, s, XX, pre, w, D, eps, yy, qq, sf, rb, rows);
  else if (per <= 2) cb::launch_k(mhc_pre_norm_kernel<2>, T, 256, 0, s, XX, pre, w, D, eps, yy, qq, sf, rb, rows);
  else if (per <= 4) cb::launch_k(mhc_pre_norm_kernel<4>, T, 256, 0, s, XX, pre, w, D, eps, yy, qq, sf, rb, rows);
  else return cudaErrorInvalidValue;
  return cudaGetLastError();
}

// Post-mix: Xn[o] = bf16(post_o * out + Σ_i comb[i][o] X_i); also sumsq[t] = Σ Xn² (for the next stats).
// X, Xn bf16 [T, 4, D] (may alias: every element is read before it is written by the same thread); out bf16 [T, D].
__global__ void mhc_post_mix_kernel(const __nv_bfloat16* X, const __nv_bfloat16* __restrict__ out,
                                    const float* __restrict__ post, const float* __restrict__ comb, int D,
                                    __nv_bfloat16* Xn, float* __restrict__ sumsq) {
  cb::pdl_entry();
  __shared__ float red[32];
  const int t = blockIdx.x;
  float pst[4], cb[16];
#pragma unroll
  for (int j = 0; j < 4; ++j) pst[j] = post[t * 4 + j];
#pragma unroll
  for (int j = 0; j < 16; ++j) cb[j] = comb[t * 16 + j];
  const __nv_bfloat16* xr = X + size_t(t) * 4 * D;
  __nv_bfloat16* xo = Xn + size_t(t) * 4 * D;
  float ss = 0.f;
  for (int col = threadIdx.x * 8; col < D; col += blockDim.x * 8) {
    float xs[4][8], ov[8];
    uint4 r0 = *reinterpret_cast<const uint4*>(out + size_t(t) * D + col);
    ov[0] = bf16_lo(r0.x); ov[1] = bf16_hi(r0.x); ov[2] = bf16_lo(r0.y); ov[3] = bf16_hi(r0.y);
    ov[4] = bf16_lo(r0.z); ov[5] = bf16_hi(r0.z); ov[6] = bf16_lo(r0.w); ov[7] = bf16_hi(r0.w);
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      uint4 raw = *reinterpret_cast<const uint4*>(xr + size_t(s) * D + col);
      xs[s][0] = bf16_lo(raw.x); xs[s][1] = bf16_hi(raw.x); xs[s][2] = bf16_lo(raw.y); xs[s][3] = bf16_hi(raw.y);
      xs[s][4] = bf16_lo(raw.z); xs[s][5] = bf16_hi(raw.z); xs[s][6] = bf16_lo(raw.w); xs[s][7] = bf16_hi(raw.w);
    }
#pragma unroll
    for (int o = 0; o < 4; ++o) {
      float r[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float a = pst[o] * ov[j];
#pragma unroll
        for (int i = 0; i < 4; ++i) a += cb[i * 4 + o] * xs[i][j];
        r[j] = __bfloat162float(__float2bfloat16_rn(a));
        ss += r[j] * r[j];
      }
      uint4 w;
      w.x = pack_bf16x2(r[0], r[1]); w.y = pack_bf16x2(r[2], r[3]);
      w.z = pack_bf16x2(r[4], r[5]); w.w = pack_bf16x2(r[6], r[7]);
      *reinterpret_cast<uint4*>(xo + size_t(o) * D + col) = w;
    }
  }
  ss = block_sum(ss, red);
  if (threadIdx.x == 0) sumsq[t] = ss;
}
cudaError_t mhc_post_mix(const void* X, const void* out, const float* post, const float* comb, int T, int D, void* Xn,
                         float* sumsq, cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  if (D % 8) return cudaErrorInvalidValue;
  cb::launch_k(mhc_post_mix_kernel, T, 256, 0, s, reinterpret_cast<const __nv_bfloat16*>(X),
                                        reinterpret_cast<const __nv_bfloat16*>(out), post, comb, D,
                                        reinterpret_cast<__nv_bfloat16*>(Xn), sumsq);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------------------------------
// Fused mHC boundary for decode-sized batches: one launch per boundary instead of post-mix, statistics GEMM,
// coefficients and pre-norm (four launches, each re-reading the residual streams).  A cluster of 8 CTAs serves TT
// tokens; CTA c owns columns [c D/8, (c+1) D/8) of every stream (128 threads, 8 columns each).
//   A  post-mix (when the previous sublayer's output is given): X_o = bf16(post_o out + Σ_i comb[i][o] X_i), written
//      in place; Σx² of the new streams (or of X as it is, for the first boundary of a step)
//   B  the next sublayer's 48 statistics (fn rows: 24 hi + 24 lo parts) over this CTA's columns of the 4 streams,
//      partial sums exchanged through distributed shared memory (every CTA sums all 8 partials itself)
//   C  coefficients: pre / post through sigmoids, comb through Sinkhorn (16 lanes, one matrix entry each)
//   D  pre-mix a = bf16(Σ_s pre_s X_s), RMSNorm with the cluster-wide Σa², bf16 output and fp8 1x128 quantisation
// The arithmetic of each step is that of the separate kernels (mhc_post_mix, mhc_coeffs, mhc_pre_norm); only the
// summation order of the reductions differs.  Reference role: the Mega-mHC boundary kernel of the reference
// (king_v10/bundle_v9/cuda_moe_prefill.py:862 sm100_mega_mhc; decode use in dec/prenorm_pair.py).
// ---------------------------------------------------------------------------------------------------------------
constexpr int kBndCluster = 8, kBndCols = 128, kBndThreads = 4 * kBndCols, kBndStats = 48, kBndWarps = kBndThreads / 32;

// Thread (k, g): column chunk k (8 columns) of this CTA's range and residual stream g.  Phase A gives each thread
// its stream's new values; phases B (statistics) and D (pre-mix over the 4 streams, from shared memory) follow.
template <int TT>
__global__ void __cluster_dims__(kBndCluster, 1, 1) __launch_bounds__(kBndThreads)
    mhc_boundary_small_kernel(__nv_bfloat16* X, int T, int D, const __nv_bfloat16* __restrict__ out,
                              const float* __restrict__ post_in, const float* __restrict__ comb_in,
                              const __nv_bfloat16* __restrict__ fn, const float* __restrict__ base,
                              const float* __restrict__ scale, int iters, float hc_eps, float rms_eps,
                              const float* __restrict__ w, __nv_bfloat16* __restrict__ y, uint8_t* __restrict__ q,
                              uint32_t* __restrict__ sf, int row_blocks, float* __restrict__ pre_out,
                              float* __restrict__ post_out, float* __restrict__ comb_out) {
  // the statistics weights (fn) do not depend on the previous kernel: the first token group's CTAs request their
  // column slice of all 48 rows x 4 streams into L2 before waiting for it
  if (blockIdx.y == 0) {
    const int cr = int(cluster_ctarank()), Dcp = D / kBndCluster;
    for (int i = threadIdx.x; i < kBndStats * 4; i += kBndThreads)
      bulk_prefetch_l2(fn + size_t(i >> 2) * 4 * D + size_t(i & 3) * D + size_t(cr) * Dcp, uint32_t(Dcp) * 2);
  }
  cb::pdl_entry();
  __shared__ float xs_sm[TT][4][kBndCols * 8];                // the new streams of this CTA's columns
  __shared__ float part[kBndWarps][TT * 8];                   // per-warp partials (phase D)
  __shared__ float pall[kBndWarps][TT * (kBndStats + 1)];     // per-warp totals of the statistics, then Σx²
  __shared__ float red[TT][kBndStats + 1];                    // this CTA's stats partials + Σx² (read cluster-wide)
  __shared__ float tot[TT][kBndStats + 1];
  __shared__ float coef[TT][24];                              // pre[4], post[4], comb[16]
  __shared__ float red2[TT];
  __shared__ float nrm[TT];
  const int c = int(cluster_ctarank());
  const int Dc = D / kBndCluster;
  const int k = threadIdx.x % kBndCols, g = threadIdx.x / kBndCols;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const bool act = k * 8 < Dc;
  const int col = c * Dc + k * 8;
  const size_t FD = size_t(4) * D;
  float xg[TT][8];                                            // stream g of this thread's 8 columns, per token
  float ss[TT];
  // ---- A: post-mix of stream g (or plain read) ----
#pragma unroll
  for (int i = 0; i < TT; ++i) {
    const int t = blockIdx.y * TT + i;
    const bool live = act && t < T;
    __nv_bfloat16* xr = X + size_t(live ? t : 0) * FD;
    ss[i] = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) xg[i][j] = 0.f;
    if (out) {
      if (live) {
        float xs[4][8], ov[8];
#pragma unroll
        for (int s = 0; s < 4; ++s) {
          const uint4 raw = *reinterpret_cast<const uint4*>(xr + size_t(s) * D + col);
          xs[s][0] = bf16_lo(raw.x); xs[s][1] = bf16_hi(raw.x); xs[s][2] = bf16_lo(raw.y); xs[s][3] = bf16_hi(raw.y);
          xs[s][4] = bf16_lo(raw.z); xs[s][5] = bf16_hi(raw.z); xs[s][6] = bf16_lo(raw.w); xs[s][7] = bf16_hi(raw.w);
        }
        const uint4 r0 = *reinterpret_cast<const uint4*>(out + size_t(t) * D + col);
        ov[0] = bf16_lo(r0.x); ov[1] = bf16_hi(r0.x); ov[2] = bf16_lo(r0.y); ov[3] = bf16_hi(r0.y);
        ov[4] = bf16_lo(r0.z); ov[5] = bf16_hi(r0.z); ov[6] = bf16_lo(r0.w); ov[7] = bf16_hi(r0.w);
        const float pst = post_in[t * 4 + g];
        float cbm[4];
#pragma unroll
        for (int ii = 0; ii < 4; ++ii) cbm[ii] = comb_in[t * 16 + ii * 4 + g];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float a = pst * ov[j];
#pragma unroll
          for (int ii = 0; ii < 4; ++ii) a += cbm[ii] * xs[ii][j];
          xg[i][j] = __bfloat162float(__float2bfloat16_rn(a));
        }
      }
      __syncthreads();                       // every stream of these columns is read before any thread writes one
      if (live) {
        uint4 wv;
        wv.x = pack_bf16x2(xg[i][0], xg[i][1]); wv.y = pack_bf16x2(xg[i][2], xg[i][3]);
        wv.z = pack_bf16x2(xg[i][4], xg[i][5]); wv.w = pack_bf16x2(xg[i][6], xg[i][7]);
        *reinterpret_cast<uint4*>(xr + size_t(g) * D + col) = wv;
      }
    } else if (live) {
      const uint4 raw = *reinterpret_cast<const uint4*>(xr + size_t(g) * D + col);
      xg[i][0] = bf16_lo(raw.x); xg[i][1] = bf16_hi(raw.x); xg[i][2] = bf16_lo(raw.y); xg[i][3] = bf16_hi(raw.y);
      xg[i][4] = bf16_lo(raw.z); xg[i][5] = bf16_hi(raw.z); xg[i][6] = bf16_lo(raw.w); xg[i][7] = bf16_hi(raw.w);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      ss[i] += xg[i][j] * xg[i][j];
      xs_sm[i][g][k * 8 + j] = xg[i][j];
    }
  }
  // ---- B: statistics partials over this CTA's columns of stream g, 8 fn rows at a time ----
  for (int r0 = 0; r0 < kBndStats; r0 += 8) {
    float acc[TT][8];
#pragma unroll
    for (int i = 0; i < TT; ++i)
#pragma unroll
      for (int rr = 0; rr < 8; ++rr) acc[i][rr] = 0.f;
    if (act) {
      uint4 fv[8];
#pragma unroll
      for (int rr = 0; rr < 8; ++rr)
        fv[rr] = __ldg(reinterpret_cast<const uint4*>(fn + size_t(r0 + rr) * FD + size_t(g) * D + col));
#pragma unroll
      for (int rr = 0; rr < 8; ++rr) {
        const float f[8] = {bf16_lo(fv[rr].x), bf16_hi(fv[rr].x), bf16_lo(fv[rr].y), bf16_hi(fv[rr].y),
                            bf16_lo(fv[rr].z), bf16_hi(fv[rr].z), bf16_lo(fv[rr].w), bf16_hi(fv[rr].w)};
#pragma unroll
        for (int i = 0; i < TT; ++i)
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[i][rr] += xg[i][j] * f[j];
      }
    }
    {
      // warp totals of the TT x 8 partials in one butterfly (TT*8 - 1 + ... shuffles instead of 5 TT*8)
      constexpr int NV = TT * 8, SH = NV == 8 ? 2 : NV == 16 ? 1 : 0;
      float flat[NV];
#pragma unroll
      for (int i = 0; i < TT; ++i)
#pragma unroll
        for (int rr = 0; rr < 8; ++rr) flat[i * 8 + rr] = acc[i][rr];
      const float v = warp_sum_many<NV>(flat, lane);
      if ((lane & ((1 << SH) - 1)) == 0) {
        const int idx = lane >> SH;                          // = token * 8 + row within the group
        pall[wid][(idx >> 3) * kBndStats + r0 + (idx & 7)] = v;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < TT; ++i) {
    const float v = warp_sum(ss[i]);
    if (lane == 0) pall[wid][TT * kBndStats + i] = v;
  }
  __syncthreads();                                           // one barrier for all 48 statistics and Σx²
  for (int e = threadIdx.x; e < TT * (kBndStats + 1); e += kBndThreads) {
    float v = 0.f;
#pragma unroll
    for (int ww = 0; ww < kBndWarps; ++ww) v += pall[ww][e];
    if (e < TT * kBndStats) red[e / kBndStats][e % kBndStats] = v;
    else red[e - TT * kBndStats][kBndStats] = v;
  }
  cluster_sync();                                            // every CTA's partials are visible cluster-wide
  for (int e = threadIdx.x; e < TT * (kBndStats + 1); e += kBndThreads) {
    const uint32_t a = smem_u32(&red[0][0] + e);
    float v = 0.f;
#pragma unroll
    for (int cc = 0; cc < kBndCluster; ++cc) {
      float x;
      asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(x) : "r"(mapa_shared(a, uint32_t(cc))));
      v += x;
    }
    (&tot[0][0])[e] = v;
  }
  __syncthreads();
  // ---- C: coefficients (warp i: token i; lanes 0-15 hold comb[lane / 4][lane % 4]) ----
  if (wid < TT) {
    const int i = wid;
    const float rsq = rsqrtf(tot[i][kBndStats] / float(FD) + rms_eps);
    if (lane < 4) {
      const float m0 = (tot[i][lane] + tot[i][24 + lane]) * rsq;
      const float m1 = (tot[i][4 + lane] + tot[i][28 + lane]) * rsq;
      coef[i][lane] = 1.f / (1.f + expf(-(m0 * scale[0] + base[lane]))) + hc_eps;
      coef[i][4 + lane] = 2.f / (1.f + expf(-(m1 * scale[1] + base[4 + lane])));
    }
    const int e = lane & 15;
    float cv = (tot[i][8 + e] + tot[i][32 + e]) * rsq * scale[2] + base[8 + e];
    float mx = fmaxf(cv, __shfl_xor_sync(0xffffffffu, cv, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    cv = expf(cv - mx);
    float s = cv + __shfl_xor_sync(0xffffffffu, cv, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    cv = cv / s + hc_eps;
    s = cv + __shfl_xor_sync(0xffffffffu, cv, 4);             // column sums
    s += __shfl_xor_sync(0xffffffffu, s, 8);
    cv /= (s + hc_eps);
    for (int it = 1; it < iters; ++it) {
      s = cv + __shfl_xor_sync(0xffffffffu, cv, 1);
      s += __shfl_xor_sync(0xffffffffu, s, 2);
      cv /= (s + hc_eps);
      s = cv + __shfl_xor_sync(0xffffffffu, cv, 4);
      s += __shfl_xor_sync(0xffffffffu, s, 8);
      cv /= (s + hc_eps);
    }
    if (lane < 16) coef[i][8 + lane] = cv;
    __syncwarp();
    const int t = blockIdx.y * TT + i;
    if (c == 0 && t < T && lane < 24) {
      const float v = coef[i][lane];
      if (lane < 4) pre_out[t * 4 + lane] = v;
      else if (lane < 8) post_out[t * 4 + lane - 4] = v;
      else comb_out[t * 16 + lane - 8] = v;
    }
  }
  __syncthreads();
  // ---- D: pre-mix of the 4 streams (thread group g < TT: token g), cluster-wide RMSNorm, bf16 + fp8 outputs ----
  const int it = g;                                          // token of this thread group in phase D
  float av[8];
  if (it < TT) {
    float s2 = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float a = 0.f;
#pragma unroll
      for (int s = 0; s < 4; ++s) a += coef[it][s] * xs_sm[it][s][k * 8 + j];
      av[j] = __bfloat162float(__float2bfloat16_rn(a));
      s2 += av[j] * av[j];
    }
    s2 = warp_sum(act ? s2 : 0.f);
    if (lane == 0) part[wid][0] = s2;
  }
  __syncthreads();
  if (threadIdx.x < TT) {
    float v = 0.f;
#pragma unroll
    for (int ww = 0; ww < kBndCols / 32; ++ww) v += part[threadIdx.x * (kBndCols / 32) + ww][0];
    red2[threadIdx.x] = v;
  }
  cluster_sync();
  if (threadIdx.x < TT) {
    const uint32_t a = smem_u32(&red2[threadIdx.x]);
    float v = 0.f;
#pragma unroll
    for (int cc = 0; cc < kBndCluster; ++cc) {
      float x;
      asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(x) : "r"(mapa_shared(a, uint32_t(cc))));
      v += x;
    }
    nrm[threadIdx.x] = rsqrtf(v / float(D) + rms_eps);
  }
  __syncthreads();
  if (it < TT) {
    const int t = blockIdx.y * TT + it;
    float amax = 0.f;
    if (act) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        av[j] = __bfloat162float(__float2bfloat16_rn(av[j] * nrm[it] * w[col + j]));
        amax = fmaxf(amax, fabsf(av[j]));
      }
      if (y && t < T) {
        uint4 o;
        o.x = pack_bf16x2(av[0], av[1]); o.y = pack_bf16x2(av[2], av[3]);
        o.z = pack_bf16x2(av[4], av[5]); o.w = pack_bf16x2(av[6], av[7]);
        *reinterpret_cast<uint4*>(y + size_t(t) * D + col) = o;
      }
    }
    if (q) {                                                 // 16 threads = one 128-column block
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      const uint32_t sb = ue8m0_for_amax(amax);
      const float inv = ue8m0_inv(sb);
      if (act && t < T) {
        uint2 wq;
        wq.x = pack_fp8x4(av[0] * inv, av[1] * inv, av[2] * inv, av[3] * inv);
        wq.y = pack_fp8x4(av[4] * inv, av[5] * inv, av[6] * inv, av[7] * inv);
        *reinterpret_cast<uint2*>(q + size_t(t) * D + col) = wq;
        if ((k & 15) == 0) reinterpret_cast<uint8_t*>(sf)[sf_byte_offset(t, col / 128, row_blocks)] = uint8_t(sb);
      }
    }
  }
  cluster_sync();                                            // no CTA leaves while a peer still reads its partials
}

cudaError_t mhc_boundary_small(void* X, int T, int D, const void* out, const float* post_in, const float* comb_in,
                               const void* fn, const float* base, const float* scale, int iters, float hc_eps,
                               float rms_eps, const float* w, void* y, void* q, uint32_t* sf, float* pre_out,
                               float* post_out, float* comb_out, cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  const int Dc = D / kBndCluster;
  if (D % (kBndCluster * 128) || Dc > kBndCols * 8 || (out && (!post_in || !comb_in))) return cudaErrorInvalidValue;
  constexpr int TT = 2;
  cb::launch_k(mhc_boundary_small_kernel<TT>, dim3(kBndCluster, ceil_div(T, TT)), kBndThreads, 0, s,
               reinterpret_cast<__nv_bfloat16*>(X), T, D, reinterpret_cast<const __nv_bfloat16*>(out), post_in,
               comb_in, reinterpret_cast<const __nv_bfloat16*>(fn), base, scale, iters, hc_eps, rms_eps, w,
               reinterpret_cast<__nv_bfloat16*>(y), reinterpret_cast<uint8_t*>(q), sf, ceil_div(T, 128), pre_out,
               post_out, comb_out);
  return cudaGetLastError();
}

// Embedding into hc streams: X[t, s, :] = E[ids[t]] for all s; sumsq[t] = hc * Σ E².  Rows of the table outside
// [row_lo, row_lo + rows) are skipped (vocab-parallel shard) and written as zeros.
__global__ void embed_hc_kernel(const __nv_bfloat16* __restrict__ table, int row_lo, int rows,
                                const int* __restrict__ ids, int D, int hc, __nv_bfloat16* __restrict__ X,
                                float* __restrict__ sumsq) {
  cb::pdl_entry();
  __shared__ float red[32];
  const int t = blockIdx.x;
  const int id = ids[t] - row_lo;
  const bool mine = id >= 0 && id < rows;
  float ss = 0.f;
  for (int col = threadIdx.x * 8; col < D; col += blockDim.x * 8) {
    uint4 raw = mine ? *reinterpret_cast<const uint4*>(table + size_t(id) * D + col) : make_uint4(0, 0, 0, 0);
    ss += bf16_lo(raw.x) * bf16_lo(raw.x) + bf16_hi(raw.x) * bf16_hi(raw.x) + bf16_lo(raw.y) * bf16_lo(raw.y) +
          bf16_hi(raw.y) * bf16_hi(raw.y) + bf16_lo(raw.z) * bf16_lo(raw.z) + bf16_hi(raw.z) * bf16_hi(raw.z) +
          bf16_lo(raw.w) * bf16_lo(raw.w) + bf16_hi(raw.w) * bf16_hi(raw.w);
    for (int s = 0; s < hc; ++s) *reinterpret_cast<uint4*>(X + (size_t(t) * hc + s) * D + col) = raw;
  }
  if (sumsq) {
    ss = block_sum(ss, red);
    if (threadIdx.x == 0) sumsq[t] = ss * hc;
  }
}
cudaError_t embed_hc(const void* table, int row_lo, int rows, const int* ids, int T, int D, int hc, void* X,
                     float* sumsq, cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  cb::launch_k(embed_hc_kernel, T, 128, 0, s, reinterpret_cast<const __nv_bfloat16*>(table), row_lo, rows, ids, D, hc,
                                    reinterpret_cast<__nv_bfloat16*>(X), sumsq);
  return cudaGetLastError();
}

// Row sum of squares of bf16 rows (length n): used where the producer of X did not emit it.
__global__ void row_sumsq_kernel(const __nv_bfloat16* __restrict__ x, int64_t n, float* __restrict__ out) {
  cb::pdl_entry();
  __shared__ float red[32];
  const int t = blockIdx.x;
  float ss = 0.f;
  for (int64_t c = threadIdx.x * 8; c < n; c += blockDim.x * 8) {
    uint4 raw = *reinterpret_cast<const uint4*>(x + size_t(t) * n + c);
    ss += bf16_lo(raw.x) * bf16_lo(raw.x) + bf16_hi(raw.x) * bf16_hi(raw.x) + bf16_lo(raw.y) * bf16_lo(raw.y) +
          bf16_hi(raw.y) * bf16_hi(raw.y) + bf16_lo(raw.z) * bf16_lo(raw.z) + bf16_hi(raw.z) * bf16_hi(raw.z) +
          bf16_lo(raw.w) * bf16_lo(raw.w) + bf16_hi(raw.w) * bf16_hi(raw.w);
  }
  ss = block_sum(ss, red);
  if (threadIdx.x == 0) out[t] = ss;
}
cudaError_t row_sumsq(const void* x, int T, int64_t n, float* out, cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  if (n % 8) return cudaErrorInvalidValue;
  cb::launch_k(row_sumsq_kernel, T, 256, 0, s, reinterpret_cast<const __nv_bfloat16*>(x), n, out);
  return cudaGetLastError();
}

// SwiGLU on a bf16 [T, 2I] tensor whose halves are (gate | up) -> bf16 [T, I].
__global__ void silu_mul_kernel(const __nv_bfloat16* __restrict__ gu, int I, float limit,
                                __nv_bfloat16* __restrict__ out) {
  cb::pdl_entry();
  const int t = blockIdx.x;
  for (int c = threadIdx.x; c < I; c += blockDim.x) {
    float g = __bfloat162float(gu[size_t(t) * 2 * I + c]);
    float u = __bfloat162float(gu[size_t(t) * 2 * I + I + c]);
    if (limit > 0.f) { g = fminf(g, limit); u = fminf(fmaxf(u, -limit), limit); }
    out[size_t(t) * I + c] = __float2bfloat16_rn(g / (1.f + expf(-g)) * u);
  }
}
cudaError_t silu_mul(const void* gu, int T, int I, float limit, void* out, cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  cb::launch_k(silu_mul_kernel, T, 256, 0, s, reinterpret_cast<const __nv_bfloat16*>(gu), I, limit,
                                    reinterpret_cast<__nv_bfloat16*>(out));
  return cudaGetLastError();
}

}  // namespace cb


namespace cb {

// DSA indexer key / weight post-processing of the fused [wk | weights_proj] projection, one launch per call:
// k[t] = RoPE(bf16(LayerNorm(kw[t, :Di]) * ln_w + ln_b)) on dims [0, dr) (interleaved pairs, the bf16 values rotated
// in fp32 and rounded again), w[t, h] = kw[t, Di + h] * wscale.  One CTA of Di threads per token (Di <= 1024, even).
__global__ void indexer_kw_post_kernel(const float* __restrict__ kw, int ld, int Di, int Hi,
                                       const float* __restrict__ ln_w, const float* __restrict__ ln_b, float eps,
                                       const float* __restrict__ cos_sin, const int* __restrict__ pos, int dr,
                                       float wscale, __nv_bfloat16* __restrict__ k, float* __restrict__ w) {
  cb::pdl_entry();
  __shared__ float red[32];
  const int t = blockIdx.x, d = threadIdx.x;
  const float* row = kw + size_t(t) * ld;
  const float x = row[d];
  const float mean = block_sum(x, red) / float(Di);
  const float dx = x - mean;
  const float var = block_sum(dx * dx, red) / float(Di);
  float y = __bfloat162float(__float2bfloat16_rn(dx * rsqrtf(var + eps) * ln_w[d] + ln_b[d]));
  const float other = __shfl_xor_sync(0xffffffffu, y, 1);    // the pair partner (pairs never straddle a warp)
  if (d < dr) {
    const int p = pos[t];
    const float c = cos_sin[size_t(p) * dr + (d & ~1)], s = cos_sin[size_t(p) * dr + (d & ~1) + 1];
    y = (d & 1) ? other * s + y * c : y * c - other * s;
  }
  k[size_t(t) * Di + d] = __float2bfloat16_rn(y);
  for (int h = d; h < Hi; h += blockDim.x) w[size_t(t) * Hi + h] = row[Di + h] * wscale;
}

cudaError_t indexer_kw_post(const float* kw, int ld, int T, int Di, int Hi, const float* ln_w, const float* ln_b,
                            float eps, const float* cos_sin, const int* pos, int dr, float wscale, void* k, float* w,
                            cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  if (Di % 32 || Di > 1024 || dr % 2 || dr > Di) return cudaErrorInvalidValue;
  cb::launch_k(indexer_kw_post_kernel, T, Di, 0, s, kw, ld, Di, Hi, ln_w, ln_b, eps, cos_sin, pos, dr, wscale,
               reinterpret_cast<__nv_bfloat16*>(k), w);
  return cudaGetLastError();
}

}  // namespace cb
