// Host side of the tcgen05 GEMMs: TMA tensor-map encoding, instantiation choice, launch.
#include <cudaTypedefs.h>
#include <mutex>
#include "gemm.cuh"
#include "gemm_pair.cuh"
#include <cstdlib>
#include "small_ops.h"

namespace cb {

static PFN_cuTensorMapEncodeTiled_v12000 tmap_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D K-major tile map: [rows, inner] with 128-byte swizzled boxes of (box_inner x box_rows).
bool make_tmap_2d(CUtensorMap* m, const void* ptr, CUtensorMapDataType dt, int elem_bytes, uint64_t inner,
                  uint64_t rows, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows,
                  CUtensorMapSwizzle swz) {
  auto fn = tmap_encode_fn();
  if (!fn) return false;
  if ((reinterpret_cast<uintptr_t>(ptr) & 15) || (row_stride_bytes & 15)) return false;
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  (void)elem_bytes;
  return r == CUDA_SUCCESS;
}

// Scale-factor tiles as a 2-D tensor of uint32: [rows = K/512 * row_blocks][128 words], one box = `box_rows` tiles.
static bool make_tmap_sf(CUtensorMap* m, const uint32_t* sf, uint64_t rows, uint32_t box_rows) {
  auto fn = tmap_encode_fn();
  if (!fn || (reinterpret_cast<uintptr_t>(sf) & 15)) return false;
  cuuint64_t dims[2] = {128, rows};
  cuuint64_t strides[1] = {512};
  cuuint32_t box[2] = {128, box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint32_t*>(sf), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// bf16 pair-GEMM epilogue: the output tile is staged in shared memory and stored row-contiguous (one fewer
// pipeline stage).  Measured on B200 (CUDA events): 8192x8192x7168 2954 -> 3183 TFLOP/s, 16384x7168x2048
// 2225 -> 2882 TFLOP/s, 16k-token MoE layer 5.65 -> 5.17 ms.  CARBON_GEMM_ROWS=0 restores row-per-lane stores.
static bool gemm_rows_epilogue() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("CARBON_GEMM_ROWS");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

// Launch of the pair-tile GEMM: clusters of PAIR CTAs, one persistent cluster per co-resident slot.
template <int KIND, int EPI, int PAIR, int ST>
static cudaError_t launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tsa,
                               const CUtensorMap& tsb, const GemmParams& p, int max_units, int num_sms,
                               cudaStream_t s) {
  using C = PairCfg<KIND, PAIR, EPI>;
  constexpr int smem = gemm_pair_smem_bytes<KIND, PAIR, ST, EPI>();
  static_assert(smem <= 227 * 1024, "pair GEMM shared memory above the per-CTA limit");
  auto kern = gemm_pair_kernel<KIND, EPI, PAIR, ST>;
  static int resident = 0;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = PAIR; attr[0].val.clusterDim.y = 1; attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;     // see cb::pdl_entry
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(C::kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  {
    cudaError_t e = cb::smem_optin(kern, smem);
    if (e != cudaSuccess) return e;
  }
  if (!resident) {
    int n = 0;
    cfg.gridDim = dim3((num_sms / PAIR) * PAIR);
    if (PAIR > 1 && cudaOccupancyMaxActiveClusters(&n, kern, &cfg) == cudaSuccess && n > 0)
      resident = n < num_sms / PAIR ? n : num_sms / PAIR;
    else
      resident = num_sms / PAIR;
    cudaGetLastError();
  }
  const int units = max_units < resident ? max_units : resident;
  if (units <= 0) return cudaSuccess;
  cfg.gridDim = dim3(units * PAIR);
  cfg.numAttrs = cb::pdl_enabled() ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kern, ta, tb, tsa, tsb, p);
}

__global__ void splitk_reduce_kernel(const float* __restrict__ part, int splits, int M, int N, int ldo,
                                     float* __restrict__ out) {
  cb::pdl_entry();
  const int64_t total = int64_t(M) * N;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int r = int(i / N), c = int(i % N);
    float acc = 0.f;
    for (int sp = 0; sp < splits; ++sp) acc += part[(size_t(sp) * M + r) * ldo + c];
    out[size_t(r) * ldo + c] = acc;
  }
}

static cudaError_t splitk_reduce(const float* part, int splits, int M, int N, int ldo, float* out, cudaStream_t s) {
  const int64_t total = int64_t(M) * N;
  const int blocks = int(total / 256 + 1 < 1024 ? total / 256 + 1 : 1024);
  cb::launch_k(splitk_reduce_kernel, blocks, 256, 0, s, part, splits, M, N, ldo, out);
  return cudaGetLastError();
}

// Sum of the float4 at p in `splits` consecutive slabs (stride `slab` floats), added in split order; the loads of up
// to U splits are issued before any is used, so a reduction costs one memory latency per U splits, not one per split.
template <int U = 8>
CB_DEVICE float4 splits_sum4(const float* __restrict__ p, size_t slab, int splits) {
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int sp0 = 0; sp0 < splits; sp0 += U) {
    float4 v[U];
#pragma unroll
    for (int j = 0; j < U; ++j)
      if (sp0 + j < splits) v[j] = *reinterpret_cast<const float4*>(p + size_t(sp0 + j) * slab);
#pragma unroll
    for (int j = 0; j < U; ++j)
      if (sp0 + j < splits) { acc.x += v[j].x; acc.y += v[j].y; acc.z += v[j].z; acc.w += v[j].w; }
  }
  return acc;
}

// Split-K partial slabs [splits][M][N] (fp32) -> output.  MODE 0: fp32, MODE 1: bf16; 4 columns per thread.
template <int MODE>
__global__ void splitk_reduce_out_kernel(const float* __restrict__ part, int splits, int M, int N, void* out,
                                         int ldo) {
  cb::pdl_entry();
  const int64_t total4 = int64_t(M) * (N / 4);
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total4; i += int64_t(gridDim.x) * blockDim.x) {
    const int r = int(i / (N / 4)), c = int(i % (N / 4)) * 4;
    const float4 acc = splits_sum4(part + size_t(r) * N + c, size_t(M) * N, splits);
    if (MODE == 0) {
      *reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + size_t(r) * ldo + c) = acc;
    } else {
      uint2 w = make_uint2(pack_bf16x2(acc.x, acc.y), pack_bf16x2(acc.z, acc.w));
      *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(out) + size_t(r) * ldo + c) = w;
    }
  }
}

// Split-K partials of an interleaved gate/up GEMM (N = 2I, 128-column chunks gate|up) -> SwiGLU -> fp8 + SF tiles,
// exactly the SwiGLU epilogue's arithmetic.  One warp per (row, 128 output columns), 4 outputs per lane.
CB_DEVICE void swiglu_reduce_row(const float* __restrict__ part, int splits, int M, int N, float limit,
                                 uint8_t* __restrict__ out, int ldo, uint32_t* __restrict__ out_sf, int sf_row_blocks,
                                 int row, int g, int lane) {
  float a[4];
  float amax = 0.f;
  // gate and up sums of this lane's 4 columns (float4 loads, every split's load in flight before the adds)
  const float* pr = part + size_t(row) * N + 256 * g + 4 * lane;
  const float4 g4 = splits_sum4<4>(pr, size_t(M) * N, splits);
  const float4 u4 = splits_sum4<4>(pr + 128, size_t(M) * N, splits);
  const float gs[4] = {g4.x, g4.y, g4.z, g4.w}, us[4] = {u4.x, u4.y, u4.z, u4.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float gv = gs[i], uv = us[i];
    if (limit > 0.f) { gv = fminf(gv, limit); uv = fminf(fmaxf(uv, -limit), limit); }
    a[i] = gv / (1.f + __expf(-gv)) * uv;
    amax = fmaxf(amax, fabsf(a[i]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const uint32_t sb = ue8m0_for_amax(amax);
  const float inv = ue8m0_inv(sb);
  *reinterpret_cast<uint32_t*>(out + size_t(row) * ldo + 128 * g + 4 * lane) =
      pack_fp8x4(a[0] * inv, a[1] * inv, a[2] * inv, a[3] * inv);
  if (lane == 0) {
    const int rb = row / 128, r = row % 128;
    uint8_t* sf = reinterpret_cast<uint8_t*>(out_sf) +
                  ((size_t(g >> 2) * sf_row_blocks + rb) * 128 + (r % 32) * 4 + (r / 32)) * 4 + (g & 3);
    *sf = uint8_t(sb);
  }
}

// Dense calls (row_valid == nullptr): warps stride over every (row, column group).  Grouped calls (a row_valid map,
// the used 128-row blocks counted on the device): one CTA per 128-row block; CTAs past the used blocks and padding
// rows return at once, so a decode call touches only its few routed rows out of the padded capacity.
__global__ void __launch_bounds__(512) splitk_reduce_swiglu_kernel(const float* __restrict__ part, int splits, int M,
                                                                   int N, float limit,
                                            uint8_t* __restrict__ out, int ldo, uint32_t* __restrict__ out_sf,
                                            int sf_row_blocks, const int* __restrict__ row_valid,
                                            const int* __restrict__ n_blocks) {
  cb::pdl_entry();
  const int chunks = N / 256;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  if (row_valid) {
    if (n_blocks && int(blockIdx.x) >= n_blocks[0]) return;
    // the block's rows that carry a token (padding rows of an expert segment are never read back), then every
    // (row, column group) pair of them spread over the warps
    __shared__ int rows_s[128];
    __shared__ int n_s;
    if (threadIdx.x == 0) n_s = 0;
    __syncthreads();
    for (int rr = threadIdx.x; rr < 128; rr += blockDim.x) {
      const int row = blockIdx.x * 128 + rr;
      if (row < M && row_valid[row] >= 0) rows_s[atomicAdd(&n_s, 1)] = row;
    }
    __syncthreads();
    const int n = n_s;
    for (int item = warp; item < n * chunks; item += nwarps)
      swiglu_reduce_row(part, splits, M, N, limit, out, ldo, out_sf, sf_row_blocks, rows_s[item / chunks],
                        item % chunks, lane);
    return;
  }
  const int rows = n_blocks ? min(M, n_blocks[0] * 128) : M;
  const int nw = gridDim.x * nwarps;
  for (int wg = blockIdx.x * nwarps + warp; wg < rows * chunks; wg += nw)
    swiglu_reduce_row(part, splits, M, N, limit, out, ldo, out_sf, sf_row_blocks, wg / chunks, wg % chunks, lane);
}

// K splits for a dense fp8 GEMM whose output tiles cannot occupy the SMs (decode-sized M): whole 512-wide scale
// groups per split, enough splits to give every SM a tile.  1 = no split.
int gemm_fp8_splits(int M, int N, int K, bool grouped, int epi, int num_sms) {
  if (grouped || M > 256) return 1;
  const int tiles = ceil_div(M, 128) * ceil_div(N, 128);
  const int kgroups = ceil_div(K, 512);
  if (tiles * 2 > num_sms || kgroups < 2) return 1;
  // the persistent grid runs tiles*splits work items on num_sms CTAs: pick the split count whose last wave is
  // fullest (ties -> fewer splits, less partial traffic)
  int best = 1;
  float best_eff = 0.f;
  for (int sp = 2; sp <= kgroups && sp <= 32; ++sp) {
    const int items = tiles * sp;
    const int waves = ceil_div(items, num_sms);
    const float eff = float(items) / float(waves * num_sms);
    if (eff > best_eff + 0.02f) { best = sp; best_eff = eff; }
  }
  (void)epi;
  return best;
}

template <int KIND, int EPI, int BN, int ST, int ACC>
static cudaError_t launch(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, int max_tiles,
                          int num_sms, cudaStream_t s) {
  constexpr int smem = gemm_smem_bytes<KIND, BN, ST>();
  auto kern = gemm_tc_kernel<KIND, EPI, BN, ST, ACC>;
  {
    cudaError_t e = cb::smem_optin(kern, smem);
    if (e != cudaSuccess) return e;
  }
  const int grid = max_tiles < num_sms ? max_tiles : num_sms;
  if (grid <= 0) return cudaSuccess;
  cb::launch_k(kern, grid, 256, smem, s, ta, tb, p);
  return cudaGetLastError();
}

cudaError_t gemm_fp8(const void* A, const void* B, const uint32_t* sfa, const uint32_t* sfb, int M, int N, int K,
                     int Nb, void* out, int ldo, int epi, uint32_t* out_sf, float swiglu_limit,
                     const int* m_block_expert, const int* num_m_blocks_dev, int max_m_blocks, int* status,
                     int num_sms, cudaStream_t s, int pair, float* work, const int* row_valid) {
  if (M <= 0 || N <= 0) return cudaSuccess;
  if (K % 128 || N % 16) return cudaErrorInvalidValue;
  // pair-tile kernel: dense prefill-sized GEMMs, and grouped GEMMs whose expert segments are 256-row aligned
  // (the caller says so with pair = 1); the 128-row kernel keeps decode-sized and fp32-output GEMMs
  const bool use_pair = epi != GEMM_OUT_F32 && (pair == 1 || (pair < 0 && !m_block_expert && M >= 512));
  if (use_pair) {
    if (N % 256 && (m_block_expert || epi == GEMM_OUT_SWIGLU_FP8)) return cudaErrorInvalidValue;
    if (m_block_expert && (max_m_blocks & 1)) return cudaErrorInvalidValue;
    CUtensorMap ta, tb, tsa, tsb;
    if (!make_tmap_2d(&ta, A, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, M, K, 128, 128, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_tmap_2d(&tb, B, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, Nb, K, 128, 64, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_tmap_sf(&tsa, sfa, uint64_t(ceil_div(K, 512)) * ceil_div(M, 128), 1) ||
        !make_tmap_sf(&tsb, sfb, uint64_t(ceil_div(K, 512)) * ceil_div(Nb, 128), 2))
      return cudaErrorInvalidValue;
    GemmParams p{};
    p.M = M; p.N = N; p.K = K;
    p.sfa = sfa; p.sfb = sfb;
    p.sfa_row_blocks = ceil_div(M, 128);
    p.sfb_row_blocks = ceil_div(Nb, 128);
    p.out = out; p.ldo = ldo; p.out_sf = out_sf; p.swiglu_limit = swiglu_limit;
    p.m_block_expert = m_block_expert; p.num_m_blocks_dev = num_m_blocks_dev; p.status = status;
    const int units = (m_block_expert ? max_m_blocks / 2 : ceil_div(M, 256)) * ceil_div(N, 256);
    if (epi == GEMM_OUT_SWIGLU_FP8)
      return launch_pair<KIND_MXF8, EPI_SWIGLU_FP8, 2, 6>(ta, tb, tsa, tsb, p, units, num_sms, s);
    if (gemm_rows_epilogue() && ldo % 8 == 0 && N % 8 == 0)      // row-contiguous staged stores (5 stages)
      return launch_pair<KIND_MXF8, EPI_BF16_ROWS, 2, 5>(ta, tb, tsa, tsb, p, units, num_sms, s);
    return launch_pair<KIND_MXF8, EPI_BF16, 2, 6>(ta, tb, tsa, tsb, p, units, num_sms, s);
  }
  if (pair == 2 && m_block_expert) {
    // decode-sized grouped GEMM (a few rows per expert): pure weight streaming.  The double-buffered 128-wide fp32
    // kernel streams best; a SwiGLU output is then formed by a row-wise pass.  Padding rows are never written.
    if (epi == GEMM_OUT_SWIGLU_FP8 && (!work || N % 256)) return cudaErrorInvalidValue;
    CUtensorMap ta, tb;
    if (!make_tmap_2d(&ta, A, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, M, K, 128, 128, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_tmap_2d(&tb, B, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, Nb, K, 128, 128, CU_TENSOR_MAP_SWIZZLE_128B))
      return cudaErrorInvalidValue;
    GemmParams p{};
    p.M = M; p.N = N; p.K = K;
    p.sfa = sfa; p.sfb = sfb;
    p.sfa_row_blocks = ceil_div(M, 128);
    p.sfb_row_blocks = ceil_div(Nb, 128);
    p.m_block_expert = m_block_expert; p.num_m_blocks_dev = num_m_blocks_dev; p.status = status;
    p.row_valid = row_valid;
    const int max_tiles = max_m_blocks * ceil_div(N, 128);
    if (epi == GEMM_OUT_SWIGLU_FP8) {
      p.out = work; p.ldo = N;
      cudaError_t e = launch<KIND_MXF8, EPI_F32, 128, 6, 2>(ta, tb, p, max_tiles, num_sms, s);
      if (e != cudaSuccess) return e;
      // one CTA per 128-row block when a row map is given (grouped call), else warps striding over the rows
      const int grid = row_valid ? ceil_div(M, 128) : min(ceil_div(M * (N / 256), 8), num_sms * 8);
      // 16 warps per row block: a decode block's few rows x 16 column groups are one or two items per warp, so
      // their loads (partials mostly evicted from L2 by the weight stream) are in flight together
      cb::launch_k(splitk_reduce_swiglu_kernel, grid, row_valid ? 512 : 256, 0, s, work, 1, M, N, swiglu_limit,
                                                                     reinterpret_cast<uint8_t*>(out), ldo, out_sf,
                                                                     ceil_div(M, 128), row_valid, num_m_blocks_dev);
      return cudaGetLastError();
    }
    p.out = out; p.ldo = ldo;
    if (epi == GEMM_OUT_F32) return launch<KIND_MXF8, EPI_F32, 128, 6, 2>(ta, tb, p, max_tiles, num_sms, s);
    return launch<KIND_MXF8, EPI_BF16, 128, 6, 2>(ta, tb, p, max_tiles, num_sms, s);
  }
  const int splits = work ? gemm_fp8_splits(M, N, K, m_block_expert != nullptr, epi, num_sms) : 1;
  if (splits > 1) {
    // partial slabs of K ranges (fp32, one 128x128 tile per CTA), then an ordered reduction into the output
    CUtensorMap ta, tb;
    if (!make_tmap_2d(&ta, A, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, M, K, 128, 128, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_tmap_2d(&tb, B, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, Nb, K, 128, 128, CU_TENSOR_MAP_SWIZZLE_128B))
      return cudaErrorInvalidValue;
    GemmParams p{};
    p.M = M; p.N = N; p.K = K;
    p.sfa = sfa; p.sfb = sfb;
    p.sfa_row_blocks = ceil_div(M, 128);
    p.sfb_row_blocks = ceil_div(Nb, 128);
    p.out = work; p.ldo = N; p.status = status;
    p.k_splits = splits;
    const int tiles = ceil_div(M, 128) * ceil_div(N, 128);
    cudaError_t e = launch<KIND_MXF8, EPI_F32, 128, 6, 2>(ta, tb, p, tiles * splits, num_sms, s);
    if (e != cudaSuccess) return e;
    const int nk_total = ceil_div(K, 128), nk_per = ceil_div(ceil_div(nk_total, splits), 4) * 4;
    const int used = ceil_div(nk_total, nk_per);
    if (epi == GEMM_OUT_SWIGLU_FP8) {
      const int warps = M * (N / 256);
      cb::launch_k(splitk_reduce_swiglu_kernel, min(ceil_div(warps, 8), num_sms * 8), 256, 0, s, work, used, M, N,
                   swiglu_limit,
                                                                     reinterpret_cast<uint8_t*>(out), ldo, out_sf,
                                                                     ceil_div(M, 128), nullptr, nullptr);
    } else {
      const int64_t total4 = int64_t(M) * (N / 4);
      const int blocks = int(total4 / 256 + 1 < 1024 ? total4 / 256 + 1 : 1024);
      if (epi == GEMM_OUT_F32) cb::launch_k(splitk_reduce_out_kernel<0>, blocks, 256, 0, s, work, used, M, N, out, ldo);
      else cb::launch_k(splitk_reduce_out_kernel<1>, blocks, 256, 0, s, work, used, M, N, out, ldo);
    }
    return cudaGetLastError();
  }
  const int BN = (epi == GEMM_OUT_SWIGLU_FP8) ? 256 : 128;
  if (m_block_expert && (N % BN)) return cudaErrorInvalidValue;
  if (BN == 256 && (Nb % 256)) return cudaErrorInvalidValue;  // SF tiles of a 256-row B block must exist
  CUtensorMap ta, tb;
  if (!make_tmap_2d(&ta, A, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, M, K, 128, 128, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap_2d(&tb, B, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, Nb, K, 128, BN, CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  GemmParams p{};
  p.M = M; p.N = N; p.K = K;
  p.sfa = sfa; p.sfb = sfb;
  p.sfa_row_blocks = ceil_div(M, 128);
  p.sfb_row_blocks = ceil_div(Nb, 128);
  p.out = out; p.ldo = ldo; p.out_sf = out_sf; p.swiglu_limit = swiglu_limit;
  p.m_block_expert = m_block_expert; p.num_m_blocks_dev = num_m_blocks_dev; p.status = status;
  const int mblocks = m_block_expert ? max_m_blocks : ceil_div(M, 128);
  const int max_tiles = mblocks * ceil_div(N, BN);
  if (epi == GEMM_OUT_SWIGLU_FP8) return launch<KIND_MXF8, EPI_SWIGLU_FP8, 256, 4, 1>(ta, tb, p, max_tiles, num_sms, s);
  if (epi == GEMM_OUT_F32) return launch<KIND_MXF8, EPI_F32, 128, 6, 2>(ta, tb, p, max_tiles, num_sms, s);
  return launch<KIND_MXF8, EPI_BF16, 128, 6, 2>(ta, tb, p, max_tiles, num_sms, s);
}

cudaError_t gemm_bf16(const void* A, int lda, const void* B, int ldb, int M, int N, int K, int Nb, void* out, int ldo,
                      int epi, const int* m_block_expert, const int* num_m_blocks_dev, int max_m_blocks, int* status,
                      int num_sms, cudaStream_t s, int k_splits, float* work) {
  if (M <= 0 || N <= 0) return cudaSuccess;
  if (K % 64 || N % 16) return cudaErrorInvalidValue;
  constexpr int BN = 128;
  CUtensorMap ta, tb;
  if (!make_tmap_2d(&ta, A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, M, uint64_t(lda) * 2, 64, 128,
                    CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap_2d(&tb, B, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, Nb, uint64_t(ldb) * 2, 64, BN,
                    CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  GemmParams p{};
  p.M = M; p.N = N; p.K = K;
  p.out = out; p.ldo = ldo;
  p.m_block_expert = m_block_expert; p.num_m_blocks_dev = num_m_blocks_dev; p.status = status;
  const int mblocks = m_block_expert ? max_m_blocks : ceil_div(M, 128);
  const int max_tiles = mblocks * ceil_div(N, BN);
  if (epi == GEMM_OUT_F32) {
    if (k_splits > 1) {
      // partials [k_splits, M, ldo] in `work`, then an in-order reduction into `out`
      if (m_block_expert || !work) return cudaErrorInvalidValue;
      p.k_splits = k_splits;
      p.out = work;
      const bool vec = (N % 4) == 0 && (ldo % 4) == 0;
      if (vec) p.ldo = N;                                              // dense [splits, M, N] slabs
      cudaError_t e = launch<KIND_BF16, EPI_F32, 128, 6, 2>(ta, tb, p, max_tiles * k_splits, num_sms, s);
      if (e != cudaSuccess) return e;
      const int nk_total = ceil_div(K, 64), nk_per = ceil_div(ceil_div(nk_total, k_splits), 4) * 4;
      const int used = ceil_div(nk_total, nk_per);                     // splits that own at least one k-block
      if (!vec) return splitk_reduce(work, used, M, N, ldo, reinterpret_cast<float*>(out), s);
      const int64_t total4 = int64_t(M) * (N / 4);
      const int blocks = int(total4 / 256 + 1 < 1024 ? total4 / 256 + 1 : 1024);
      cb::launch_k(splitk_reduce_out_kernel<0>, blocks, 256, 0, s, static_cast<const float*>(work), used, M, N, out,
                   ldo);
      return cudaGetLastError();
    }
    return launch<KIND_BF16, EPI_F32, 128, 6, 2>(ta, tb, p, max_tiles, num_sms, s);
  }
  return launch<KIND_BF16, EPI_BF16, 128, 6, 2>(ta, tb, p, max_tiles, num_sms, s);
}

// o_proj GEMM fused with the reduce-scatter data movement: fp8 A [M,K] x B [N,K]^T, each output row stored into its
// token owner's slot over NVLink (see EPI_BF16_SCATTER).
cudaError_t gemm_fp8_scatter(const void* A, const void* B, const uint32_t* sfa, const uint32_t* sfb, int M, int N,
                             int K, const uint64_t* scatter_ptrs, const int* bounds, int world, int my_rank,
                             int slot_rows, int* status, int num_sms, cudaStream_t s) {
  if (M <= 0 || N <= 0) return cudaSuccess;
  if (K % 128 || N % 16 || N % 8) return cudaErrorInvalidValue;
  CUtensorMap ta, tb;
  if (!make_tmap_2d(&ta, A, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, M, K, 128, 128, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap_2d(&tb, B, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, N, K, 128, 128, CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  GemmParams p{};
  p.M = M; p.N = N; p.K = K;
  p.sfa = sfa; p.sfb = sfb;
  p.sfa_row_blocks = ceil_div(M, 128);
  p.sfb_row_blocks = ceil_div(N, 128);
  p.ldo = N; p.status = status;
  p.scatter_ptrs = scatter_ptrs; p.scatter_bounds = bounds; p.scatter_world = world; p.scatter_rank = my_rank;
  p.scatter_rows = slot_rows;
  if (M >= 512) {
    CUtensorMap tb2, tsa, tsb;
    if (!make_tmap_2d(&tb2, B, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, N, K, 128, 64, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_tmap_sf(&tsa, sfa, uint64_t(ceil_div(K, 512)) * ceil_div(M, 128), 1) ||
        !make_tmap_sf(&tsb, sfb, uint64_t(ceil_div(K, 512)) * ceil_div(N, 128), 2))
      return cudaErrorInvalidValue;
    // five stages leave room for the epilogue's peer-store staging
    return launch_pair<KIND_MXF8, EPI_BF16_SCATTER, 2, 5>(ta, tb2, tsa, tsb, p, ceil_div(M, 256) * ceil_div(N, 256),
                                                        num_sms, s);
  }
  return launch<KIND_MXF8, EPI_BF16_SCATTER, 128, 6, 2>(ta, tb, p, ceil_div(M, 128) * ceil_div(N, 128), num_sms, s);
}

// Grouped expert GEMM fused with the EP combine's data movement: fp8 A [M,K] (expert-sorted received rows, 256-row
// aligned segments) x B [E*N, K]^T; each output row is stored over NVLink straight into its token's home-rank
// combine slot (see EPI_BF16_PUSH), row-contiguous from the staged epilogue.  Padding rows (row_dst < 0) are skipped.
cudaError_t gemm_fp8_push(const void* A, const void* B, const uint32_t* sfa, const uint32_t* sfb, int M, int N, int K,
                          int Nb, const int* m_block_expert, const int* num_m_blocks_dev, int max_m_blocks,
                          const int* row_dst, const uint64_t* home_ptrs, int world, int* status, int num_sms,
                          cudaStream_t s) {
  if (M <= 0 || N <= 0) return cudaSuccess;
  if (K % 128 || N % 256 || (max_m_blocks & 1) || !m_block_expert || !row_dst) return cudaErrorInvalidValue;
  CUtensorMap ta, tb, tsa, tsb;
  if (!make_tmap_2d(&ta, A, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, M, K, 128, 128, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap_2d(&tb, B, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, Nb, K, 128, 64, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap_sf(&tsa, sfa, uint64_t(ceil_div(K, 512)) * ceil_div(M, 128), 1) ||
      !make_tmap_sf(&tsb, sfb, uint64_t(ceil_div(K, 512)) * ceil_div(Nb, 128), 2))
    return cudaErrorInvalidValue;
  GemmParams p{};
  p.M = M; p.N = N; p.K = K;
  p.sfa = sfa; p.sfb = sfb;
  p.sfa_row_blocks = ceil_div(M, 128);
  p.sfb_row_blocks = ceil_div(Nb, 128);
  p.ldo = N; p.status = status;
  p.m_block_expert = m_block_expert; p.num_m_blocks_dev = num_m_blocks_dev;
  p.row_dst = row_dst; p.scatter_ptrs = home_ptrs; p.scatter_world = world;
  const int units = (max_m_blocks / 2) * ceil_div(N, 256);
  return launch_pair<KIND_MXF8, EPI_BF16_PUSH, 2, 5>(ta, tb, tsa, tsb, p, units, num_sms, s);
}

// DSA indexer logits: keys [L, Di] bf16, q [Tq*H, Di] bf16, w [Tq, H] fp32 -> logits [Tq, ldo] fp32 (causal).
cudaError_t indexer_logits(const void* keys, int L, const void* q, int Tq, int H, int Di, const float* w, float* out,
                           int ldo, bool causal, int* status, int num_sms, cudaStream_t s) {
  if (L <= 0 || Tq <= 0) return cudaSuccess;
  constexpr int BN = 256;
  if (Di % 64 || BN % H || H % 16) return cudaErrorInvalidValue;
  if ((BN / H) % 2) return cudaErrorInvalidValue;          // two epilogue halves split a tile's queries
  CUtensorMap ta, tb;
  if (!make_tmap_2d(&ta, keys, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, Di, L, uint64_t(Di) * 2, 64, 128,
                    CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap_2d(&tb, q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, Di, uint64_t(Tq) * H, uint64_t(Di) * 2, 64, 64,
                    CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  GemmParams p{};
  p.M = L; p.N = Tq * H; p.K = Di;
  p.out = out; p.ldo = ldo; p.status = status;
  p.idx_w = w; p.idx_heads = H; p.causal = causal ? 1 : 0;
  const int units = ceil_div(L, 256) * ceil_div(Tq * H, BN);
  return launch_pair<KIND_BF16, EPI_INDEXER, 2, 6>(ta, tb, ta, tb, p, units, num_sms, s);
}

// The same with fp8 e4m3 keys and queries (1x128 UE8M0 scale per row, SF-tile layout of act_quant): block-scaled
// tcgen05 MMAs at twice the bf16 rate.  keys [L, Di] fp8 + SF, q [Tq*H, Di] fp8 + SF.
cudaError_t indexer_logits_fp8(const void* keys, const uint32_t* keys_sf, int L, const void* q, const uint32_t* q_sf,
                               int Tq, int H, int Di, const float* w, float* out, int ldo, bool causal, int* status,
                               int num_sms, cudaStream_t s) {
  if (L <= 0 || Tq <= 0) return cudaSuccess;
  constexpr int BN = 256;
  if (Di % 128 || BN % H || H % 16) return cudaErrorInvalidValue;
  if ((BN / H) % 2) return cudaErrorInvalidValue;
  const int N = Tq * H;
  CUtensorMap ta, tb, tsa, tsb;
  if (!make_tmap_2d(&ta, keys, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, Di, L, Di, 128, 128, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap_2d(&tb, q, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, Di, N, Di, 128, 64, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap_sf(&tsa, keys_sf, uint64_t(ceil_div(Di, 512)) * ceil_div(L, 128), 1) ||
      !make_tmap_sf(&tsb, q_sf, uint64_t(ceil_div(Di, 512)) * ceil_div(N, 128), 2))
    return cudaErrorInvalidValue;
  GemmParams p{};
  p.M = L; p.N = N; p.K = Di;
  p.sfa = keys_sf; p.sfb = q_sf;
  p.sfa_row_blocks = ceil_div(L, 128);
  p.sfb_row_blocks = ceil_div(N, 128);
  p.out = out; p.ldo = ldo; p.status = status;
  p.idx_w = w; p.idx_heads = H; p.causal = causal ? 1 : 0;
  const int units = ceil_div(L, 256) * ceil_div(N, BN);
  return launch_pair<KIND_MXF8, EPI_INDEXER, 2, 6>(ta, tb, tsa, tsb, p, units, num_sms, s);
}

}  // namespace cb
