// Per-head matmul for decode-size batches on sm_100a:
//
//     out[t, h, n] = sum_k x[t, h, k] * w[h, n, k]        (x, w bf16; fp32 accumulation; bf16 or fp16 output)
//
// with an optional tail: out[t, h, N + j] = x[t, h, K + j] for j < tail (the absorbed MLA query
// [q_nope · W_uk | q_rope] is assembled in the same launch).
//
// Swap-AB tiling.  A decode batch has few tokens per head (T <= 256) while every head's weight block is 128 KB, so
// the weight rows take the MMA's M dimension and the tokens its N dimension: a CTA (n-block nb, head h) computes
// D[128, TB] = W_h[128 nb : 128 nb + 128, :] · X_h^T with one tcgen05 kind::f16 MMA chain (M = 128, N = TB = T rounded
// up to 16, K in 64-element steps), the accumulator in TMEM (TB fp32 columns).  No row padding to 128 tokens per
// head and no head-major staging copy: the token rows of head h are read in place through a 3-D tensor map
// (K, H, T) whose box (64, 1, TB) lands as TB swizzled 128-byte rows, and the epilogue writes the token-major
// output directly (lane = output column n, TMEM column = token t; a warp stores 32 consecutive n of one token).
//
// Roles (128 threads): warp 0 TMA producer, warp 1 MMA issuer, warp 2 TMEM owner; all four warps run the epilogue
// (warp w reads TMEM lanes 32w..32w+31).  Every wait is bounded (ptx.cuh); a wait that runs out records an error code
// in `status` (when given) and the CTA skips its remaining work.
//
// Reference counterpart: the per-group decode projection einsum `fp8_einsum` (`king_v10/bundle_v9/dec/dgt.py:121-126`,
// its wo_a kernel); here the same per-head contraction serves the MLA query absorption (W_uk), the value
// un-absorption (W_uv) and the grouped output projection (wo_a) of decode batches.
#include <cudaTypedefs.h>
#include <algorithm>
#include <mutex>
#include <type_traits>
#include "ptx.cuh"
#include "small_ops.h"

namespace cb {
namespace hb {

constexpr int BM = 128;                 // weight rows (output columns n) per CTA
constexpr int BK = 64;                  // bf16 elements per 128-byte swizzle row
constexpr int TILE_A = BM * 128;        // bytes of one A stage
constexpr int kMaxStages = 8;
constexpr int kStageBudget = 200 * 1024;   // shared memory for the stage ring (every K chunk in flight when it fits)
constexpr int kThreads = 128;
constexpr int kMaxT = 256;

__host__ __device__ inline int tmem_cols_for(int tb) { return tb <= 32 ? 32 : tb <= 64 ? 64 : tb <= 128 ? 128 : 256; }

template <typename OutT>
__device__ __forceinline__ OutT cvt_out(float v);
template <>
__device__ __forceinline__ __nv_bfloat16 cvt_out<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half cvt_out<__half>(float v) { return __float2half_rn(v); }

struct Args {
  int T, TB, N, K, stages;
  void* out;
  long long os_t, os_h;                 // output strides (elements)
  const __nv_bfloat16* x;               // tail source (same tensor as the tensor map's)
  long long xs_t, xs_h;
  int tail;
  int* status;
};

template <typename OutT>
__global__ void __launch_bounds__(kThreads) head_bmm_kernel(const __grid_constant__ CUtensorMap tw,
                                                             const __grid_constant__ CUtensorMap tx, const Args a) {
#if defined(__CUDA_ARCH__) && __CUDA_ARCH__ >= 1000
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int stages = a.stages;
  const uint32_t tile_b = uint32_t(a.TB) * 128u;
  uint8_t* sA = smem;
  uint8_t* sB = sA + stages * TILE_A;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + stages * tile_b);
  uint64_t* empty = full + kMaxStages;
  uint64_t* done = empty + kMaxStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int nb = blockIdx.x, h = blockIdx.y;
  const uint32_t warp = warp_id(), lane = lane_id();
  const uint32_t cols = uint32_t(tmem_cols_for(a.TB));
  const int nk = a.K / BK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < stages; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], 1); }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) { tma_prefetch_desc(&tw); tma_prefetch_desc(&tx); }
  if (warp == 2) { tmem_alloc(tmem_slot, cols); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto fail = [&](int code) {
    if (a.status) atomicCAS(a.status, 0, code);
    *abort_flag = 1;
  };

  // The weights do not depend on the previous kernel: the first ring's weight tiles are requested before waiting
  // for it (programmatic dependent launch), the token rows after.
  const int pre = nk < stages ? nk : stages;
  if (warp == 0) {
    if (elect_one()) {
      for (int kb = 0; kb < pre; ++kb) {
        mbar_arrive_expect_tx(&full[kb], uint32_t(TILE_A) + tile_b);
        tma_load_2d(sA + kb * TILE_A, &tw, &full[kb], kb * BK, h * a.N + nb * BM);
      }
      pdl_wait();
      for (int kb = 0; kb < nk && !*abort_flag; ++kb) {
        const int s = kb % stages;
        const uint32_t ph = uint32_t(kb / stages) & 1u;
        if (kb >= pre) {
          if (!mbar_wait(&empty[s], ph ^ 1u)) { fail(kErrTimeoutEmpty); break; }
          mbar_arrive_expect_tx(&full[s], uint32_t(TILE_A) + tile_b);
          tma_load_2d(sA + s * TILE_A, &tw, &full[s], kb * BK, h * a.N + nb * BM);
        }
        tma_load_3d(sB + s * tile_b, &tx, &full[s], kb * BK, h, 0);
      }
    } else {
      pdl_wait();
    }
    pdl_launch_dependents();
  } else {
    pdl_wait();
    pdl_launch_dependents();
  }
  if (warp == 1) {
    if (elect_one()) {
      const uint32_t idesc = idesc_bf16(BM, a.TB);
      bool ok = true;
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % stages;
        const uint32_t ph = uint32_t(kb / stages) & 1u;
        if (!mbar_wait(&full[s], ph)) { fail(kErrTimeoutFull); ok = false; break; }
        tc_fence_after();
        const uint64_t ad = smem_desc_sw128(sA + s * TILE_A);
        const uint64_t bd = smem_desc_sw128(sB + s * tile_b);
#pragma unroll
        for (int k = 0; k < BK / 16; ++k) {
          const uint64_t koff = uint64_t((k * 16 * 2) >> 4);       // 32 bytes along K inside the swizzle atom
          mma_f16_ss(tmem, ad + koff, bd + koff, idesc, (kb > 0 || k > 0) ? 1u : 0u);
        }
        mma_commit(&empty[s]);
      }
      if (ok) mma_commit(done);
    }
  }
  __syncwarp();

  // tail columns (x[..., K:K+tail] copied unchanged) while the MMAs run, spread over the head's n-block CTAs in
  // 16-byte pieces (the host checks that rows, strides and offsets are 8-element multiples)
  if (a.tail > 0) {
    OutT* o = reinterpret_cast<OutT*>(a.out) + size_t(h) * a.os_h + a.N;
    const __nv_bfloat16* xs = a.x + size_t(h) * a.xs_h + a.K;
    const int per_row = a.tail / 8, items = a.T * per_row;
    for (int i = nb * kThreads + threadIdx.x; i < items; i += gridDim.x * kThreads) {
      const int t = i / per_row, j = (i - t * per_row) * 8;
      const uint4 v = *reinterpret_cast<const uint4*>(xs + size_t(t) * a.xs_t + j);
      uint4 r = v;
      if constexpr (sizeof(OutT) == 2 && !std::is_same<OutT, __nv_bfloat16>::value) {
        const uint32_t in[4] = {v.x, v.y, v.z, v.w};
        uint32_t outw[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const __half2 hv = __floats2half2_rn(bf16_lo(in[e]), bf16_hi(in[e]));
          outw[e] = *reinterpret_cast<const uint32_t*>(&hv);
        }
        r = make_uint4(outw[0], outw[1], outw[2], outw[3]);
      }
      *reinterpret_cast<uint4*>(o + size_t(t) * a.os_t + j) = r;
    }
  }

  // epilogue: TMEM lane = output column n, TMEM column = token t
  const bool ok = mbar_wait(done, 0);
  if (!ok) fail(kErrTimeoutTmem);
  tc_fence_after();
  if (ok && !*abort_flag) {
    const int n = nb * BM + int(warp) * 32 + int(lane);
    OutT* o = reinterpret_cast<OutT*>(a.out) + size_t(h) * a.os_h + n;
    const uint32_t trow = tmem + ((warp * 32u) << 16);
#pragma unroll 1
    for (int c = 0; c < a.TB; c += 16) {
      uint32_t v[16];
      tmem_ld_32x32b_x16(trow + uint32_t(c), v);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (c + j < a.T) o[size_t(c + j) * a.os_t] = cvt_out<OutT>(__uint_as_float(v[j]));
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, cols);
  }
#endif
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

// bf16 tensor map with 128-byte swizzled boxes; the base and every stride must be 16-byte multiples
static bool encode(CUtensorMap* m, const void* ptr, int rank, const cuuint64_t* dims, const cuuint64_t* strides,
                   const cuuint32_t* box) {
  auto fn = encode_fn();
  if (!fn || (reinterpret_cast<uintptr_t>(ptr) & 15)) return false;
  for (int i = 0; i + 1 < rank; ++i)
    if (strides[i] & 15) return false;
  const cuuint32_t es[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, cuuint32_t(rank), const_cast<void*>(ptr), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// stage count: every K chunk in flight at once when the ring fits the budget, at least one stage
static int head_bmm_stages(int tb, int K) {
  const int per = TILE_A + tb * 128;
  return std::max(1, std::min({kMaxStages, K / BK, kStageBudget / per}));
}

}  // namespace hb

int head_bmm_smem_bytes(int T, int K) {
  using namespace hb;
  const int tb = ((T + 15) / 16) * 16;
  const int stages = head_bmm_stages(tb, K);
  const int need = 1024 + stages * (TILE_A + tb * 128) + 8 * (2 * kMaxStages + 1) + 16;
  // a floor that admits at most 512 / cols CTAs per SM, so every resident CTA's TMEM allocation succeeds at once
  const int floor_bytes = tmem_cols_for(tb) * 454;
  return std::max(need, floor_bytes);
}

cudaError_t head_bmm(const void* x, long long xs_t, long long xs_h, const void* w, int T, int H, int N, int K,
                     void* out, bool out_f16, long long os_t, long long os_h, int tail, int* status,
                     cudaStream_t s) {
  using namespace hb;
  if (T <= 0 || H <= 0) return cudaSuccess;
  if (T > kMaxT || N % BM || K % BK || K <= 0 || tail < 0 || tail % 8 || xs_t % 8 || xs_h % 8 || os_t % 8 ||
      os_h % 8 || (reinterpret_cast<uintptr_t>(out) & 15))
    return cudaErrorInvalidValue;
  Args a;
  a.T = T;
  a.TB = ((T + 15) / 16) * 16;
  a.N = N;
  a.K = K;
  a.stages = head_bmm_stages(a.TB, K);
  a.out = out;
  a.os_t = os_t;
  a.os_h = os_h;
  a.x = reinterpret_cast<const __nv_bfloat16*>(x);
  a.xs_t = xs_t;
  a.xs_h = xs_h;
  a.tail = tail;
  a.status = status;
  CUtensorMap tw, tx;
  const cuuint64_t wd[2] = {cuuint64_t(K), cuuint64_t(H) * N};
  const cuuint64_t ws[1] = {cuuint64_t(K) * 2};
  const cuuint32_t wb[2] = {BK, BM};
  const cuuint64_t xd[3] = {cuuint64_t(K), cuuint64_t(H), cuuint64_t(T)};
  const cuuint64_t xst[2] = {cuuint64_t(xs_h) * 2, cuuint64_t(xs_t) * 2};
  const cuuint32_t xb[3] = {BK, 1, cuuint32_t(a.TB)};
  if (!encode(&tw, w, 2, wd, ws, wb) || !encode(&tx, x, 3, xd, xst, xb)) return cudaErrorInvalidValue;
  const int smem = head_bmm_smem_bytes(T, K);
  const dim3 grid(N / BM, H);
  cudaError_t e;
  if (out_f16) {
    e = smem_optin(head_bmm_kernel<__half>, smem);
    if (e != cudaSuccess) return e;
    return launch_k(head_bmm_kernel<__half>, grid, dim3(kThreads), smem, s, tw, tx, a);
  }
  e = smem_optin(head_bmm_kernel<__nv_bfloat16>, smem);
  if (e != cudaSuccess) return e;
  return launch_k(head_bmm_kernel<__nv_bfloat16>, grid, dim3(kThreads), smem, s, tw, tx, a);
}

}  // namespace cb
