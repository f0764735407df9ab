// Decode-side DSA lightning indexer logits on tcgen05 (sm_100a):
//
//   logits[t, j] = Σ_h w[t, h] · relu(q[t, h, :] · kc[key_slots[t, j], :])      for j < n_keys[t]  (else -inf)
//
// Each decode token has its own key list (cache slots in causal order), so the contraction is one small GEMM per
// token with the keys as M: S[128 keys, H heads] = K_tile · Q_tᵀ (K = 128 dims).  The key rows are gathered straight
// from the paged indexer-key cache with TMA tile::gather4 (box one row high, 64 dims = 128 bytes per row piece), the
// token's queries [H, 128] are loaded once by a 3-D TMA, the accumulator lives in TMEM (H fp32 columns per tile,
// double-buffered), and the epilogue warps apply relu and the per-head weights while draining TMEM (one key row per
// thread).
//
// Roles (192 threads): warp 0 TMA (Q once, then gathered key tiles through a STAGES-deep ring), warp 1 MMA (one
// elected thread issues tcgen05.mma) and TMEM allocation, warps 2-5 epilogue (TMEM lane quadrant = warp % 4).  Every
// wait is bounded; a wait that runs out records an error code and stops the CTA.
//
// Reference kernel with the same role: the paged indexer logits of the decode role, a block-scaled UMMA over fp4
// keys (king_v10/bundle_v9/dec/cuda_paged_logits.py:115); this one reads bf16 keys.
#include <cudaTypedefs.h>
#include "ptx.cuh"

namespace cb {
namespace idxd {

constexpr int KT = 128;                 // keys per tile (MMA M)
constexpr int DK = 128;                 // key / query dims (two 64-dim swizzle atoms)
constexpr int STAGES = 2;               // 84 KB of shared memory: two CTAs per SM (one wave for 32 x 4k keys)
constexpr int TILES_PER_CTA = 4;
constexpr int A_ATOM = KT * 128;        // 16 KB: 128 key rows x 64 dims
constexpr int A_BYTES = 2 * A_ATOM;     // 32 KB per stage
constexpr int HMAX = 128;

CB_HOST_DEVICE int smem_bytes(int H) { return 1024 + 2 * H * 128 + STAGES * A_BYTES + H * 4 + 256; }

struct Params {
  const int* key_slots;     // [T, Lmax]
  const int* n_keys;        // [T]
  const float* w;           // [T, H]
  float* out;               // [T, Lmax]
  int Lmax, H, tiles;       // tiles = ceil(Lmax / KT)
  int* status;
};

CB_DEVICE void tma_gather4(void* dst, const void* tmap, uint64_t* bar, int col, int r0, int r1, int r2, int r3) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(col), "r"(r0), "r"(r1),
      "r"(r2), "r"(r3)
      : "memory");
}

__global__ void __launch_bounds__(192) indexer_decode_kernel(const __grid_constant__ CUtensorMap tm_q,
                                                              const __grid_constant__ CUtensorMap tm_k,
                                                              const Params p) {
  cb::pdl_entry();
#if defined(__CUDA_ARCH__) && __CUDA_ARCH__ >= 1000
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int H = p.H;
  const int q_atom = H * 128;
  uint8_t* sA = smem;                                   // STAGES x [2 atoms x 128 rows x 128 B]
  uint8_t* sQ = sA + STAGES * A_BYTES;                  // [2 atoms x H rows x 128 B]
  float* sw = reinterpret_cast<float*>(sQ + 2 * q_atom);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sw + H);
  uint64_t* q_full = bars;
  uint64_t* a_full = bars + 1;                          // [STAGES]
  uint64_t* a_empty = a_full + STAGES;                  // [STAGES]
  uint64_t* acc_full = a_empty + STAGES;                // [2]
  uint64_t* acc_empty = acc_full + 2;                   // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int t = blockIdx.x;
  const int acc_cols = H <= 64 ? 64 : 128;             // TMEM columns per accumulator (two accumulators)
  const int n = min(p.n_keys[t], p.Lmax);
  const int tile0 = blockIdx.y * TILES_PER_CTA;
  const int tile1 = min(p.tiles, tile0 + TILES_PER_CTA);
  // tiles holding at least one key below n run the MMA; the rest of this CTA's keys are written as -inf
  const int mma_tiles = max(0, min(tile1, (n + KT - 1) / KT) - tile0);
  const int* slots_t = p.key_slots + size_t(t) * p.Lmax;
  const uint32_t warp = warp_id(), lane = lane_id();

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < STAGES; ++i) { mbar_init(&a_full[i], 1); mbar_init(&a_empty[i], 1); }
    for (int i = 0; i < 2; ++i) { mbar_init(&acc_full[i], 1); mbar_init(&acc_empty[i], 128); }
    *abort_flag = 0;
    fence_barrier_init();
  }
  for (int h = threadIdx.x; h < H; h += blockDim.x) sw[h] = p.w[size_t(t) * H + h];
  if (warp == 1) { tmem_alloc(tmem_slot, 2 * acc_cols); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto fail = [&](int code) { if (p.status) atomicCAS(p.status, 0, code); *abort_flag = 1; };

  if (warp == 0) {
    // ---------------- TMA: Q once, then the gathered key rows of each tile ----------------
    if (lane == 0 && mma_tiles > 0) {
      tma_prefetch_desc(&tm_q); tma_prefetch_desc(&tm_k);
      mbar_arrive_expect_tx(q_full, 2 * q_atom);
      tma_load_3d(sQ, &tm_q, q_full, 0, 0, t);
      tma_load_3d(sQ + q_atom, &tm_q, q_full, 64, 0, t);
    }
    // lane owns keys 4*lane .. 4*lane+3 of a tile; the next tile's slots are loaded one tile ahead
    auto load_slots = [&](int j, int (&r)[4]) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int key = (tile0 + j) * KT + lane * 4 + i;
        const int slot = (j < mma_tiles && key < n) ? slots_t[key] : 0;
        r[i] = slot < 0 ? 0 : slot;                     // masked in the epilogue; keep the address valid
      }
    };
    int nxt[4];
    load_slots(0, nxt);
    for (int j = 0; j < mma_tiles; ++j) {
      const int s = j % STAGES;
      int r[4] = {nxt[0], nxt[1], nxt[2], nxt[3]};
      load_slots(j + 1, nxt);
      int ok = 1;
      if (lane == 0) {
        ok = mbar_wait(&a_empty[s], ((j / STAGES) & 1) ^ 1) ? 1 : 0;
        if (ok) mbar_arrive_expect_tx(&a_full[s], A_BYTES);
        else fail(kErrTimeoutEmpty);
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok || *abort_flag) break;
      uint8_t* dst = sA + s * A_BYTES + lane * 4 * 128;
      tma_gather4(dst, &tm_k, &a_full[s], 0, r[0], r[1], r[2], r[3]);
      tma_gather4(dst + A_ATOM, &tm_k, &a_full[s], 64, r[0], r[1], r[2], r[3]);
      __syncwarp();
    }
  } else if (warp == 1) {
    // ---------------- MMA: S[128 keys, H] = K_tile · Q_tᵀ ----------------
    if (elect_one() && mma_tiles > 0) {
      const uint32_t idesc = idesc_bf16(KT, H);
      bool ok = mbar_wait(q_full, 0);
      if (!ok) fail(kErrTimeoutFull);
      for (int j = 0; ok && j < mma_tiles && !*abort_flag; ++j) {
        const int s = j % STAGES, b = j & 1;
        if (!mbar_wait(&a_full[s], (j / STAGES) & 1)) { fail(kErrTimeoutFull); break; }
        if (!mbar_wait(&acc_empty[b], ((j >> 1) & 1) ^ 1)) { fail(kErrTimeoutTmem); break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < DK / 16; ++kk) {
          const int a = kk >> 2, off = (kk & 3) * 32;
          mma_f16_ss(tmem + b * acc_cols, smem_desc_sw128(sA + s * A_BYTES + a * A_ATOM + off),
                     smem_desc_sw128(sQ + a * q_atom + off), idesc, kk > 0);
        }
        mma_commit(&a_empty[s]);
        mma_commit(&acc_full[b]);
      }
    }
  } else {
    // ---------------- epilogue: relu, per-head weights, one key row per thread ----------------
    const uint32_t quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t t_lane = tmem + ((quad * 32) << 16);
    float* out_t = p.out + size_t(t) * p.Lmax;
    for (int j = 0; j < mma_tiles; ++j) {
      const int b = j & 1;
      if (!mbar_wait(&acc_full[b], (j >> 1) & 1)) { fail(kErrTimeoutTmem); break; }
      tc_fence_after();
      float acc = 0.f;
      for (int c = 0; c < H; c += 16) {
        uint32_t v[16];
        tmem_ld_32x32b_x16(t_lane + b * acc_cols + c, v);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i) acc += sw[c + i] * fmaxf(__uint_as_float(v[i]), 0.f);
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[b]);
      const int key = (tile0 + j) * KT + row;
      if (key < p.Lmax) out_t[key] = (key < n && slots_t[key] >= 0) ? acc : -INFINITY;
    }
    // keys of this CTA's tiles that are all at or beyond n
    for (int key = (tile0 + mma_tiles) * KT + row; key < min(tile1 * KT, p.Lmax); key += KT) out_t[key] = -INFINITY;
  }
  __syncthreads();
  if (warp == 1) { tc_fence_after(); tmem_dealloc(tmem, 2 * acc_cols); }
#endif
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) ==
            cudaSuccess && q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

}  // namespace idxd

// q [T, H, 128] bf16, w [T, H] fp32, kc [S, 128] bf16 (indexer-key cache), key_slots [T, Lmax] int32 (-1 = none),
// n_keys [T] int32 -> out [T, Lmax] fp32 (-inf beyond n_keys or at slot -1).  H a multiple of 16, <= 128.
cudaError_t indexer_decode_logits(const void* q, const float* w, const void* kc, int S, const int* key_slots,
                                  const int* n_keys, int T, int Lmax, int H, int D, float* out, int* status,
                                  cudaStream_t s) {
  using namespace idxd;
  if (T == 0 || Lmax == 0) return cudaSuccess;
  if (D != DK || H % 16 || H < 16 || H > HMAX) return cudaErrorInvalidValue;
  auto fn = encode_fn();
  if (!fn) return cudaErrorInvalidValue;
  CUtensorMap tq, tk;
  {
    cuuint64_t dims[3] = {cuuint64_t(DK), cuuint64_t(H), cuuint64_t(T)};
    cuuint64_t str[2] = {cuuint64_t(DK) * 2, cuuint64_t(H) * DK * 2};
    cuuint32_t box[3] = {64, cuuint32_t(H), 1};
    cuuint32_t es[3] = {1, 1, 1};
    if (fn(&tq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(q), dims, str, box, es,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  {
    cuuint64_t dims[2] = {cuuint64_t(DK), cuuint64_t(S)};
    cuuint64_t str[1] = {cuuint64_t(DK) * 2};
    cuuint32_t box[2] = {64, 1};
    cuuint32_t es[2] = {1, 1};
    if (fn(&tk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(kc), dims, str, box, es,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  const int smem = smem_bytes(H);
  cudaError_t e = smem_optin(indexer_decode_kernel, smem);
  if (e != cudaSuccess) return e;
  Params p;
  p.key_slots = key_slots; p.n_keys = n_keys; p.w = w; p.out = out;
  p.Lmax = Lmax; p.H = H; p.tiles = (Lmax + KT - 1) / KT; p.status = status;
  dim3 grid(T, (p.tiles + TILES_PER_CTA - 1) / TILES_PER_CTA);
  cb::launch_k(indexer_decode_kernel, grid, 192, smem, s, tq, tk, p);
  return cudaGetLastError();
}

}  // namespace cb
