// Persistent warp-specialised tcgen05 GEMM for sm_100a:  D[M,N] = A[M,K] · B[N,K]^T  (both K-major).
//
//  * KIND_MXF8 : A, B fp8 e4m3 with UE8M0 block scales (A: 1x128 per row, B: 128x128), kind::mxf8f6f4.block_scale.
//  * KIND_BF16 : A, B bf16, kind::f16, fp32 accumulate.
//
// Roles (256 threads): warp 0 = TMA producer, warp 1 = MMA issuer, warp 2 = TMEM owner, warps 4..7 = epilogue
// (TMEM -> registers -> global).  A/B tiles arrive by TMA (128-byte swizzle) into a STAGES-deep ring; scale-factor
// tiles arrive by 1-D bulk copies in the layout tcgen05.cp 32x128b.warpx4 expects, so no transpose is needed.
// Accumulators live in TMEM (ACC_STAGES buffers of BLOCK_N fp32 columns) so the epilogue of tile i overlaps the
// MMAs of tile i+1.
//
// Grouped mode (MoE): A rows are expert-sorted and each 128-row block belongs to one expert
// (`m_block_expert[mb]`, -1 = unused block); B is [E*N, K] and the tile's B rows start at expert*N.
//
// Scale-factor tile layout ("SF tiles"): for every 512-wide K group kg and every 128-row block rb, 128 uint32
// words; word (l*4 + j) holds the four UE8M0 bytes (k-blocks 4kg..4kg+3, byte = k-block % 4) of row 32*j + l.
// Tiles are stored [kg][rb][128].
#pragma once
#include "ptx.cuh"

namespace cb {

enum GemmKind { KIND_MXF8 = 0, KIND_BF16 = 1 };
// EPI_BF16_ROWS: EPI_BF16 with the output staged in shared memory and stored row-contiguous (pair kernel only)
// EPI_BF16_PUSH: grouped expert GEMM whose output rows go straight to the routed token's home rank (EP combine)
enum GemmEpi { EPI_BF16 = 0, EPI_SWIGLU_FP8 = 1, EPI_F32 = 2, EPI_INDEXER = 3, EPI_BF16_SCATTER = 4,
               EPI_BF16_ROWS = 5, EPI_BF16_PUSH = 6 };

struct GemmParams {
  int M, N, K;                 // N = per-expert N in grouped mode
  const uint32_t* sfa;         // SF tiles of A  [K/512][ceil(M/128)][128]
  const uint32_t* sfb;         // SF tiles of B  [K/512][ceil(Nb/128)][128]  (Nb = rows of B)
  int sfa_row_blocks;          // ceil(M/128)
  int sfb_row_blocks;          // ceil(Nb/128)
  void* out;                   // EPI_BF16: bf16 [M, ldo]; EPI_F32: fp32; EPI_SWIGLU_FP8: fp8 [M, ldo]
  int ldo;
  uint32_t* out_sf;            // EPI_SWIGLU_FP8: SF tiles of the output [N/2/512][ceil(M/128)][128]
  float swiglu_limit;
  const int* m_block_expert;   // grouped: expert of each 128-row block (or -1); nullptr = dense
  const int* num_m_blocks_dev; // grouped: number of valid m blocks (device), nullptr => ceil(M/128)
  int* status;                 // error word (0 = ok)
  // EPI_INDEXER (DSA lightning indexer): A = keys [L, Di], B = queries x heads [Tq*H, Di]; the epilogue writes
  // logits[q, key] = sum_h w[q, h] * relu(acc[key, q*H + h]) (fp32, row stride ldo), -inf for key > q (causal).
  const float* idx_w;          // [Tq, idx_heads]
  int idx_heads;
  int causal;                  // skip tiles whose first key is after their last query
  int k_splits;                // EPI_F32 only: K split over CTAs; split s writes out + s*M*ldo (summed afterwards)
  // EPI_BF16_SCATTER (GEMM -> reduce-scatter over NVLink): output row `row` belongs to the rank r with
  // bounds[r] <= row < bounds[r+1]; it is stored straight into r's slot [my_rank] of its per-source partial buffer,
  // scatter_ptrs[r] + (my_rank * slot_rows + row - bounds[r]) * ldo.
  const uint64_t* scatter_ptrs;
  const int* scatter_bounds;
  int scatter_world, scatter_rank, scatter_rows;
  // optional: rows with row_valid[row] < 0 (expert-segment padding) are not written by the epilogue
  const int* row_valid;
  // EPI_BF16_PUSH (expert GEMM -> EP combine over NVLink): row_dst[row] = (home rank << 24) | slot, or -1 for a
  // padding row; the row is stored at scatter_ptrs[home] + slot * ldo (the home's [tokens * k, ldo] combine slots).
  const int* row_dst;
};

template <int BLOCK_N>
struct GemmSmem {
  static constexpr int BLOCK_M = 128;
  static constexpr int TILE_A = BLOCK_M * 128;   // bytes: 128 rows x 128 B
  static constexpr int TILE_B = BLOCK_N * 128;
  static constexpr int SFA_BYTES = 512;
  static constexpr int SFB_BYTES = (BLOCK_N / 128) * 512;
};

// Dense GEMMs: L2 prefetch of the B (weight) boxes of this CTA's first work item, up to one ring of k-blocks,
// issued before the kernel waits for its predecessor (programmatic dependent launch), so the weight stream of a
// decode-size GEMM starts while the previous kernel still runs.  The tile arithmetic is tile_coords' below.
template <int BLOCK_N, int STAGES, int BLOCK_K, bool SPLIT>
__device__ __forceinline__ void gemm_prefetch_first_b(const CUtensorMap* tmap_b, const GemmParams& p) {
#if defined(__CUDA_ARCH__) && __CUDA_ARCH__ >= 1000
  constexpr int GROUP_M = 16;
  const int num_mb = ceil_div(p.M, 128), num_nb = ceil_div(p.N, BLOCK_N);
  const int ksplit = (SPLIT && p.k_splits > 1) ? p.k_splits : 1;
  const int t = int(blockIdx.x);
  if (t >= num_mb * num_nb * ksplit) return;
  const int tt = t / ksplit;
  const int per_group = GROUP_M * num_nb;
  const int g = tt / per_group, r = tt - g * per_group;
  const int rows = min(GROUP_M, num_mb - g * GROUP_M);
  const int nb = r / rows;
  const int nk_total = ceil_div(p.K, BLOCK_K);
  const int nk_per = ceil_div(ceil_div(nk_total, ksplit), 4) * 4;
  const int kb0 = (t % ksplit) * nk_per, kb1 = min(nk_total, min(kb0 + nk_per, kb0 + STAGES));
  for (int kb = kb0; kb < kb1; ++kb) tma_prefetch_l2_2d(tmap_b, kb * BLOCK_K, nb * BLOCK_N);
#endif
}

template <int KIND, int EPI, int BLOCK_N, int STAGES, int ACC_STAGES>
__global__ void __launch_bounds__(256, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_a,
                                                         const __grid_constant__ CUtensorMap tmap_b,
                                                         const GemmParams p) {
  if (threadIdx.x == 0 && p.m_block_expert == nullptr)
    gemm_prefetch_first_b<BLOCK_N, STAGES, (KIND == KIND_MXF8 ? 128 : 64), EPI == EPI_F32>(&tmap_b, p);
  cb::pdl_entry();
#if defined(__CUDA_ARCH__) && __CUDA_ARCH__ >= 1000
  using S = GemmSmem<BLOCK_N>;
  constexpr int BLOCK_M = 128;
  constexpr bool kScaled = (KIND == KIND_MXF8);
  constexpr int kElemBytes = kScaled ? 1 : 2;
  constexpr int BLOCK_K = 128 / kElemBytes;              // one 128-byte swizzle atom of K per stage
  constexpr int UMMA_K = kScaled ? 32 : 16;
  constexpr int kMmaPerStage = BLOCK_K / UMMA_K;          // = 4
  constexpr int kSfbTiles = BLOCK_N / 128;
  constexpr uint32_t kAccCols = ACC_STAGES * BLOCK_N;
  constexpr uint32_t kSfaCol = kAccCols;
  constexpr uint32_t kSfbCol = kAccCols + 4;
  constexpr uint32_t kNeedCols = kAccCols + (kScaled ? 4 + 4 * kSfbTiles : 0);
  constexpr uint32_t kTmemCols = kNeedCols <= 32 ? 32 : kNeedCols <= 64 ? 64 : kNeedCols <= 128 ? 128
                                 : kNeedCols <= 256 ? 256 : 512;
  static_assert(kNeedCols <= 512, "TMEM budget");
  static_assert(BLOCK_N % 128 == 0 || !kScaled, "scaled GEMM needs BLOCK_N multiple of 128");

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * S::TILE_A;
  uint8_t* sSFA = sB + STAGES * S::TILE_B;
  uint8_t* sSFB = sSFA + (kScaled ? STAGES * S::SFA_BYTES : 0);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sSFB + (kScaled ? STAGES * S::SFB_BYTES : 0));
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + STAGES;
  uint64_t* tfull_bar = bars + 2 * STAGES;
  uint64_t* tempty_bar = bars + 2 * STAGES + ACC_STAGES;
  uint32_t* tmem_base_smem = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 2 * ACC_STAGES);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_smem + 1);

  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) { mbar_init(&full_bar[i], 1); mbar_init(&empty_bar[i], 1); }
    for (int i = 0; i < ACC_STAGES; ++i) { mbar_init(&tfull_bar[i], 1); mbar_init(&tempty_bar[i], 128); }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) { tma_prefetch_desc(&tmap_a); tma_prefetch_desc(&tmap_b); }
  if (warp == 2) { tmem_alloc(tmem_base_smem, kTmemCols); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_smem;

  // ---- tile schedule (identical in every role) ----
  const bool grouped = p.m_block_expert != nullptr;
  const int num_mb = grouped ? (p.num_m_blocks_dev ? *p.num_m_blocks_dev : ceil_div(p.M, BLOCK_M))
                             : ceil_div(p.M, BLOCK_M);
  const int num_nb = ceil_div(p.N, BLOCK_N);
  const int ksplit = (EPI == EPI_F32 && p.k_splits > 1) ? p.k_splits : 1;
  const int num_tiles = num_mb * num_nb * ksplit;
  const int nk_total = ceil_div(p.K, BLOCK_K);
  const int nk_per = ceil_div(ceil_div(nk_total, ksplit), 4) * 4;   // whole SF groups per split
  constexpr int GROUP_M = 16;
  auto tile_coords = [&](int t, int& mb, int& nb) {
    t /= ksplit;
    const int per_group = GROUP_M * num_nb;
    const int g = t / per_group, r = t - g * per_group;
    const int rows = min(GROUP_M, num_mb - g * GROUP_M);
    mb = g * GROUP_M + r % rows;
    nb = r / rows;
  };
  auto fail = [&](int code) {
    if (p.status) atomicCAS(p.status, 0, code);
    *abort_flag = 1;
  };
  // causal tile skip (indexer): queries of tile nb are [nb*QPT, nb*QPT+QPT)
  auto skip_tile = [&](int mb, int nb, int t) -> bool {
    if (ksplit > 1 && (t % ksplit) * nk_per >= nk_total) return true;   // empty K split
    if constexpr (EPI == EPI_INDEXER) {
      const int qpt = BLOCK_N / p.idx_heads;
      return p.causal && mb * BLOCK_M > nb * qpt + qpt - 1;
    } else {
      return false;
    }
  };

  if (warp == 0) {
    // ================= TMA producer =================
    if (elect_one()) {
      int stage = 0; uint32_t phase = 0;
      for (int t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x) {
        int mb, nb; tile_coords(t, mb, nb);
        if (skip_tile(mb, nb, t)) continue;
        int expert = 0;
        if (grouped) { expert = p.m_block_expert[mb]; if (expert < 0) continue; }
        const int a_row = mb * BLOCK_M;
        const int b_row = expert * p.N + nb * BLOCK_N;
        const int kb0 = (t % ksplit) * nk_per, kb1 = min(nk_total, kb0 + nk_per);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1)) { fail(kErrTimeoutEmpty); break; }
          uint32_t bytes = S::TILE_A + S::TILE_B;
          if (kScaled && (kb & 3) == 0) {
            const int kg = kb >> 2;
            bulk_load(sSFA + stage * S::SFA_BYTES, p.sfa + (size_t(kg) * p.sfa_row_blocks + mb) * 128,
                      S::SFA_BYTES, &full_bar[stage]);
            bulk_load(sSFB + stage * S::SFB_BYTES, p.sfb + (size_t(kg) * p.sfb_row_blocks + b_row / 128) * 128,
                      S::SFB_BYTES, &full_bar[stage]);
            bytes += S::SFA_BYTES + S::SFB_BYTES;
          }
          mbar_arrive_expect_tx(&full_bar[stage], bytes);
          tma_load_2d(sA + stage * S::TILE_A, &tmap_a, &full_bar[stage], kb * BLOCK_K, a_row);
          tma_load_2d(sB + stage * S::TILE_B, &tmap_b, &full_bar[stage], kb * BLOCK_K, b_row);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ================= MMA issuer =================
    if (elect_one()) {
      int stage = 0; uint32_t phase = 0; int iter = 0;
      for (int t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x) {
        int mb, nb; tile_coords(t, mb, nb);
        if (skip_tile(mb, nb, t)) continue;
        if (grouped && p.m_block_expert[mb] < 0) continue;
        const int acc = iter % ACC_STAGES;
        const uint32_t acc_phase = (iter / ACC_STAGES) & 1;
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1)) { fail(kErrTimeoutTmem); break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BLOCK_N;
        bool ok = true;
        const int kb0 = (t % ksplit) * nk_per, kb1 = min(nk_total, kb0 + nk_per);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase)) { fail(kErrTimeoutFull); ok = false; break; }
          tc_fence_after();
          if constexpr (kScaled) {
            if ((kb & 3) == 0) {
              tmem_cp_32x128b_x4(tmem_base + kSfaCol, smem_desc_sf(sSFA + stage * S::SFA_BYTES));
#pragma unroll
              for (int i = 0; i < kSfbTiles; ++i)
                tmem_cp_32x128b_x4(tmem_base + kSfbCol + 4 * i, smem_desc_sf(sSFB + stage * S::SFB_BYTES + i * 512));
            }
          }
          const uint64_t a_desc = smem_desc_sw128(sA + stage * S::TILE_A);
          const uint64_t b_desc = smem_desc_sw128(sB + stage * S::TILE_B);
#pragma unroll
          for (int k = 0; k < kMmaPerStage; ++k) {
            const uint64_t koff = uint64_t((k * UMMA_K * kElemBytes) >> 4);  // advance inside the swizzle atom
            const uint32_t accum = (kb > kb0 || k > 0) ? 1u : 0u;
            if constexpr (kScaled) {
              const uint32_t sf_id = uint32_t(kb & 3);
              mma_mxf8_ss(d_tmem, a_desc + koff, b_desc + koff, idesc_mxf8(BLOCK_M, BLOCK_N, sf_id, sf_id),
                          tmem_base + kSfaCol, tmem_base + kSfbCol, accum);
            } else {
              mma_f16_ss(d_tmem, a_desc + koff, b_desc + koff, idesc_bf16(BLOCK_M, BLOCK_N), accum);
            }
          }
          mma_commit(&empty_bar[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        mma_commit(&tfull_bar[acc]);
        ++iter;
      }
    }
  } else if (warp >= 4) {
    // ================= epilogue =================
    const uint32_t q = warp & 3;                 // TMEM lane quadrant of this warp
    const uint32_t row_in_tile = q * 32 + lane;
    int iter = 0;
    for (int t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x) {
      int mb, nb; tile_coords(t, mb, nb);
      if (skip_tile(mb, nb, t)) continue;
      if (grouped && p.m_block_expert[mb] < 0) continue;
      const int acc = iter % ACC_STAGES;
      const uint32_t acc_phase = (iter / ACC_STAGES) & 1;
      if (!mbar_wait(&tfull_bar[acc], acc_phase)) { fail(kErrTimeoutTmem); break; }
      tc_fence_after();
      const int row = mb * BLOCK_M + row_in_tile;
      const bool row_ok = row < p.M && (p.row_valid == nullptr || p.row_valid[row] >= 0);
      const uint32_t t_row = tmem_base + ((q * 32) << 16) + acc * BLOCK_N;
      if constexpr (EPI == EPI_BF16 || EPI == EPI_F32 || EPI == EPI_BF16_SCATTER) {
        __nv_bfloat16* row_base = nullptr;
        if constexpr (EPI == EPI_BF16_SCATTER) {
          int r = 0;
          while (r + 1 < p.scatter_world && row >= p.scatter_bounds[r + 1]) ++r;
          row_base = reinterpret_cast<__nv_bfloat16*>(p.scatter_ptrs[r]) +
                     (size_t(p.scatter_rank) * p.scatter_rows + (row - p.scatter_bounds[r])) * size_t(p.ldo);
        } else if constexpr (EPI == EPI_BF16) {
          row_base = reinterpret_cast<__nv_bfloat16*>(p.out) + size_t(row) * p.ldo;
        }
#pragma unroll 1
        for (int c = 0; c < BLOCK_N; c += 32) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(t_row + c, v);
          tmem_ld_wait();
          const int col0 = nb * BLOCK_N + c;
          if (row_ok && col0 < p.N) {
            if constexpr (EPI == EPI_BF16 || EPI == EPI_BF16_SCATTER) {
              __nv_bfloat16* o = row_base + col0;
              if (col0 + 32 <= p.N && (p.ldo % 8) == 0) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  uint4 w;
                  w.x = pack_bf16x2(__uint_as_float(v[8 * j + 0]), __uint_as_float(v[8 * j + 1]));
                  w.y = pack_bf16x2(__uint_as_float(v[8 * j + 2]), __uint_as_float(v[8 * j + 3]));
                  w.z = pack_bf16x2(__uint_as_float(v[8 * j + 4]), __uint_as_float(v[8 * j + 5]));
                  w.w = pack_bf16x2(__uint_as_float(v[8 * j + 6]), __uint_as_float(v[8 * j + 7]));
                  reinterpret_cast<uint4*>(o)[j] = w;
                }
              } else {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (col0 + j < p.N) o[j] = __float2bfloat16_rn(__uint_as_float(v[j]));
              }
            } else {
              float* o = reinterpret_cast<float*>(p.out) + size_t(row) * p.ldo + col0;
              if (ksplit > 1) {
                // deterministic split-K: each split writes its own partial slab; a reduce kernel sums them in order
                o += size_t(t % ksplit) * size_t(p.M) * p.ldo;
              }
              if (col0 + 32 <= p.N && (p.ldo % 4) == 0) {
#pragma unroll
                for (int j = 0; j < 8; ++j)
                  reinterpret_cast<uint4*>(o)[j] = make_uint4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
              } else {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (col0 + j < p.N) o[j] = __uint_as_float(v[j]);
              }
            }
          }
        }
      } else if constexpr (EPI == EPI_INDEXER) {
        const int qpt = BLOCK_N / p.idx_heads;
        const int key = row;                                   // A rows are keys
        for (int j = 0; j < qpt; ++j) {
          const int qi = nb * qpt + j;
          const bool q_ok = qi * p.idx_heads < p.N;
          const float* wq = p.idx_w + size_t(q_ok ? qi : 0) * p.idx_heads;
          float acc_l = 0.f;
#pragma unroll 1
          for (int c = 0; c < p.idx_heads; c += 32) {
            // two 16-column loads in flight, one wait (the head count is a multiple of 16)
            uint32_t v[32];
            uint32_t (&v0)[16] = *reinterpret_cast<uint32_t(*)[16]>(&v[0]);
            uint32_t (&v1)[16] = *reinterpret_cast<uint32_t(*)[16]>(&v[16]);
            const bool two = c + 16 < p.idx_heads;
            tmem_ld_32x32b_x16(t_row + j * p.idx_heads + c, v0);
            if (two) tmem_ld_32x32b_x16(t_row + j * p.idx_heads + c + 16, v1);
            const float4* w4 = reinterpret_cast<const float4*>(wq + c);
            float wv[32];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float4 x = (i < 4 || two) ? w4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
              wv[4 * i] = x.x; wv[4 * i + 1] = x.y; wv[4 * i + 2] = x.z; wv[4 * i + 3] = x.w;
            }
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 16; ++i) acc_l += wv[i] * fmaxf(__uint_as_float(v[i]), 0.f);
            if (two)
#pragma unroll
              for (int i = 16; i < 32; ++i) acc_l += wv[i] * fmaxf(__uint_as_float(v[i]), 0.f);
          }
          if (row_ok && q_ok) {
            float* o = reinterpret_cast<float*>(p.out) + size_t(qi) * p.ldo + key;
            *o = (p.causal && key > qi) ? -INFINITY : acc_l;
          }
        }
      } else {
        // SwiGLU + fp8 requant: tile columns [0, BLOCK_N/2) are gate, [BLOCK_N/2, BLOCK_N) are up, both for the
        // same BLOCK_N/2 output columns; the output block of 128 columns gets one UE8M0 scale per row.
        static_assert(EPI != EPI_SWIGLU_FP8 || BLOCK_N == 256, "SwiGLU epilogue uses 256-wide tiles");
        constexpr int HALF = BLOCK_N / 2;
        float act[HALF];
        float amax = 0.f;
#pragma unroll
        for (int c = 0; c < HALF; c += 16) {
          uint32_t g[16], u[16];
          tmem_ld_32x32b_x16(t_row + c, g);
          tmem_ld_32x32b_x16(t_row + HALF + c, u);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float gv = __uint_as_float(g[j]), uv = __uint_as_float(u[j]);
            if (p.swiglu_limit > 0.f) { gv = fminf(gv, p.swiglu_limit); uv = fminf(fmaxf(uv, -p.swiglu_limit), p.swiglu_limit); }
            const float a = gv / (1.f + __expf(-gv)) * uv;
            act[c + j] = a;
            amax = fmaxf(amax, fabsf(a));
          }
        }
        // every TMEM read of this tile is done: hand the accumulator back before quantising and storing, so the
        // MMAs of the next tile overlap this epilogue even with a single accumulator stage
        tc_fence_before();
        mbar_arrive(&tempty_bar[acc]);
        if (row_ok) {
          const uint32_t sb = ue8m0_for_amax(amax);
          const float inv = ue8m0_inv(sb);
          const int ocol0 = nb * HALF;                        // output column of this tile
          uint8_t* o = reinterpret_cast<uint8_t*>(p.out) + size_t(row) * p.ldo + ocol0;
#pragma unroll
          for (int j = 0; j < HALF / 16; ++j) {
            uint4 w;
            w.x = pack_fp8x4(act[16 * j + 0] * inv, act[16 * j + 1] * inv, act[16 * j + 2] * inv, act[16 * j + 3] * inv);
            w.y = pack_fp8x4(act[16 * j + 4] * inv, act[16 * j + 5] * inv, act[16 * j + 6] * inv, act[16 * j + 7] * inv);
            w.z = pack_fp8x4(act[16 * j + 8] * inv, act[16 * j + 9] * inv, act[16 * j + 10] * inv, act[16 * j + 11] * inv);
            w.w = pack_fp8x4(act[16 * j + 12] * inv, act[16 * j + 13] * inv, act[16 * j + 14] * inv, act[16 * j + 15] * inv);
            reinterpret_cast<uint4*>(o)[j] = w;
          }
          // scale byte: k-block kbo = ocol0/128 of the output, row `row`
          const int kbo = ocol0 / 128;
          const int rb = row / 128, r = row % 128;
          uint8_t* sf = reinterpret_cast<uint8_t*>(p.out_sf) +
                        ((size_t(kbo >> 2) * p.sfa_row_blocks + rb) * 128 + (r % 32) * 4 + (r / 32)) * 4 + (kbo & 3);
          *sf = uint8_t(sb);
        }
      }
      if constexpr (EPI != EPI_SWIGLU_FP8) {
        tc_fence_before();
        mbar_arrive(&tempty_bar[acc]);
      }
      ++iter;
    }
    if constexpr (EPI == EPI_BF16_SCATTER) __threadfence_system();   // peer stores performed before any barrier
  }

  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
#endif
}

template <int KIND, int BLOCK_N, int STAGES>
constexpr int gemm_smem_bytes() {
  using S = GemmSmem<BLOCK_N>;
  return 1024 /*align slack*/ + STAGES * (S::TILE_A + S::TILE_B) +
         (KIND == KIND_MXF8 ? STAGES * (S::SFA_BYTES + S::SFB_BYTES) : 0) + 8 * (2 * STAGES + 4) + 16;
}

}  // namespace cb
