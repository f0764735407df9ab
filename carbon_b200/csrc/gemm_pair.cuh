// Persistent tcgen05 GEMM on 256x256 tiles computed by a CTA pair (cta_group::2), sm_100a:
//   D[M,N] = A[M,K] · B[N,K]^T, both K-major; KIND_MXF8 (e4m3 + UE8M0 1x128 / 128x128 scales) or KIND_BF16.
//
// Why pairs: one 128x128 tile per SM re-reads every A and B byte N/128 resp. M/128 times from L2, and on B200 the
// L2->SM path saturates before the tensor pipe does.  A pair tile of 256x256 is one MMA of M=256, N=256 issued by
// the leader CTA: each CTA stages its own 128 rows of A and its own 128 rows of B, the tensor core reads both
// CTAs' shared memory and writes each CTA's 128 accumulator rows into that CTA's TMEM.  Per SM the L2 traffic per
// FLOP halves.  With PAIR = 1 the same kernel runs 128x256 tiles on one CTA.
//
// Roles (384 threads per CTA): warp 0 TMA producer (both CTAs, each loads its half), warp 1 MMA issuer (leader
// only), warp 2 TMEM allocation, warps 4..11 epilogue (two warps per TMEM lane quadrant, each owning 128 of the 256
// accumulator columns).
//
// TMEM (512 columns): scale factors in [0,32), accumulator stage 0 in [32,288), stage 1 in [256,512).  The two
// stages overlap in [256,288), so the epilogue drains those 32 columns first and releases them on `tempty_ovl`,
// then the rest on `tempty_full`; the MMAs of tile j wait for the full release of tile j-2 (same stage) and the
// overlap release of tile j-1.  This gives double-buffered 256-column accumulators next to the scale factors.
// Without scale factors (KIND_BF16) the stages are [0,256) and [256,512) and do not overlap.
//
// Barriers live in each CTA; the leader's `full` barrier counts the TMA bytes of both CTAs, the leader's MMA
// completion is multicast to both CTAs' `empty`/`tfull` barriers, and both CTAs' epilogue warps arrive on the
// leader's `tempty_*` barriers.  Every wait is bounded (ptx.cuh: mbar_wait); on timeout the CTA records an error
// code, stops its loops and still reaches the final cluster barrier and TMEM release.
#pragma once
#include "gemm.cuh"

namespace cb {

template <int KIND, int PAIR, int EPI = EPI_BF16>
struct PairCfg {
  static constexpr int BN = 256;                       // tile N (each CTA stages BN/PAIR rows of B)
  static constexpr int BM = 128 * PAIR;                // tile M (each CTA: 128 rows of A, 128 accumulator lanes)
  static constexpr bool kScaled = KIND == KIND_MXF8;
  static constexpr int kElemBytes = kScaled ? 1 : 2;
  static constexpr int BK = 128 / kElemBytes;          // one 128-byte swizzle atom of K per stage
  static constexpr int UMMA_K = kScaled ? 32 : 16;
  static constexpr int TILE_A = 128 * 128;
  static constexpr int TILE_B = (BN / PAIR) * 128;
  static constexpr int SFA_BYTES = kScaled ? 512 : 0;
  static constexpr int SFB_BYTES = kScaled ? (BN / 128) * 512 : 0;
  static constexpr uint32_t kSfaCol = 0, kSfbCol = 4;
  static constexpr uint32_t kAcc0 = kScaled ? 32 : 0;
  static constexpr uint32_t kAcc1 = 512 - BN;
  static constexpr int kOvl = int(kAcc0) + BN - int(kAcc1);   // columns shared by the two stages (32 or 0)
  // the indexer epilogue is latency bound (one short reduction per query): four warps per lane quadrant
  static constexpr int kEpiWarps = EPI == EPI_INDEXER ? 16 : 8;
  static constexpr int kParts = kEpiWarps / 4;         // epilogue warps per TMEM lane quadrant
  static constexpr int kThreads = 128 + 32 * kEpiWarps;
};

// Peer-store staging of the scatter epilogue: per epilogue warp 32 rows x 64 bf16 columns, rows padded to 144 bytes
// so that the row-per-lane writes (8 lanes per 16-byte phase) and the row-contiguous reads are bank-conflict free.
constexpr int kScatterRowBytes = 144;
constexpr int kScatterWarpBytes = 32 * kScatterRowBytes;

// SwiGLU epilogue staging: per TMEM lane quadrant the 32 rows x 128 fp8 output bytes of a tile (both column
// halves), rows padded to 144 bytes
constexpr int kSwiQuadBytes = 32 * kScatterRowBytes;

template <int KIND, int PAIR, int STAGES, int EPI = EPI_BF16>
constexpr int gemm_pair_smem_bytes() {
  using C = PairCfg<KIND, PAIR, EPI>;
  return 1024 + STAGES * (C::TILE_A + C::TILE_B + C::SFA_BYTES + C::SFB_BYTES) + 8 * (2 * STAGES + 8) + 16 +
         2 * 2 * 128 * 4 +
         (EPI == EPI_BF16_SCATTER || EPI == EPI_BF16_ROWS || EPI == EPI_BF16_PUSH
              ? 16 + C::kEpiWarps * kScatterWarpBytes : 0) +
         (EPI == EPI_SWIGLU_FP8 ? 16 + 4 * kSwiQuadBytes + 4 * 8 : 0);
}

template <int KIND, int EPI, int PAIR, int STAGES>
__global__ void __launch_bounds__(PairCfg<KIND, PAIR, EPI>::kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                     const __grid_constant__ CUtensorMap tmap_sfa, const __grid_constant__ CUtensorMap tmap_sfb,
                     const GemmParams p) {
  cb::pdl_entry();
#if defined(__CUDA_ARCH__) && __CUDA_ARCH__ >= 1000
  using C = PairCfg<KIND, PAIR, EPI>;
  constexpr int BN = C::BN, BM = C::BM, BK = C::BK;
  constexpr bool kScaled = C::kScaled;
  constexpr int kMmaPerStage = BK / C::UMMA_K;
  static_assert(EPI == EPI_BF16 || EPI == EPI_BF16_SCATTER || EPI == EPI_BF16_ROWS || EPI == EPI_BF16_PUSH ||
                    EPI == EPI_SWIGLU_FP8 ||
                    EPI == EPI_INDEXER,
                "pair GEMM epilogues");
  static_assert(EPI != EPI_SWIGLU_FP8 || kScaled, "SwiGLU requant epilogue follows an fp8 GEMM");

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * C::TILE_A;
  uint8_t* sSFA = sB + STAGES * C::TILE_B;
  uint8_t* sSFB = sSFA + STAGES * C::SFA_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sSFB + STAGES * C::SFB_BYTES);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + STAGES;
  uint64_t* tfull_bar = bars + 2 * STAGES;            // [2]
  uint64_t* tempty_full = bars + 2 * STAGES + 2;      // [2] (leader's are used)
  uint64_t* tempty_ovl = bars + 2 * STAGES + 4;       // [2] (leader's are used)
  uint64_t* xbar = bars + 2 * STAGES + 6;             // SwiGLU amax exchange between the two column halves
  uint32_t* tmem_base_smem = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_smem + 1);
  float* xamax = reinterpret_cast<float*>(tmem_base_smem + 4);   // [2 tiles][2 halves][128 rows]
  uint8_t* xstage = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(xamax + 2 * 2 * 128) + 15) & ~uintptr_t(15));
  // SwiGLU: one mbarrier per TMEM lane quadrant pairs its two epilogue warps around the staging rows (bounded waits)
  uint64_t* qbar = reinterpret_cast<uint64_t*>(xstage + 4 * kSwiQuadBytes);

  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();
  const uint32_t rank = PAIR == 2 ? cluster_ctarank() : 0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) { mbar_init(&full_bar[i], 1); mbar_init(&empty_bar[i], 1); }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull_bar[i], 1);
      mbar_init(&tempty_full[i], C::kEpiWarps * PAIR);
      // the indexer epilogue releases the overlap columns with the full drain (every warp arrives)
      mbar_init(&tempty_ovl[i], (EPI == EPI_INDEXER ? C::kEpiWarps : C::kEpiWarps / 2) * PAIR);
    }
    mbar_init(xbar, 32 * C::kEpiWarps);
    if constexpr (EPI == EPI_SWIGLU_FP8)
      for (int i = 0; i < 4; ++i) mbar_init(&qbar[i], 64);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_a); tma_prefetch_desc(&tmap_b);
    if (kScaled) { tma_prefetch_desc(&tmap_sfa); tma_prefetch_desc(&tmap_sfb); }
  }
  if (warp == 2) {
    if constexpr (PAIR == 2) { tmem_alloc_pair(tmem_base_smem, 512); tmem_relinquish_pair(); }
    else { tmem_alloc(tmem_base_smem, 512); tmem_relinquish(); }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR == 2) cluster_sync();   // the peer's barriers exist before any cross-CTA signal
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_smem;

  // ---- tile schedule (identical in every role and in both CTAs of a pair) ----
  const int unit = blockIdx.x / PAIR, n_units = gridDim.x / PAIR;
  const bool grouped = p.m_block_expert != nullptr;
  const int num_mb = grouped ? (p.num_m_blocks_dev ? *p.num_m_blocks_dev : ceil_div(p.M, 128)) / PAIR
                             : ceil_div(p.M, BM);
  const int num_nb = ceil_div(p.N, BN);
  const int num_tiles = num_mb * num_nb;
  const int nk = ceil_div(p.K, BK);
  constexpr int GROUP_M = 8;
  auto tile_coords = [&](int t, int& mb, int& nb) {
    const int per_group = GROUP_M * num_nb;
    const int g = t / per_group, r = t - g * per_group;
    const int rows = min(GROUP_M, num_mb - g * GROUP_M);
    mb = g * GROUP_M + r % rows;
    nb = r / rows;
  };
  auto tile_expert = [&](int mb) -> int { return grouped ? p.m_block_expert[mb * PAIR] : 0; };
  auto skip_tile = [&](int mb, int nb) -> bool {
    if (grouped && tile_expert(mb) < 0) return true;
    if constexpr (EPI == EPI_INDEXER) {
      const int qpt = BN / p.idx_heads;
      return p.causal && mb * BM > nb * qpt + qpt - 1;
    }
    return false;
  };
  auto fail = [&](int code) {
    if (p.status) atomicCAS(p.status, 0, code);
    *abort_flag = 1;
  };
  // leader-CTA address of a barrier (the leader's own barriers are addressed the same way)
  auto leader_bar = [&](uint64_t* bar) -> uint32_t {
    return PAIR == 2 ? mapa_shared(smem_u32(bar), 0) : smem_u32(bar);
  };

  if (warp == 0) {
    // ================= TMA producer (each CTA loads its own half) =================
    if (elect_one()) {
      int stage = 0; uint32_t phase = 0;
      for (int t = unit; t < num_tiles && !*abort_flag; t += n_units) {
        int mb, nb; tile_coords(t, mb, nb);
        if (skip_tile(mb, nb)) continue;
        const int expert = tile_expert(mb);
        const int a_row = mb * BM + int(rank) * 128;
        const int b_tile = expert * p.N + nb * BN;
        // B rows of this CTA: pair -> [r*64, r*64+64) and [128+r*64, 128+r*64+64) of the tile, so that the MMA
        // half h (N columns [128h, 128h+128)) reads 64 rows from each CTA; single CTA -> the whole 256 rows
        const int b_row = b_tile + int(rank) * 64;
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1)) { fail(kErrTimeoutEmpty); break; }
          const bool sf_now = kScaled && (kb & 3) == 0;
          const uint32_t bytes = C::TILE_A + C::TILE_B + (sf_now ? C::SFA_BYTES + C::SFB_BYTES : 0);
          if (rank == 0) mbar_arrive_expect_tx(&full_bar[stage], bytes * PAIR);
          if constexpr (PAIR == 2) {
            const uint32_t fb = leader_bar(&full_bar[stage]);
            tma_load_2d_pair(sA + stage * C::TILE_A, &tmap_a, fb, kb * BK, a_row);
            tma_load_2d_pair(sB + stage * C::TILE_B, &tmap_b, fb, kb * BK, b_row);
            tma_load_2d_pair(sB + stage * C::TILE_B + C::TILE_B / 2, &tmap_b, fb, kb * BK, b_row + 128);
            if (sf_now) {
              const int kg = kb >> 2;
              tma_load_2d_pair(sSFA + stage * C::SFA_BYTES, &tmap_sfa, fb, 0, kg * p.sfa_row_blocks + mb * PAIR + rank);
              tma_load_2d_pair(sSFB + stage * C::SFB_BYTES, &tmap_sfb, fb, 0, kg * p.sfb_row_blocks + b_tile / 128);
            }
          } else {
            tma_load_2d(sA + stage * C::TILE_A, &tmap_a, &full_bar[stage], kb * BK, a_row);
            tma_load_2d(sB + stage * C::TILE_B, &tmap_b, &full_bar[stage], kb * BK, b_row);
            if (sf_now) {
              const int kg = kb >> 2;
              tma_load_2d(sSFA + stage * C::SFA_BYTES, &tmap_sfa, &full_bar[stage], 0, kg * p.sfa_row_blocks + mb);
              tma_load_2d(sSFB + stage * C::SFB_BYTES, &tmap_sfb, &full_bar[stage], 0, kg * p.sfb_row_blocks + b_tile / 128);
            }
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ================= MMA issuer (leader CTA) =================
    // Each k-step is two N=128 MMAs, one per accumulator half (lo = local columns [0,128), hi = [128,256)).
    // The half that contains this stage's overlap columns waits for the previous tile's overlap drain; the other
    // half starts at once, and the overlap half of up to kDefer k-blocks (all inside the first scale group, so the
    // scale factors in TMEM are still the right ones) is issued when the drain has arrived.
    if (rank == 0 && elect_one()) {
      constexpr int kDefer = 3;
      int stage = 0; uint32_t phase = 0; int j = 0;
      const uint32_t idesc_h = kScaled ? 0u : idesc_bf16(BM, 128);
      for (int t = unit; t < num_tiles && !*abort_flag; t += n_units) {
        int mb, nb; tile_coords(t, mb, nb);
        if (skip_tile(mb, nb)) continue;
        const int s = j & 1;
        if (!mbar_wait(&tempty_full[s], ((j >> 1) & 1) ^ 1)) { fail(kErrTimeoutTmem); break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (s ? C::kAcc1 : C::kAcc0);
        const int free_half = s == 0 ? 0 : 1;             // half without overlap columns
        bool ovl_ready = C::kOvl == 0 || j == 0;
        int deferred = 0;
        int dstage[kDefer];
        auto issue_half = [&](int half, int st, int kb) {
          const uint64_t a_desc = smem_desc_sw128(sA + st * C::TILE_A);
          const uint64_t b_desc = smem_desc_sw128(sB + st * C::TILE_B + half * (C::TILE_B / 2));
          const uint32_t d = d_tmem + 128 * half;
#pragma unroll
          for (int k = 0; k < kMmaPerStage; ++k) {
            const uint64_t koff = uint64_t((k * C::UMMA_K * C::kElemBytes) >> 4);
            const uint32_t accum = (kb > 0 || k > 0) ? 1u : 0u;
            if constexpr (kScaled) {
              const uint32_t sf_id = uint32_t(kb & 3);
              const uint32_t id = idesc_mxf8(BM, 128, sf_id, sf_id);
              const uint32_t sfb = tmem_base + C::kSfbCol + 4 * half;
              if constexpr (PAIR == 2) mma_mxf8_ss_pair(d, a_desc + koff, b_desc + koff, id, tmem_base + C::kSfaCol, sfb, accum);
              else mma_mxf8_ss(d, a_desc + koff, b_desc + koff, id, tmem_base + C::kSfaCol, sfb, accum);
            } else {
              if constexpr (PAIR == 2) mma_f16_ss_pair(d, a_desc + koff, b_desc + koff, idesc_h, accum);
              else mma_f16_ss(d, a_desc + koff, b_desc + koff, idesc_h, accum);
            }
          }
        };
        auto release_stage = [&](int st) {
          if constexpr (PAIR == 2) mma_commit_pair(&empty_bar[st], 0x3);
          else mma_commit(&empty_bar[st]);
        };
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase)) { fail(kErrTimeoutFull); ok = false; break; }
          tc_fence_after();
          if constexpr (kScaled) {
            if ((kb & 3) == 0) {
              const uint64_t da = smem_desc_sf(sSFA + stage * C::SFA_BYTES);
              if constexpr (PAIR == 2) tmem_cp_32x128b_x4_pair(tmem_base + C::kSfaCol, da);
              else tmem_cp_32x128b_x4(tmem_base + C::kSfaCol, da);
#pragma unroll
              for (int i = 0; i < BN / 128; ++i) {
                const uint64_t db = smem_desc_sf(sSFB + stage * C::SFB_BYTES + i * 512);
                if constexpr (PAIR == 2) tmem_cp_32x128b_x4_pair(tmem_base + C::kSfbCol + 4 * i, db);
                else tmem_cp_32x128b_x4(tmem_base + C::kSfbCol + 4 * i, db);
              }
            }
          }
          issue_half(free_half, stage, kb);
          if (ovl_ready) {
            issue_half(free_half ^ 1, stage, kb);
            release_stage(stage);
          } else {
            dstage[deferred++] = stage;
            if (deferred == kDefer || kb == nk - 1) {
              if (!mbar_wait(&tempty_ovl[s ^ 1], ((j - 1) >> 1) & 1)) { fail(kErrTimeoutTmem); ok = false; break; }
              tc_fence_after();
              for (int i = 0; i < deferred; ++i) {
                issue_half(free_half ^ 1, dstage[i], kb - deferred + 1 + i);
                release_stage(dstage[i]);
              }
              ovl_ready = true;
            }
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        if constexpr (PAIR == 2) mma_commit_pair(&tfull_bar[s], 0x3);
        else mma_commit(&tfull_bar[s]);
        ++j;
      }
    }
  } else if (warp >= 4) {
    // ================= epilogue: quadrant q = warp % 4, part h (column half, or query slot for the indexer) ======
    const uint32_t q = warp & 3;
    const uint32_t h = (warp - 4) >> 2;
    const int row_in_cta = int(q * 32 + lane);
    auto release = [&](uint64_t* bar) {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(leader_bar(bar));
    };
    int j = 0;
    for (int t = unit; t < num_tiles && !*abort_flag; t += n_units) {
      int mb, nb; tile_coords(t, mb, nb);
      if (skip_tile(mb, nb)) continue;
      const int s = j & 1;
      if (!mbar_wait(&tfull_bar[s], (j >> 1) & 1)) { fail(kErrTimeoutTmem); break; }
      tc_fence_after();
      const int row = mb * BM + int(rank) * 128 + row_in_cta;
      const bool row_ok = row < p.M && (p.row_valid == nullptr || p.row_valid[row] >= 0);
      const uint32_t t_row = tmem_base + ((q * 32) << 16) + (s ? C::kAcc1 : C::kAcc0);
      // the warp that owns this stage's overlap columns drains them first
      const bool ovl_first = C::kOvl > 0 && s == 0 && h == 1;       // stage 0: local columns [224,256)
      const bool ovl_owner = C::kOvl > 0 && ((s == 0 && h == 1) || (s == 1 && h == 0));

      if constexpr (EPI == EPI_BF16_SCATTER || EPI == EPI_BF16_ROWS || EPI == EPI_BF16_PUSH) {
        // A row-per-lane store would put 32 rows' 16-byte pieces into one warp instruction: 32 small NVLink writes
        // (scatter: rows go to their owners' slots in peer HBM) or 32 partial-sector L2 writes (local rows).
        // Instead each 64-column slab of the warp's 32 rows is staged in shared memory and written back
        // row-contiguous: one instruction covers four 128-byte row segments.  (Requires ldo % 8 == 0 and
        // N % 8 == 0, checked by the host.)
        uint8_t* stg = xstage + (warp - 4) * kScatterWarpBytes;
        __nv_bfloat16* my_base = nullptr;
        if (row_ok) {
          if constexpr (EPI == EPI_BF16_SCATTER) {
            int r = 0;
            while (r + 1 < p.scatter_world && row >= p.scatter_bounds[r + 1]) ++r;
            my_base = reinterpret_cast<__nv_bfloat16*>(p.scatter_ptrs[r]) +
                      (size_t(p.scatter_rank) * p.scatter_rows + (row - p.scatter_bounds[r])) * size_t(p.ldo);
          } else if constexpr (EPI == EPI_BF16_PUSH) {
            const int dst = p.row_dst[row];
            const int home = dst >> 24;
            if (dst >= 0 && home < p.scatter_world)
              my_base = reinterpret_cast<__nv_bfloat16*>(p.scatter_ptrs[home]) + size_t(dst & 0xffffff) * p.ldo;
          } else {
            my_base = reinterpret_cast<__nv_bfloat16*>(p.out) + size_t(row) * p.ldo;
          }
        }
        const uint64_t my_base_u = reinterpret_cast<uint64_t>(my_base);
#pragma unroll 1
        for (int pp = 0; pp < 2; ++pp) {
          const int slab = ovl_first ? 1 - pp : pp;          // ovl_first: the slab holding chunk 3 goes first
#pragma unroll 1
          for (int cc = 0; cc < 2; ++cc) {
            const int c = 2 * slab + (ovl_first ? 1 - cc : cc);
            const int lc = 128 * int(h) + 32 * c;
            uint32_t v[32];
            tmem_ld_32x32b_x32(t_row + lc, v);
            tmem_ld_wait();
            if (pp == 0 && cc == 0 && ovl_owner) release(&tempty_ovl[s]);
            uint4* d = reinterpret_cast<uint4*>(stg + lane * kScatterRowBytes + (c & 1) * 64);
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
              uint4 w;
              w.x = pack_bf16x2(__uint_as_float(v[8 * jj + 0]), __uint_as_float(v[8 * jj + 1]));
              w.y = pack_bf16x2(__uint_as_float(v[8 * jj + 2]), __uint_as_float(v[8 * jj + 3]));
              w.z = pack_bf16x2(__uint_as_float(v[8 * jj + 4]), __uint_as_float(v[8 * jj + 5]));
              w.w = pack_bf16x2(__uint_as_float(v[8 * jj + 6]), __uint_as_float(v[8 * jj + 7]));
              d[jj] = w;
            }
          }
          __syncwarp();
          const int col = nb * BN + 128 * int(h) + 64 * slab + 8 * int(lane & 7);
#pragma unroll
          for (int it = 0; it < 8; ++it) {
            const int r = 4 * it + int(lane >> 3);
            const uint64_t base = __shfl_sync(0xffffffffu, my_base_u, r);
            const uint4 w = *reinterpret_cast<const uint4*>(stg + r * kScatterRowBytes + (lane & 7) * 16);
            if (base != 0 && col < p.N) *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(base) + col) = w;
          }
          __syncwarp();
        }
        release(&tempty_full[s]);
      } else if constexpr (EPI == EPI_BF16) {
        __nv_bfloat16* row_base = reinterpret_cast<__nv_bfloat16*>(p.out) + size_t(row) * p.ldo;
#pragma unroll 1
        for (int i = 0; i < 4; ++i) {
          const int c = ovl_first ? ((i + 3) & 3) : i;
          const int lc = 128 * int(h) + 32 * c;
          uint32_t v[32];
          tmem_ld_32x32b_x32(t_row + lc, v);
          tmem_ld_wait();
          if (i == 0 && ovl_owner) release(&tempty_ovl[s]);
          const int col0 = nb * BN + lc;
          if (row_ok && col0 < p.N) {
            __nv_bfloat16* o = row_base + col0;
            if (col0 + 32 <= p.N && (p.ldo % 8) == 0) {
#pragma unroll
              for (int jj = 0; jj < 4; ++jj) {
                uint4 w;
                w.x = pack_bf16x2(__uint_as_float(v[8 * jj + 0]), __uint_as_float(v[8 * jj + 1]));
                w.y = pack_bf16x2(__uint_as_float(v[8 * jj + 2]), __uint_as_float(v[8 * jj + 3]));
                w.z = pack_bf16x2(__uint_as_float(v[8 * jj + 4]), __uint_as_float(v[8 * jj + 5]));
                w.w = pack_bf16x2(__uint_as_float(v[8 * jj + 6]), __uint_as_float(v[8 * jj + 7]));
                reinterpret_cast<uint4*>(o)[jj] = w;
              }
            } else {
#pragma unroll
              for (int jj = 0; jj < 32; ++jj)
                if (col0 + jj < p.N) o[jj] = __float2bfloat16_rn(__uint_as_float(v[jj]));
            }
          }
        }
        release(&tempty_full[s]);
      } else if constexpr (EPI == EPI_SWIGLU_FP8) {
        // tile columns: gate [0,128), up [128,256) for the tile's 128 output columns; half h owns outputs
        // [64h, 64h+64) in two chunks of 32
        float a0[32], a1[32];
        int oc0 = 0;
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int oc = ovl_first ? 1 - i : i;
          if (i == 0) oc0 = oc;
          const int o0 = 64 * int(h) + 32 * oc;
          uint32_t g[32], u[32];
          tmem_ld_32x32b_x32(t_row + o0, g);
          tmem_ld_32x32b_x32(t_row + 128 + o0, u);
          tmem_ld_wait();
          if (i == 0 && ovl_owner) release(&tempty_ovl[s]);
          float* a = i == 0 ? a0 : a1;
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) {
            float gv = __uint_as_float(g[jj]), uv = __uint_as_float(u[jj]);
            if (p.swiglu_limit > 0.f) { gv = fminf(gv, p.swiglu_limit); uv = fminf(fmaxf(uv, -p.swiglu_limit), p.swiglu_limit); }
            const float av = gv / (1.f + __expf(-gv)) * uv;
            a[jj] = av;
            amax = fmaxf(amax, fabsf(av));
          }
        }
        release(&tempty_full[s]);
        // one UE8M0 scale per row and 128 output columns: combine the two halves' amax
        float* xa = xamax + (j & 1) * 256;
        xa[h * 128 + row_in_cta] = amax;
        mbar_arrive(xbar);
        if (!mbar_wait(xbar, j & 1)) { fail(kErrTimeoutTmem); break; }
        amax = fmaxf(amax, xa[(h ^ 1) * 128 + row_in_cta]);
        {
          // quantised bytes of both column halves meet in the quadrant's staging rows; the two warps of the
          // quadrant then store whole 128-byte row segments (16 rows each), not 16-byte pieces of 32 rows
          const uint32_t sb = ue8m0_for_amax(amax);
          const float inv = ue8m0_inv(sb);
          uint8_t* qst = xstage + q * kSwiQuadBytes;
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const float* a = i == 0 ? a0 : a1;
            const int oc = i == 0 ? oc0 : 1 - oc0;
            uint4* o = reinterpret_cast<uint4*>(qst + lane * kScatterRowBytes + 64 * h + 32 * oc);
#pragma unroll
            for (int jj = 0; jj < 2; ++jj) {
              uint4 w;
              w.x = pack_fp8x4(a[16 * jj + 0] * inv, a[16 * jj + 1] * inv, a[16 * jj + 2] * inv, a[16 * jj + 3] * inv);
              w.y = pack_fp8x4(a[16 * jj + 4] * inv, a[16 * jj + 5] * inv, a[16 * jj + 6] * inv, a[16 * jj + 7] * inv);
              w.z = pack_fp8x4(a[16 * jj + 8] * inv, a[16 * jj + 9] * inv, a[16 * jj + 10] * inv, a[16 * jj + 11] * inv);
              w.w = pack_fp8x4(a[16 * jj + 12] * inv, a[16 * jj + 13] * inv, a[16 * jj + 14] * inv, a[16 * jj + 15] * inv);
              o[jj] = w;
            }
          }
          // each processed tile completes qbar[q] twice (staged, then stored): parities 0 and 1
          mbar_arrive(&qbar[q]);
          if (!mbar_wait(&qbar[q], 0)) { fail(kErrTimeoutTmem); break; }
          const int row0 = mb * BM + int(rank) * 128 + int(q) * 32;     // first row of this quadrant
#pragma unroll
          for (int it = 0; it < 4; ++it) {
            const int r = 16 * int(h) + 4 * it + int(lane >> 3);          // this warp's 16 rows, 4 per instruction
            const int ok = __shfl_sync(0xffffffffu, row_ok ? 1 : 0, r);    // lane r of either warp owns row r
            const uint4 w = *reinterpret_cast<const uint4*>(qst + r * kScatterRowBytes + (lane & 7) * 16);
            if (ok)
              *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(p.out) + size_t(row0 + r) * p.ldo + nb * 128 +
                                        (lane & 7) * 16) = w;
          }
          mbar_arrive(&qbar[q]);                                           // staging free for the next tile
          if (!mbar_wait(&qbar[q], 1)) { fail(kErrTimeoutTmem); break; }
        }
        if (row_ok) {
          const uint32_t sb = ue8m0_for_amax(amax);
          if (h == 0) {
            const int kbo = nb;                               // output k-block (128 columns per tile)
            const int rb = row / 128, r = row % 128;
            uint8_t* sf = reinterpret_cast<uint8_t*>(p.out_sf) +
                          ((size_t(kbo >> 2) * p.sfa_row_blocks + rb) * 128 + (r % 32) * 4 + (r / 32)) * 4 + (kbo & 3);
            *sf = uint8_t(sb);
          }
        }
      } else {
        // DSA indexer: A rows are keys, tile columns are qpt queries x H heads; part h of the quadrant owns queries
        // h, h + kParts, ...  logits[q, key] = sum_h w[q,h] * relu(acc[key, q*H + h]); -inf where key > q.
        const int H = p.idx_heads;
        const int qpt = BN / H;
        const int key = row;
#pragma unroll 1
        for (int jq = int(h); jq < qpt; jq += C::kParts) {
          const int qi = nb * qpt + jq;
          const bool q_ok = qi * H < p.N;
          const float* wq = p.idx_w + size_t(q_ok ? qi : 0) * H;
          float acc4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
          for (int c = 0; c < H; c += 32) {
            // two 16-column loads in flight, one wait (the head count is a multiple of 16)
            uint32_t v[32];
            uint32_t (&v0)[16] = *reinterpret_cast<uint32_t(*)[16]>(&v[0]);
            uint32_t (&v1)[16] = *reinterpret_cast<uint32_t(*)[16]>(&v[16]);
            const bool two = c + 16 < H;
            tmem_ld_32x32b_x16(t_row + jq * H + c, v0);
            if (two) tmem_ld_32x32b_x16(t_row + jq * H + c + 16, v1);
            const float4* w4 = reinterpret_cast<const float4*>(wq + c);
            float wv[32];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float4 x = (i < 4 || two) ? w4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
              wv[4 * i] = x.x; wv[4 * i + 1] = x.y; wv[4 * i + 2] = x.z; wv[4 * i + 3] = x.w;
            }
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 16; ++i) acc4[i & 3] = fmaf(wv[i], fmaxf(__uint_as_float(v[i]), 0.f), acc4[i & 3]);
            if (two)
#pragma unroll
              for (int i = 16; i < 32; ++i) acc4[i & 3] = fmaf(wv[i], fmaxf(__uint_as_float(v[i]), 0.f), acc4[i & 3]);
          }
          if (row_ok && q_ok) {
            float* o = reinterpret_cast<float*>(p.out) + size_t(qi) * p.ldo + key;
            *o = (p.causal && key > qi) ? -INFINITY : (acc4[0] + acc4[1]) + (acc4[2] + acc4[3]);
          }
        }
        if constexpr (C::kOvl > 0) release(&tempty_ovl[s]);       // fp8 (scaled) layout: stages share 32 columns
        release(&tempty_full[s]);
      }
      ++j;
    }
    if constexpr (EPI == EPI_BF16_SCATTER || EPI == EPI_BF16_PUSH)
      __threadfence_system();                                       // peer stores performed before any barrier
  }

  __syncthreads();
  if constexpr (PAIR == 2) cluster_sync();   // no cross-CTA signal or MMA into this CTA is still pending
  if (warp == 2) {
    tc_fence_after();
    if constexpr (PAIR == 2) tmem_dealloc_pair(tmem_base, 512);
    else tmem_dealloc(tmem_base, 512);
  }
#endif
}

}  // namespace cb
