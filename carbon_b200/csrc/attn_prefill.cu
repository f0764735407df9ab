// MLA prefill attention on tcgen05 (sm_100a): O = softmax(Q·Kᵀ·scale, causal [+ DSA key mask])·V
// per (sequence, head, 128-query tile).  Q/K head dim 192 (= 128 nope + 64 rope), V head dim 128, bf16 in/out.
//
// CTA roles (256 threads):
//   warp 0  TMA: Q once, then K tiles into a 2-deep ring          warp 3  TMA: V tiles (1 stage)
//   warp 1  MMA: S[j%2] = Q·K_jᵀ (TMEM), O += P_j·V_j (TMEM)        warp 2  TMEM allocator
//   warps 4-11 softmax: two warps per TMEM lane quadrant, each one query row x 64 score columns per thread;
//            row max exchanged through shared memory; P (bf16) to shared memory in the 128B-swizzled K-major
//            layout the MMA reads; lazy rescale of O in TMEM (only when the row max grows by > 2^8); O/l out.
//            Tiles wholly below the diagonal and without a DSA mask skip the per-key mask work.
// TMEM: S0 cols [0,128), S1 [128,256), O [256,384).
// Shared memory: Q 48 KB | K 2 x 48 KB | V 32 KB | P 32 KB  (= 208 KB) + barriers.
//
// The DSA variant passes a bit matrix mask[T, W] (bit j of word w = key 32w+j of the query's sequence allowed):
// the indexer's top-k selection is applied inside the dense causal tile loop.  Reference kernel with the same
// role: the FlashMLA-derived sparse prefill (king_v10/bundle_v9/cuda_prefill_attn.py:1449), whose head layout
// (latent MQA 64x512) differs from this model's MLA (128 heads, 192/128).
#include <cudaTypedefs.h>
#include "ptx.cuh"

namespace cb {

bool make_tmap_2d(CUtensorMap* m, const void* ptr, CUtensorMapDataType dt, int elem_bytes, uint64_t inner,
                  uint64_t rows, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows,
                  CUtensorMapSwizzle swz);

namespace fa {

constexpr int BM = 128, BN = 128, DQK = 192, DV = 128;
constexpr int Q_BYTES = BM * DQK * 2;          // 48 KB (3 swizzle atoms of 64 dims)
constexpr int K_BYTES = BN * DQK * 2;          // 48 KB
constexpr int V_BYTES = BN * DV * 2;           // 32 KB (2 atoms of 64 dims)
constexpr int P_BYTES = BM * BN * 2;           // 32 KB (2 atoms of 64 keys)
constexpr int ATOM = 128 * 128;                // bytes of one [128 rows x 128 B] swizzled box
constexpr int SMEM = 1024 + Q_BYTES + 2 * K_BYTES + V_BYTES + P_BYTES + 256 + 2048 + 64;
constexpr float kRescaleThresh = 8.0f;         // log2 units

struct Params {
  const int4* tiles;      // [n_tiles] (seq_start, seq_len, q0, unused)
  const uint32_t* mask;   // optional [T, mask_words]
  int mask_words;
  int H;
  float scale_log2;       // softmax scale * log2(e)
  __nv_bfloat16* out;     // [T, H, DV]
  int* status;
  // optional event trace of CTA (0,0) (two-tile kernel): [0] = event count, then (clock64, kind<<32 | t<<16 | j)
  unsigned long long* trace;
  int trace_cap;
  const float* sink;      // optional [H]: per-head sink logit (softmax units; one extra denominator term)
};

// Records one event of the traced CTA (kinds: 1 MMA saw P ready, 2 MMA issued PV+QK, 3 softmax waits for S,
// 4 S arrived, 5 P written).
CB_DEVICE void trace_event(const Params& p, int kind, int t, int j) {
  if (p.trace == nullptr || blockIdx.x != 0 || blockIdx.y != 0) return;
  const unsigned long long i = atomicAdd(p.trace, 1ull);
  if (int(i) < p.trace_cap) {
    p.trace[1 + 2 * i] = clock64();
    p.trace[2 + 2 * i] = (static_cast<unsigned long long>(kind) << 32) | (static_cast<unsigned long long>(t) << 16) |
                         static_cast<unsigned long long>(j);
  }
}

// MN-major (V as the B operand, N = dv contiguous) 128B-swizzled descriptor: LBO = bytes between 64-wide dv
// atoms, SBO = bytes between 8-row key groups.
CB_DEVICE uint64_t desc_mn_sw128(const void* p, uint32_t lbo, uint32_t sbo) {
  const uint64_t addr = smem_u32(p);
  uint64_t d = 0;
  d |= (addr >> 4) & 0x3FFFull;
  d |= uint64_t((lbo >> 4) & 0x3FFF) << 16;
  d |= uint64_t((sbo >> 4) & 0x3FFF) << 32;
  d |= uint64_t(1) << 46;
  d |= uint64_t(2) << 61;
  return d;
}

// 2^x with the hardware approximation (MUFU ex2, flush-to-zero); softmax inputs are <= 0 after the max shift.
CB_DEVICE float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

CB_HOST_DEVICE uint32_t idesc_bf16_bmn(int M, int N) {  // A K-major, B MN-major
  return idesc_bf16(M, N) | (1u << 16);
}

// tm_kv: the wkv_b output [T, H, 256] (k_nope dims 0..127 | v dims 128..255); tm_kpe: the shared RoPE key [T, 64].
__global__ void __launch_bounds__(384, 1) attn_prefill_kernel(const __grid_constant__ CUtensorMap tm_q,
                                                              const __grid_constant__ CUtensorMap tm_kv,
                                                              const __grid_constant__ CUtensorMap tm_kpe,
                                                              const Params p) {
  cb::pdl_entry();
#if defined(__CUDA_ARCH__) && __CUDA_ARCH__ >= 1000
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + Q_BYTES;                 // 2 stages
  uint8_t* sV = sK + 2 * K_BYTES;
  uint8_t* sP = sV + V_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + P_BYTES);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;    // [2]
  uint64_t* k_empty = bars + 3;   // [2]
  uint64_t* v_full = bars + 5;
  uint64_t* v_empty = bars + 6;
  uint64_t* s_full = bars + 7;    // [2]
  uint64_t* s_empty = bars + 9;   // [2]
  uint64_t* p_full = bars + 11;
  uint64_t* pv_done = bars + 12;
  uint64_t* x_bar = bars + 13;    // [2] row-max / row-sum exchange between the two softmax halves
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 15);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int4 tile = p.tiles[blockIdx.x];
  const int seq_start = tile.x, seq_len = tile.y, q0 = tile.z;
  const int h = blockIdx.y;
  const int q_end = min(q0 + BM, seq_len);
  const int n_kt = (q_end + BN - 1) / BN;     // causal: keys [0, q_end)

  const uint32_t warp = warp_id(), lane = lane_id();
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) { mbar_init(&k_full[i], 1); mbar_init(&k_empty[i], 1);
                                  mbar_init(&s_full[i], 1); mbar_init(&s_empty[i], 256); }
    mbar_init(v_full, 1); mbar_init(v_empty, 1); mbar_init(p_full, 256); mbar_init(pv_done, 1);
    mbar_init(&x_bar[0], 256); mbar_init(&x_bar[1], 256);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 2) { tmem_alloc(tmem_slot, 512); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto fail = [&](int code) { if (p.status) atomicCAS(p.status, 0, code); *abort_flag = 1; };

  if (warp == 0) {
    if (elect_one()) {
      tma_prefetch_desc(&tm_q); tma_prefetch_desc(&tm_kv); tma_prefetch_desc(&tm_kpe);
      mbar_arrive_expect_tx(q_full, Q_BYTES);
      for (int a = 0; a < 3; ++a) tma_load_3d(sQ + a * ATOM, &tm_q, q_full, a * 64, h, seq_start + q0);
      for (int j = 0; j < n_kt && !*abort_flag; ++j) {
        const int s = j & 1;
        if (!mbar_wait(&k_empty[s], ((j >> 1) & 1) ^ 1)) { fail(kErrTimeoutEmpty); break; }
        mbar_arrive_expect_tx(&k_full[s], K_BYTES);
        for (int a = 0; a < 2; ++a)
          tma_load_3d(sK + s * K_BYTES + a * ATOM, &tm_kv, &k_full[s], a * 64, h, seq_start + j * BN);
        tma_load_2d(sK + s * K_BYTES + 2 * ATOM, &tm_kpe, &k_full[s], 0, seq_start + j * BN);
      }
    }
  } else if (warp == 3) {
    if (elect_one()) {
      for (int j = 0; j < n_kt && !*abort_flag; ++j) {
        if (!mbar_wait(v_empty, (j & 1) ^ 1)) { fail(kErrTimeoutEmpty); break; }
        mbar_arrive_expect_tx(v_full, V_BYTES);
        for (int a = 0; a < 2; ++a) tma_load_3d(sV + a * ATOM, &tm_kv, v_full, 128 + a * 64, h, seq_start + j * BN);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      const uint32_t id_qk = idesc_bf16(BM, BN);
      const uint32_t id_pv = idesc_bf16_bmn(BM, DV);
      bool ok = mbar_wait(q_full, 0);
      if (!ok) fail(kErrTimeoutFull);
      auto issue_qk = [&](int j) -> bool {
        const int s = j & 1;
        if (!mbar_wait(&k_full[s], (j >> 1) & 1)) { fail(kErrTimeoutFull); return false; }
        if (!mbar_wait(&s_empty[s], ((j >> 1) & 1) ^ 1)) { fail(kErrTimeoutTmem); return false; }
        tc_fence_after();
        for (int k = 0; k < DQK / 16; ++k) {
          const int a = k >> 2, off = (k & 3) * 32;
          mma_f16_ss(tmem + s * 128, smem_desc_sw128(sQ + a * ATOM + off),
                     smem_desc_sw128(sK + s * K_BYTES + a * ATOM + off), id_qk, k > 0);
        }
        mma_commit(&s_full[s]);
        mma_commit(&k_empty[s]);
        return true;
      };
      auto issue_pv = [&](int j) -> bool {
        if (!mbar_wait(p_full, j & 1)) { fail(kErrTimeoutFull); return false; }
        if (!mbar_wait(v_full, j & 1)) { fail(kErrTimeoutFull); return false; }
        tc_fence_after();
        for (int k = 0; k < BN / 16; ++k) {
          // A = P (K-major, keys along K): atom k/4, 32-byte step inside the atom
          const uint64_t a_desc = smem_desc_sw128(sP + (k >> 2) * ATOM + (k & 3) * 32);
          // B = V (MN-major): 16 keys = 16 rows of 128 B
          const uint64_t b_desc = desc_mn_sw128(sV + k * 16 * 128, ATOM, 1024);
          mma_f16_ss(tmem + 256, a_desc, b_desc, id_pv, (j > 0 || k > 0) ? 1u : 0u);
        }
        mma_commit(pv_done);
        mma_commit(v_empty);
        return true;
      };
      if (ok) ok = issue_qk(0);
      for (int j = 0; ok && j < n_kt && !*abort_flag; ++j) {
        if (j + 1 < n_kt) ok = issue_qk(j + 1);
        if (ok) ok = issue_pv(j);
      }
    }
  } else if (warp >= 4) {
    // ---------------- softmax / correction / epilogue: 8 warps, two per TMEM lane quadrant ----------------
    // warp (4 + half*4 + q) owns rows 32q..32q+31 and score columns [64*half, 64*half + 64).
    const uint32_t q = warp & 3;
    const int half = int(warp - 4) >> 2;
    const int row = q * 32 + lane;               // query row within the tile
    const int qi = q0 + row;                     // query index within the sequence
    const int tok = seq_start + qi;
    const uint32_t t_lane = tmem + ((q * 32) << 16);
    // [2 parities][2 halves][128 rows]: row maxima, and after the loop the row sums
    float* red = reinterpret_cast<float*>(const_cast<int*>(abort_flag) + 1);
    auto exchange = [&](int it, float v, float& other) -> bool {
      float* slot = red + (it & 1) * 256;
      slot[half * 128 + row] = v;
      mbar_arrive(&x_bar[it & 1]);
      if (!mbar_wait(&x_bar[it & 1], (it >> 1) & 1)) return false;
      other = slot[(half ^ 1) * 128 + row];
      return true;
    };
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kt; ++j) {
      const int s = j & 1;
      if (!mbar_wait(&s_full[s], (j >> 1) & 1)) { fail(kErrTimeoutTmem); ok = false; break; }
      tc_fence_after();
      float sv[64];
      {
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_lane + s * 128 + half * 64, r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) sv[i] = __uint_as_float(r[i]);
        tmem_ld_32x32b_x32(t_lane + s * 128 + half * 64 + 32, r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) sv[32 + i] = __uint_as_float(r[i]);
      }
      tc_fence_before();
      mbar_arrive(&s_empty[s]);
      const int k0 = j * BN + half * 64;
      float mt = -INFINITY;
      const bool dense_tile = (p.mask == nullptr) && (j * BN + BN - 1 <= q0);   // every key <= every query
      if (dense_tile) {
#pragma unroll
        for (int i = 0; i < 64; ++i) mt = fmaxf(mt, sv[i]);
        mt *= p.scale_log2;
      } else {
        uint32_t w0 = 0xffffffffu, w1 = 0xffffffffu;
        if (p.mask && qi < seq_len) {
          const int wi = k0 >> 5;
          w0 = wi < p.mask_words ? p.mask[size_t(tok) * p.mask_words + wi] : 0u;
          w1 = wi + 1 < p.mask_words ? p.mask[size_t(tok) * p.mask_words + wi + 1] : 0u;
        }
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          const uint32_t bit = ((i < 32 ? w0 : w1) >> (i & 31)) & 1u;
          const bool allowed = (k0 + i <= qi) && bit;
          sv[i] = allowed ? sv[i] : -INFINITY;
          mt = fmaxf(mt, sv[i]);
        }
        mt = mt == -INFINITY ? mt : mt * p.scale_log2;
      }
      // row max across the two column halves
      float mt_other;
      if (!exchange(j, mt, mt_other)) { fail(kErrTimeoutTmem); ok = false; break; }
      mt = fmaxf(mt, mt_other);
      const bool need = (j > 0) && (mt > m_used + kRescaleThresh);
      const float m_new = (need || j == 0) ? fmaxf(m_used, mt) : m_used;
      const float m_ref = m_new == -INFINITY ? 0.f : m_new;
      float alpha = 1.f;
      if (need && m_used != -INFINITY) alpha = fast_exp2(m_used - m_ref);
      float rs = 0.f;
      uint32_t pk[32];
#pragma unroll
      for (int i = 0; i < 64; i += 2) {
        const float a = fast_exp2(fmaf(sv[i], p.scale_log2, -m_ref));
        const float b = fast_exp2(fmaf(sv[i + 1], p.scale_log2, -m_ref));
        rs += a + b;
        pk[i / 2] = pack_bf16x2(a, b);
      }
      l = l * alpha + rs;
      m_used = m_new;
      if (j > 0) {
        if (!mbar_wait(pv_done, (j - 1) & 1)) { fail(kErrTimeoutTmem); ok = false; break; }
        tc_fence_after();
        if (__any_sync(0xffffffffu, need)) {
#pragma unroll 1
          for (int c = 0; c < 64; c += 16) {
            uint32_t r[16];
            tmem_ld_32x32b_x16(t_lane + 256 + half * 64 + c, r);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 16; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
            tmem_st_32x32b_x16(t_lane + 256 + half * 64 + c, r);
          }
          tmem_st_wait();
        }
      }
      // P: this half's 64 keys form swizzle atom `half` of the P tile
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint8_t* dst = sP + half * ATOM + row * 128 + ((c ^ (row & 7)) << 4);
        *reinterpret_cast<uint4*>(dst) = make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
      }
      fence_proxy_async();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok && n_kt > 0) {
      if (!mbar_wait(pv_done, (n_kt - 1) & 1)) { fail(kErrTimeoutTmem); ok = false; }
    }
    // full row sum = sum of the two halves' partial sums (alpha sequences are identical in both halves)
    float l_other = 0.f;
    if (ok && !exchange(n_kt, l, l_other)) { fail(kErrTimeoutTmem); ok = false; }
    l += l_other;
    if (p.sink) l += fast_exp2(p.sink[h] * 1.4426950408889634f - (m_used == -INFINITY ? 0.f : m_used));
    if (ok) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* o = p.out + (size_t(tok) * p.H + h) * DV + half * 64;
#pragma unroll 1
      for (int c = 0; c < 64; c += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_lane + 256 + half * 64 + c, r);
        tmem_ld_wait();
        if (qi < seq_len) {
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(r[8 * v + 0]) * inv, __uint_as_float(r[8 * v + 1]) * inv);
            w.y = pack_bf16x2(__uint_as_float(r[8 * v + 2]) * inv, __uint_as_float(r[8 * v + 3]) * inv);
            w.z = pack_bf16x2(__uint_as_float(r[8 * v + 4]) * inv, __uint_as_float(r[8 * v + 5]) * inv);
            w.w = pack_bf16x2(__uint_as_float(r[8 * v + 6]) * inv, __uint_as_float(r[8 * v + 7]) * inv);
            reinterpret_cast<uint4*>(o + c)[v] = w;
          }
        }
      }
    }
  }
  __syncthreads();
  if (warp == 2) { tc_fence_after(); tmem_dealloc(tmem, 512); }
#endif
}

static bool make_tmap_3d(CUtensorMap* m, const void* ptr, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1,
                         uint64_t s2, uint32_t b0, uint32_t b1, uint32_t b2);

}  // namespace fa

// ---------------------------------------------------------------------------------------------------------------
// Two-tile variant: one CTA runs two 128-row Q tiles of the same (sequence, head) against each K/V tile.
//
//   warp 0  TMA: Q0/Q1 once, then K(j) (3 chunks: k_nope 0-63, 64-127, shared RoPE key) and V(j) (2 chunks) into a
//           FIFO ring of NCH 16 KB chunks, so V(j+1) streams in as soon as K(j) has been consumed
//   warp 1  MMA, issue order  QK0(0) QK1(0) | PV0(0) QK0(1) PV1(0) QK1(1) | PV0(1) QK0(2) ...: while the softmax of
//           one tile runs, the tensor core works on the other tile
//   warp 2  TMEM allocator
//   warps 4-7 / 8-11  softmax of tile 0 / tile 1: one query row per thread (all 128 scores in registers, no
//           cross-warp reduction), lazy O rescale, P written back into TMEM over S as bf16 and read by the PV MMA
//           straight from TMEM (A operand in tensor memory); O/l written out at the end
// TMEM: tile t uses columns [256t, 256t+128) for S (P in its first 64 columns) and [256t+128, 256t+256) for O.
// ---------------------------------------------------------------------------------------------------------------
namespace fa2 {

constexpr int BM = 128, BN = 128, DQK = 192, DV = 128;
constexpr int ATOM = 128 * 128;                 // one [128 rows x 128 B] swizzled box = one ring chunk
constexpr int Q_BYTES = 3 * ATOM;               // 48 KB per Q tile
constexpr int NCH = 8;                          // ring chunks (K = 3, V = 2 per KV tile)
constexpr int CH_PER_KV = 5;
constexpr int SMEM = 1024 + 2 * Q_BYTES + NCH * ATOM + 512;
constexpr float kRescaleThresh = 8.0f;

__global__ void __launch_bounds__(384, 1) attn_prefill2_kernel(const __grid_constant__ CUtensorMap tm_q,
                                                               const __grid_constant__ CUtensorMap tm_kv,
                                                               const __grid_constant__ CUtensorMap tm_kpe,
                                                               const fa::Params p) {
  cb::pdl_entry();
#if defined(__CUDA_ARCH__) && __CUDA_ARCH__ >= 1000
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                          // [2 tiles][3 atoms]
  uint8_t* sR = sQ + 2 * Q_BYTES;              // ring [NCH][ATOM]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sR + NCH * ATOM);
  uint64_t* q_full = bars;                     // 1
  uint64_t* r_full = bars + 1;                 // [NCH]
  uint64_t* r_empty = bars + 1 + NCH;          // [NCH]
  uint64_t* s_full = bars + 1 + 2 * NCH;       // [2]
  uint64_t* p_full = bars + 3 + 2 * NCH;       // [2]
  uint64_t* o_done = bars + 5 + 2 * NCH;       // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 7 + 2 * NCH);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int4 tile = p.tiles[blockIdx.x];
  const int seq_start = tile.x, seq_len = tile.y, q0 = tile.z;
  const int h = blockIdx.y;
  int n_kt_t[2];
  for (int t = 0; t < 2; ++t) {
    const int qt0 = q0 + BM * t;
    n_kt_t[t] = qt0 < seq_len ? (min(qt0 + BM, seq_len) + BN - 1) / BN : 0;
  }
  const int n_kt = max(n_kt_t[0], n_kt_t[1]);
  const bool two = n_kt_t[1] > 0;

  const uint32_t warp = warp_id(), lane = lane_id();
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < NCH; ++i) { mbar_init(&r_full[i], 1); mbar_init(&r_empty[i], 1); }
    for (int t = 0; t < 2; ++t) { mbar_init(&s_full[t], 1); mbar_init(&p_full[t], 128); mbar_init(&o_done[t], 1); }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 2) { tmem_alloc(tmem_slot, 512); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto fail = [&](int code) { if (p.status) atomicCAS(p.status, 0, code); *abort_flag = 1; };
  auto chunk = [&](int idx) -> uint8_t* { return sR + (idx % NCH) * ATOM; };

  if (warp == 0) {
    // ================= TMA producer =================
    if (elect_one()) {
      tma_prefetch_desc(&tm_q); tma_prefetch_desc(&tm_kv); tma_prefetch_desc(&tm_kpe);
      mbar_arrive_expect_tx(q_full, (two ? 2 : 1) * Q_BYTES);
      for (int t = 0; t < (two ? 2 : 1); ++t)
        for (int a = 0; a < 3; ++a)
          tma_load_3d(sQ + t * Q_BYTES + a * ATOM, &tm_q, q_full, a * 64, h, seq_start + q0 + BM * t);
      for (int idx = 0; idx < n_kt * CH_PER_KV && !*abort_flag; ++idx) {
        const int slot = idx % NCH, use = idx / NCH;
        if (!mbar_wait(&r_empty[slot], (use & 1) ^ 1)) { fail(kErrTimeoutEmpty); break; }
        mbar_arrive_expect_tx(&r_full[slot], ATOM);
        const int j = idx / CH_PER_KV, c = idx % CH_PER_KV;
        const int row = seq_start + j * BN;
        if (c < 2) tma_load_3d(sR + slot * ATOM, &tm_kv, &r_full[slot], c * 64, h, row);          // k_nope
        else if (c == 2) tma_load_2d(sR + slot * ATOM, &tm_kpe, &r_full[slot], 0, row);            // RoPE key
        else tma_load_3d(sR + slot * ATOM, &tm_kv, &r_full[slot], 128 + (c - 3) * 64, h, row);    // v
      }
    }
  } else if (warp == 1) {
    // ================= MMA issuer =================
    if (elect_one()) {
      const uint32_t id_qk = idesc_bf16(BM, BN);
      const uint32_t id_pv = fa::idesc_bf16_bmn(BM, 64);
      bool ok = mbar_wait(q_full, 0);
      if (!ok) fail(kErrTimeoutFull);
      auto wait_chunks = [&](int first, int n) -> bool {
        for (int i = 0; i < n; ++i) {
          const int idx = first + i;
          if (!mbar_wait(&r_full[idx % NCH], (idx / NCH) & 1)) { fail(kErrTimeoutFull); return false; }
        }
        tc_fence_after();
        return true;
      };
      auto release_chunks = [&](int first, int n) {
        for (int i = 0; i < n; ++i) mma_commit(&r_empty[(first + i) % NCH]);
      };
      auto qk = [&](int t, int j) {
        const int kc = j * CH_PER_KV;
#pragma unroll
        for (int k = 0; k < DQK / 16; ++k) {
          const int a = k >> 2, off = (k & 3) * 32;
          mma_f16_ss(tmem + 256 * t, smem_desc_sw128(sQ + t * Q_BYTES + a * ATOM + off),
                     smem_desc_sw128(chunk(kc + a) + off), id_qk, k > 0);
        }
        mma_commit(&s_full[t]);
      };
      auto pv = [&](int t, int j) {
        const int vc = j * CH_PER_KV + 3;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint8_t* v = chunk(vc + half);
#pragma unroll
          for (int k = 0; k < BN / 16; ++k) {
            // A = P from TMEM: 16 keys = 8 columns of packed bf16; B = V chunk (MN-major, 64 dv wide)
            mma_f16_ts(tmem + 256 * t + 128 + 64 * half, tmem + 256 * t + 8 * k,
                       fa::desc_mn_sw128(v + k * 16 * 128, ATOM, 1024), id_pv, (j > 0 || k > 0) ? 1u : 0u);
          }
        }
        mma_commit(&o_done[t]);
      };
      if (ok && n_kt > 0) {
        ok = wait_chunks(0, 3);
        if (ok) {
          qk(0, 0);
          if (two) qk(1, 0);
          release_chunks(0, 3);
        }
      }
      for (int j = 0; ok && j < n_kt && !*abort_flag; ++j) {
        bool v_ready = false, k_ready = false;
        for (int t = 0; t < 2 && ok; ++t) {
          if (j >= n_kt_t[t]) continue;
          if (!mbar_wait(&p_full[t], j & 1)) { fail(kErrTimeoutTmem); ok = false; break; }
          fa::trace_event(p, 1, t, j);
          tc_fence_after();
          if (!v_ready) { ok = wait_chunks(j * CH_PER_KV + 3, 2); v_ready = true; if (!ok) break; }
          pv(t, j);
          if (j + 1 < n_kt_t[t]) {
            if (!k_ready) { ok = wait_chunks((j + 1) * CH_PER_KV, 3); k_ready = true; if (!ok) break; }
            qk(t, j + 1);
          }
          fa::trace_event(p, 2, t, j);
        }
        if (!ok) break;
        release_chunks(j * CH_PER_KV + 3, 2);
        if (j + 1 < n_kt) release_chunks((j + 1) * CH_PER_KV, 3);
      }
    }
  } else if (warp >= 4) {
    // ================= softmax: tile t = (warp-4)/4, TMEM lane quadrant q, one query row per thread =================
    const int t = int(warp - 4) >> 2;
    const uint32_t q = warp & 3;
    const int row = int(q * 32 + lane);
    const int qt0 = q0 + BM * t;
    const int qi = qt0 + row;
    const int tok = seq_start + qi;
    const uint32_t t_lane = tmem + ((q * 32) << 16) + 256 * t;
    const int nkt = n_kt_t[t];
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    const bool tracer = (q == 0 && lane == 0);
    // DSA mask words of a step are fetched one step ahead, off the softmax's critical path
    const bool use_mask = p.mask != nullptr && qi < seq_len;
    auto load_mask = [&](int jj, uint32_t (&w)[4]) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int wi = ((jj * BN) >> 5) + c;
        w[c] = wi < p.mask_words ? p.mask[size_t(tok) * p.mask_words + wi] : 0u;
      }
    };
    uint32_t mwn[4] = {0xffffffffu, 0xffffffffu, 0xffffffffu, 0xffffffffu};
    if (use_mask && nkt > 0) load_mask(0, mwn);
    for (int j = 0; j < nkt; ++j) {
      if (tracer) fa::trace_event(p, 3, t, j);
      if (!mbar_wait(&s_full[t], j & 1)) { fail(kErrTimeoutTmem); ok = false; break; }
      if (tracer) fa::trace_event(p, 4, t, j);
      tc_fence_after();
      float sv[128];
      {
        uint32_t (&r0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&sv[0]);
        uint32_t (&r1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&sv[32]);
        uint32_t (&r2)[32] = *reinterpret_cast<uint32_t(*)[32]>(&sv[64]);
        uint32_t (&r3)[32] = *reinterpret_cast<uint32_t(*)[32]>(&sv[96]);
        tmem_ld_32x32b_x32(t_lane + 0, r0);
        tmem_ld_32x32b_x32(t_lane + 32, r1);
        tmem_ld_32x32b_x32(t_lane + 64, r2);
        tmem_ld_32x32b_x32(t_lane + 96, r3);
        tmem_ld_wait();
      }
      const int k0 = j * BN;
      float mt = -INFINITY;
      uint32_t mw[4] = {mwn[0], mwn[1], mwn[2], mwn[3]};
      if (use_mask && j + 1 < nkt) load_mask(j + 1, mwn);    // next step's words load under this step's work
      // no per-key work when every row of the warp sees all 128 keys (below the diagonal, mask words all ones:
      // e.g. DSA rows with fewer candidates than top-k)
      const bool full_row = (k0 + BN - 1 <= qi) && ((mw[0] & mw[1] & mw[2] & mw[3]) == 0xffffffffu);
      if (__all_sync(0xffffffffu, full_row)) {
#pragma unroll
        for (int i = 0; i < 128; ++i) mt = fmaxf(mt, sv[i]);
        mt *= p.scale_log2;
      } else {
#pragma unroll
        for (int i = 0; i < 128; ++i) {
          const bool allowed = (k0 + i <= qi) && ((mw[i >> 5] >> (i & 31)) & 1u);
          sv[i] = allowed ? sv[i] : -INFINITY;
          mt = fmaxf(mt, sv[i]);
        }
        mt = mt == -INFINITY ? mt : mt * p.scale_log2;
      }
      const bool need = (j > 0) && (mt > m_used + kRescaleThresh);
      const float m_new = (need || j == 0) ? fmaxf(m_used, mt) : m_used;
      const float m_ref = m_new == -INFINITY ? 0.f : m_new;
      float alpha = 1.f;
      if (need && m_used != -INFINITY) alpha = fa::fast_exp2(m_used - m_ref);
      if (j > 0 && __any_sync(0xffffffffu, need)) {
        // O still holds the sums of earlier tiles at the old max: wait for the last PV, then rescale in TMEM
        if (!mbar_wait(&o_done[t], (j - 1) & 1)) { fail(kErrTimeoutTmem); ok = false; break; }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < 128; c += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(t_lane + 128 + c, r);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
          tmem_st_32x32b_x32(t_lane + 128 + c, r);
        }
      }
      float rs = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float a = fa::fast_exp2(fmaf(sv[32 * c + 2 * i], p.scale_log2, -m_ref));
          const float b = fa::fast_exp2(fmaf(sv[32 * c + 2 * i + 1], p.scale_log2, -m_ref));
          rs += a + b;
          pk[i] = pack_bf16x2(a, b);
        }
        tmem_st_32x32b_x16(t_lane + 16 * c, pk);     // P over the first 64 columns of S
      }
      l = l * alpha + rs;
      m_used = m_new;
      tmem_st_wait();
      tc_fence_before();
      if (tracer) fa::trace_event(p, 5, t, j);
      mbar_arrive(&p_full[t]);
    }
    if (ok && nkt > 0) {
      if (!mbar_wait(&o_done[t], (nkt - 1) & 1)) { fail(kErrTimeoutTmem); ok = false; }
    }
    if (p.sink) l += fa::fast_exp2(p.sink[h] * 1.4426950408889634f - (m_used == -INFINITY ? 0.f : m_used));
    if (ok && nkt > 0) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* o = p.out + (size_t(tok) * p.H + h) * DV;
#pragma unroll 1
      for (int c = 0; c < DV; c += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_lane + 128 + c, r);
        tmem_ld_wait();
        if (qi < seq_len) {
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(r[8 * v + 0]) * inv, __uint_as_float(r[8 * v + 1]) * inv);
            w.y = pack_bf16x2(__uint_as_float(r[8 * v + 2]) * inv, __uint_as_float(r[8 * v + 3]) * inv);
            w.z = pack_bf16x2(__uint_as_float(r[8 * v + 4]) * inv, __uint_as_float(r[8 * v + 5]) * inv);
            w.w = pack_bf16x2(__uint_as_float(r[8 * v + 6]) * inv, __uint_as_float(r[8 * v + 7]) * inv);
            reinterpret_cast<uint4*>(o + c)[v] = w;
          }
        }
      }
    }
  }
  __syncthreads();
  if (warp == 2) { tc_fence_after(); tmem_dealloc(tmem, 512); }
#endif
}

}  // namespace fa2

// ---------------------------------------------------------------------------------------------------------------
// Two-tile kernel with 64-key steps and double-buffered S (the default): per step a KV tile of 64 keys is 40 KB,
// so the 16-slot ring (8 KB chunks) holds three steps of K/V and loads run well ahead; each Q tile has two 64-column
// S buffers in TMEM, so QK(j+2) is issued right after PV(j) and the softmax of a tile runs back to back.
//   MMA order: QK0(0) QK1(0) QK0(1) QK1(1) | PV0(0) QK0(2) PV1(0) QK1(2) | PV0(1) QK0(3) ...
// TMEM of tile t: S buffers at 256t + {0, 64} (P, bf16, over the first 32 columns of the buffer), O at 256t + 128.
// ---------------------------------------------------------------------------------------------------------------
namespace fa3 {

constexpr int BM = 128, BN = 64, DQK = 192, DV = 128;
constexpr int QATOM = 128 * 128;                // Q: 128 rows x 64 dims
constexpr int Q_BYTES = 3 * QATOM;
constexpr int CH = 64 * 128;                    // ring chunk: 64 keys x 64 dims (one 128-byte-swizzled box)
constexpr int NCH = 16;
constexpr int CH_PER_KV = 5;                    // K: k_nope 0-63, 64-127, RoPE key; V: dv 0-63, 64-127
constexpr int SMEM = 1024 + 2 * Q_BYTES + NCH * CH + 512;
constexpr float kRescaleThresh = 8.0f;

__global__ void __launch_bounds__(384, 1) attn_prefill3_kernel(const __grid_constant__ CUtensorMap tm_q,
                                                               const __grid_constant__ CUtensorMap tm_kv,
                                                               const __grid_constant__ CUtensorMap tm_kpe,
                                                               const fa::Params p) {
  cb::pdl_entry();
#if defined(__CUDA_ARCH__) && __CUDA_ARCH__ >= 1000
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sR = sQ + 2 * Q_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sR + NCH * CH);
  uint64_t* q_full = bars;                     // 1
  uint64_t* r_full = bars + 1;                 // [NCH]
  uint64_t* r_empty = bars + 1 + NCH;          // [NCH]
  uint64_t* s_full = bars + 1 + 2 * NCH;       // [2 tiles][2 buffers]
  // P(j) ready, one barrier per S buffer: with double-buffered S the softmax of a tile can finish step j+1 before
  // the MMA warp waits for step j, so a single barrier could be two phases ahead of its waiter (parity aliasing)
  uint64_t* p_full = bars + 5 + 2 * NCH;       // [2 tiles][2 buffers]
  // PV(j) done, also one barrier per step parity: the softmax can finish while PV(j-1) is still pending, so a
  // single barrier could be two phases behind the PV that a waiter needs
  uint64_t* o_done = bars + 9 + 2 * NCH;       // [2 tiles][2 step parities]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13 + 2 * NCH);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int4 tile = p.tiles[blockIdx.x];
  const int seq_start = tile.x, seq_len = tile.y, q0 = tile.z;
  const int h = blockIdx.y;
  int n_kt_t[2];
  for (int t = 0; t < 2; ++t) {
    const int qt0 = q0 + BM * t;
    n_kt_t[t] = qt0 < seq_len ? (min(qt0 + BM, seq_len) + BN - 1) / BN : 0;
  }
  const int n_kt = max(n_kt_t[0], n_kt_t[1]);
  const bool two = n_kt_t[1] > 0;

  const uint32_t warp = warp_id(), lane = lane_id();
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < NCH; ++i) { mbar_init(&r_full[i], 1); mbar_init(&r_empty[i], 1); }
    for (int i = 0; i < 4; ++i) mbar_init(&s_full[i], 1);
    for (int i = 0; i < 4; ++i) mbar_init(&p_full[i], 128);
    for (int i = 0; i < 4; ++i) mbar_init(&o_done[i], 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 2) { tmem_alloc(tmem_slot, 512); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto fail = [&](int code) { if (p.status) atomicCAS(p.status, 0, code); *abort_flag = 1; };
  auto chunk = [&](int idx) -> uint8_t* { return sR + (idx % NCH) * CH; };

  if (warp == 0) {
    // ================= TMA producer: Q once, then K(j), V(j) chunks in step order =================
    if (elect_one()) {
      tma_prefetch_desc(&tm_q); tma_prefetch_desc(&tm_kv); tma_prefetch_desc(&tm_kpe);
      mbar_arrive_expect_tx(q_full, (two ? 2 : 1) * Q_BYTES);
      for (int t = 0; t < (two ? 2 : 1); ++t)
        for (int a = 0; a < 3; ++a)
          tma_load_3d(sQ + t * Q_BYTES + a * QATOM, &tm_q, q_full, a * 64, h, seq_start + q0 + BM * t);
      for (int idx = 0; idx < n_kt * CH_PER_KV && !*abort_flag; ++idx) {
        const int slot = idx % NCH, use = idx / NCH;
        if (!mbar_wait(&r_empty[slot], (use & 1) ^ 1)) { fail(kErrTimeoutEmpty); break; }
        mbar_arrive_expect_tx(&r_full[slot], CH);
        const int j = idx / CH_PER_KV, c = idx % CH_PER_KV;
        const int row = seq_start + j * BN;
        if (c < 2) tma_load_3d(sR + slot * CH, &tm_kv, &r_full[slot], c * 64, h, row);
        else if (c == 2) tma_load_2d(sR + slot * CH, &tm_kpe, &r_full[slot], 0, row);
        else tma_load_3d(sR + slot * CH, &tm_kv, &r_full[slot], 128 + (c - 3) * 64, h, row);
      }
    }
  } else if (warp == 1) {
    // ================= MMA issuer =================
    if (elect_one()) {
      const uint32_t id_qk = idesc_bf16(BM, BN);
      const uint32_t id_pv = fa::idesc_bf16_bmn(BM, 64);
      bool ok = mbar_wait(q_full, 0);
      if (!ok) fail(kErrTimeoutFull);
      auto wait_chunks = [&](int first, int n) -> bool {
        for (int i = 0; i < n; ++i) {
          const int idx = first + i;
          if (!mbar_wait(&r_full[idx % NCH], (idx / NCH) & 1)) { fail(kErrTimeoutFull); return false; }
        }
        tc_fence_after();
        return true;
      };
      auto release_chunks = [&](int first, int n) {
        for (int i = 0; i < n; ++i) mma_commit(&r_empty[(first + i) % NCH]);
      };
      auto qk = [&](int t, int j) {
        const int kc = j * CH_PER_KV;
        const uint32_t d = tmem + 256 * t + 64 * (j & 1);
#pragma unroll
        for (int k = 0; k < DQK / 16; ++k) {
          const int a = k >> 2, off = (k & 3) * 32;
          mma_f16_ss(d, smem_desc_sw128(sQ + t * Q_BYTES + a * QATOM + off), smem_desc_sw128(chunk(kc + a) + off),
                     id_qk, k > 0);
        }
        mma_commit(&s_full[2 * t + (j & 1)]);
      };
      auto pv = [&](int t, int j) {
        const int vc = j * CH_PER_KV + 3;
        const uint32_t pcol = tmem + 256 * t + 64 * (j & 1);
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint8_t* v = chunk(vc + half);
#pragma unroll
          for (int k = 0; k < BN / 16; ++k)
            mma_f16_ts(tmem + 256 * t + 128 + 64 * half, pcol + 8 * k,
                       fa::desc_mn_sw128(v + k * 16 * 128, CH, 1024), id_pv, (j > 0 || k > 0) ? 1u : 0u);
        }
        mma_commit(&o_done[2 * t + (j & 1)]);
      };
      // prologue: the S of the first two steps of both tiles
      for (int j = 0; ok && j < 2 && j < n_kt; ++j) {
        ok = wait_chunks(j * CH_PER_KV, 3);
        if (!ok) break;
        for (int t = 0; t < 2; ++t)
          if (j < n_kt_t[t]) qk(t, j);
        release_chunks(j * CH_PER_KV, 3);
      }
      for (int j = 0; ok && j < n_kt && !*abort_flag; ++j) {
        bool v_ready = false, k_ready = false;
        for (int t = 0; t < 2 && ok; ++t) {
          if (j >= n_kt_t[t]) continue;
          if (!mbar_wait(&p_full[2 * t + (j & 1)], (j >> 1) & 1)) { fail(kErrTimeoutTmem); ok = false; break; }
          fa::trace_event(p, 1, t, j);
          tc_fence_after();
          if (!v_ready) { ok = wait_chunks(j * CH_PER_KV + 3, 2); v_ready = true; if (!ok) break; }
          pv(t, j);
          if (j + 2 < n_kt_t[t]) {
            if (!k_ready) { ok = wait_chunks((j + 2) * CH_PER_KV, 3); k_ready = true; if (!ok) break; }
            qk(t, j + 2);
          }
          fa::trace_event(p, 2, t, j);
        }
        if (!ok) break;
        release_chunks(j * CH_PER_KV + 3, 2);
        if (j + 2 < n_kt) release_chunks((j + 2) * CH_PER_KV, 3);
      }
    }
  } else if (warp >= 4) {
    // ================= softmax: tile t = (warp-4)/4, TMEM lane quadrant q, one query row per thread =================
    const int t = int(warp - 4) >> 2;
    const uint32_t q = warp & 3;
    const int row = int(q * 32 + lane);
    const int qt0 = q0 + BM * t;
    const int qi = qt0 + row;
    const int tok = seq_start + qi;
    const uint32_t t_lane = tmem + ((q * 32) << 16) + 256 * t;
    const int nkt = n_kt_t[t];
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    const bool tracer = (q == 0 && lane == 0);
    // DSA mask words of a step are fetched one step ahead, off the softmax's critical path
    const bool use_mask = p.mask != nullptr && qi < seq_len;
    auto load_mask = [&](int jj, uint32_t& w0, uint32_t& w1) {
      const int wi = (jj * BN) >> 5;
      w0 = wi < p.mask_words ? p.mask[size_t(tok) * p.mask_words + wi] : 0u;
      w1 = wi + 1 < p.mask_words ? p.mask[size_t(tok) * p.mask_words + wi + 1] : 0u;
    };
    uint32_t mwn0 = 0xffffffffu, mwn1 = 0xffffffffu;
    if (use_mask && nkt > 0) load_mask(0, mwn0, mwn1);
    for (int j = 0; j < nkt; ++j) {
      const int b = j & 1;
      if (tracer) fa::trace_event(p, 3, t, j);
      if (!mbar_wait(&s_full[2 * t + b], (j >> 1) & 1)) { fail(kErrTimeoutTmem); ok = false; break; }
      if (tracer) fa::trace_event(p, 4, t, j);
      tc_fence_after();
      float sv[64];
      {
        uint32_t (&r0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&sv[0]);
        uint32_t (&r1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&sv[32]);
        tmem_ld_32x32b_x32(t_lane + 64 * b, r0);
        tmem_ld_32x32b_x32(t_lane + 64 * b + 32, r1);
        tmem_ld_wait();
      }
      const int k0 = j * BN;
      const uint32_t mw0 = mwn0, mw1 = mwn1;
      if (use_mask && j + 1 < nkt) load_mask(j + 1, mwn0, mwn1);   // next step's words load under this step
      const bool full_row = (k0 + BN - 1 <= qi) && ((mw0 & mw1) == 0xffffffffu);
      float pm[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      if (__all_sync(0xffffffffu, full_row)) {
#pragma unroll
        for (int i = 0; i < 64; ++i) pm[i & 3] = fmaxf(pm[i & 3], sv[i]);
      } else {
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          const bool allowed = (k0 + i <= qi) && ((((i < 32) ? mw0 : mw1) >> (i & 31)) & 1u);
          sv[i] = allowed ? sv[i] : -INFINITY;
          pm[i & 3] = fmaxf(pm[i & 3], sv[i]);
        }
      }
      float mt = fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3]));
      mt = mt == -INFINITY ? mt : mt * p.scale_log2;
      const bool need = (j > 0) && (mt > m_used + kRescaleThresh);
      const float m_new = (need || j == 0) ? fmaxf(m_used, mt) : m_used;
      const float m_ref = m_new == -INFINITY ? 0.f : m_new;
      float alpha = 1.f;
      if (need && m_used != -INFINITY) alpha = fa::fast_exp2(m_used - m_ref);
      if (j > 0 && __any_sync(0xffffffffu, need)) {
        // O holds the sums of earlier steps at the old max: wait for the last PV, then rescale it in TMEM
        if (!mbar_wait(&o_done[2 * t + ((j - 1) & 1)], ((j - 1) >> 1) & 1)) {
          fail(kErrTimeoutTmem); ok = false; break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < DV; c += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(t_lane + 128 + c, r);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
          tmem_st_32x32b_x32(t_lane + 128 + c, r);
        }
      }
      float rsp[4] = {0.f, 0.f, 0.f, 0.f};
      uint32_t pk[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float a = fa::fast_exp2(fmaf(sv[2 * i], p.scale_log2, -m_ref));
        const float c = fa::fast_exp2(fmaf(sv[2 * i + 1], p.scale_log2, -m_ref));
        rsp[i & 3] += a + c;
        pk[i] = pack_bf16x2(a, c);
      }
      tmem_st_32x32b_x32(t_lane + 64 * b, pk);     // P over the first 32 columns of this S buffer
      l = l * alpha + ((rsp[0] + rsp[1]) + (rsp[2] + rsp[3]));
      m_used = m_new;
      tmem_st_wait();
      tc_fence_before();
      if (tracer) fa::trace_event(p, 5, t, j);
      mbar_arrive(&p_full[2 * t + b]);
    }
    if (p.sink) l += fa::fast_exp2(p.sink[h] * 1.4426950408889634f - (m_used == -INFINITY ? 0.f : m_used));
    if (ok && nkt > 0) {
      if (!mbar_wait(&o_done[2 * t + ((nkt - 1) & 1)], ((nkt - 1) >> 1) & 1)) { fail(kErrTimeoutTmem); ok = false; }
    }
    if (ok && nkt > 0) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* o = p.out + (size_t(tok) * p.H + h) * DV;
#pragma unroll 1
      for (int c = 0; c < DV; c += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_lane + 128 + c, r);
        tmem_ld_wait();
        if (qi < seq_len) {
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(r[8 * v + 0]) * inv, __uint_as_float(r[8 * v + 1]) * inv);
            w.y = pack_bf16x2(__uint_as_float(r[8 * v + 2]) * inv, __uint_as_float(r[8 * v + 3]) * inv);
            w.z = pack_bf16x2(__uint_as_float(r[8 * v + 4]) * inv, __uint_as_float(r[8 * v + 5]) * inv);
            w.w = pack_bf16x2(__uint_as_float(r[8 * v + 6]) * inv, __uint_as_float(r[8 * v + 7]) * inv);
            reinterpret_cast<uint4*>(o + c)[v] = w;
          }
        }
      }
    }
  }
  __syncthreads();
  if (warp == 2) { tc_fence_after(); tmem_dealloc(tmem, 512); }
#endif
}

}  // namespace fa3


// Host: q [T,H,192], kvb [T,H,256] (k_nope | v), kpe [T,64] bf16 contiguous; tiles [n_tiles] int4; out [T,H,128].
cudaError_t attn_prefill(const void* q, const void* kvb, const void* kpe, int T, int H, const int* tiles,
                         int n_tiles, const uint32_t* mask, int mask_words, float scale, void* out, int* status,
                         cudaStream_t s, const float* sink);

}  // namespace cb

// ---------------------------------------------------------------------------------------------------------------
namespace cb {
namespace fa {
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}
static bool make_tmap_3d(CUtensorMap* m, const void* ptr, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1,
                         uint64_t s2, uint32_t b0, uint32_t b1, uint32_t b2) {
  auto fn = encode_fn();
  if (!fn || (reinterpret_cast<uintptr_t>(ptr) & 15) || (s1 & 15) || (s2 & 15)) return false;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {s1, s2};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t es[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
}  // namespace fa

cudaError_t attn_prefill(const void* q, const void* kvb, const void* kpe, int T, int H, const int* tiles,
                         int n_tiles, const uint32_t* mask, int mask_words, float scale, void* out, int* status,
                         cudaStream_t s, const float* sink) {
  using namespace fa;
  if (n_tiles == 0) return cudaSuccess;
  CUtensorMap tq, tkv, tkpe;
  if (!make_tmap_3d(&tq, q, DQK, H, T, DQK * 2, uint64_t(H) * DQK * 2, 64, 1, BM) ||
      !make_tmap_3d(&tkv, kvb, 256, H, T, 256 * 2, uint64_t(H) * 256 * 2, 64, 1, BN) ||
      !make_tmap_2d(&tkpe, kpe, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 64, T, 64 * 2, 64, BN,
                    CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  {
    cudaError_t e = cb::smem_optin(attn_prefill_kernel, SMEM);
    if (e != cudaSuccess) return e;
  }
  Params p;
  p.tiles = reinterpret_cast<const int4*>(tiles);
  p.mask = mask;
  p.mask_words = mask_words;
  p.H = H;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  p.status = status;
  p.trace = nullptr;
  p.trace_cap = 0;
  p.sink = sink;
  dim3 grid(n_tiles, H);
  cb::launch_k(attn_prefill_kernel, grid, 384, SMEM, s, tq, tkv, tkpe, p);
  return cudaGetLastError();
}

// Two-tile kernel: tiles are (seq_start, seq_len, q0, 0) with q0 a multiple of 256.
cudaError_t attn_prefill2(const void* q, const void* kvb, const void* kpe, int T, int H, const int* tiles,
                          int n_tiles, const uint32_t* mask, int mask_words, float scale, void* out, int* status,
                          cudaStream_t s, int64_t* trace, int trace_cap, const float* sink) {
  using namespace fa;
  if (n_tiles == 0) return cudaSuccess;
  CUtensorMap tq, tkv, tkpe;
  if (!make_tmap_3d(&tq, q, DQK, H, T, DQK * 2, uint64_t(H) * DQK * 2, 64, 1, BM) ||
      !make_tmap_3d(&tkv, kvb, 256, H, T, 256 * 2, uint64_t(H) * 256 * 2, 64, 1, BN) ||
      !make_tmap_2d(&tkpe, kpe, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 64, T, 64 * 2, 64, BN,
                    CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  {
    cudaError_t e = cb::smem_optin(fa2::attn_prefill2_kernel, fa2::SMEM);
    if (e != cudaSuccess) return e;
  }
  Params p;
  p.tiles = reinterpret_cast<const int4*>(tiles);
  p.mask = mask;
  p.mask_words = mask_words;
  p.H = H;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  p.status = status;
  p.trace = reinterpret_cast<unsigned long long*>(trace);
  p.trace_cap = trace_cap;
  p.sink = sink;
  dim3 grid(n_tiles, H);
  cb::launch_k(fa2::attn_prefill2_kernel, grid, 384, fa2::SMEM, s, tq, tkv, tkpe, p);
  return cudaGetLastError();
}

// 64-key-step kernel (fa3): tiles as for attn_prefill2.
cudaError_t attn_prefill3(const void* q, const void* kvb, const void* kpe, int T, int H, const int* tiles,
                          int n_tiles, const uint32_t* mask, int mask_words, float scale, void* out, int* status,
                          cudaStream_t s, int64_t* trace, int trace_cap, const float* sink) {
  using namespace fa;
  if (n_tiles == 0) return cudaSuccess;
  CUtensorMap tq, tkv, tkpe;
  if (!make_tmap_3d(&tq, q, DQK, H, T, DQK * 2, uint64_t(H) * DQK * 2, 64, 1, 128) ||
      !make_tmap_3d(&tkv, kvb, 256, H, T, 256 * 2, uint64_t(H) * 256 * 2, 64, 1, fa3::BN) ||
      !make_tmap_2d(&tkpe, kpe, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 64, T, 64 * 2, 64, fa3::BN,
                    CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  {
    cudaError_t e = cb::smem_optin(fa3::attn_prefill3_kernel, fa3::SMEM);
    if (e != cudaSuccess) return e;
  }
  Params p;
  p.tiles = reinterpret_cast<const int4*>(tiles);
  p.mask = mask;
  p.mask_words = mask_words;
  p.H = H;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  p.status = status;
  p.trace = reinterpret_cast<unsigned long long*>(trace);
  p.trace_cap = trace_cap;
  p.sink = sink;
  dim3 grid(n_tiles, H);
  cb::launch_k(fa3::attn_prefill3_kernel, grid, 384, fa3::SMEM, s, tq, tkv, tkpe, p);
  return cudaGetLastError();
}

}  // namespace cb
