// Absorbed-MLA sparse attention (decode / long-context) on tcgen05 (sm_100a).
//
//   o_lat[t, h, :] = softmax_j( q[t, h, :] · kv[idx[t, j], :] · scale ) · kv[idx[t, j], :512]
//
// q: [T, H, 576] bf16 (512 absorbed-nope + 64 rope), kv: latent cache [S, 576] bf16, idx: [T, K] int32 cache slots
// (-1 = no key).  All H <= 128 heads of a token share every KV row (MQA), so a CTA computes S[128 heads, 32 keys]
// = Q·Kᵀ with M = 128 (heads) and streams the token's selected rows through shared memory with TMA gather4 (four
// 128-byte row pieces per instruction, one-row-high box).  The value half (256 of the 512 latent dims) of the CTA
// accumulates O[128, 256] in TMEM; the other half is computed by a sibling CTA (both need all of S).  S is
// double-buffered in TMEM and the softmax writes P back over its S buffer as bf16, where the P·V MMA reads it as
// its A operand (no shared-memory round trip for P).  Keys are split across CTAs (flash-decoding); a combine kernel
// merges the (m, l, O) partials.
//
// Roles (256 threads): warp 0 TMA (Q once, then gathered KV tiles, 2-stage ring of 32-key tiles), warp 1 MMA,
// warp 2 TMEM, warps 4-7 softmax (one head row per thread, lazy O rescale).  Every wait is bounded.
// Reference kernels with the same role: FlashMLA-derived decode / verify attention over the paged latent cache
// (king_v10/bundle_v9/dec/cuda_decode_attn.py:20-116, dec/cuda_vattn.py:4654).
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include "ptx.cuh"

namespace cb {
namespace mla {

// Timeline instrumentation for profiling builds (-DCB_DECODE_TRACE): the first CTA pair (token 0, split 0) records
// the SM clock of each pipeline event of each tile into g_attn_trace[(cta * 8 + event) * 64 + tile].  Compiled out
// otherwise.
#ifdef CB_DECODE_TRACE
__device__ long long* g_attn_trace;
#define CB_ATTN_TRACE(ev, j)                                                                                     \
  do {                                                                                                           \
    if (g_attn_trace && blockIdx.x == 0 && blockIdx.z == 0 && (j) < 64)                                          \
      g_attn_trace[(int(cluster_ctarank()) * 8 + (ev)) * 64 + (j)] = clock64();                                 \
  } while (0)
#else
#define CB_ATTN_TRACE(ev, j) \
  do {                       \
  } while (0)
#endif

constexpr int HM = 128;                // head rows per CTA (M)
// A row is NA 64-dim atoms: NA = 9 for MLA (512 latent + 64 RoPE key), NA = 8 for latent MQA (one 512-dim head whose
// last 64 dims carry RoPE).  The value is always the first DL = 512 dims of the row.
constexpr int DL = 512, DHALF = 256;
constexpr int KT = 32;                 // keys per tile (N of Q·Kᵀ, K of P·V)
constexpr int NAC_MAX = 5;             // atoms one CTA of the pair owns (value half + the RoPE atom)
constexpr int Q_ATOM = HM * 128;       // 16 KB: 128 rows x 64 dims
constexpr int KV_ATOM = KT * 128;      // 4 KB: 32 rows x 64 dims
// bf16 rows: the gathered atoms go straight into 5 operand stages
constexpr int STAGES = 5;
constexpr int KV_STAGE = NAC_MAX * KV_ATOM;
// fp8 rows (byte layout: values of dims 0..255 | 8 scale bytes + 8 zero | values of dims 256..511 | fp16 RoPE key):
// each CTA of the pair gathers ONE contiguous piece per row -- CTA 0 bytes [0, 272), CTA 1 bytes [256, row end) --
// with one TMA gather4 per 4 rows (the TMA unit's cost is per request, so few large pieces beat many 128-byte
// ones) into 3 staging slots; two converter warps expand the value atoms to fp16 operand tiles in the 128B-swizzled
// layout (3 stages) and copy CTA 1's fp16 RoPE atom beside them.  In a slot, rows come in groups of four
// (one gather each) at 128-byte aligned group strides.
constexpr int F8_SLOTS = 3, F8_STAGES = 3;
constexpr int F8_KV_STAGE = NAC_MAX * KV_ATOM;
constexpr int F8_SLOT = 13312;
constexpr int F8_PITCH0 = 272;                     // CTA 0: values 0..255 + scales
CB_HOST_DEVICE constexpr int f8_pitch1(int na) { return na == 9 ? 400 : 272; }   // CTA 1: scales + values (+ RoPE)
CB_HOST_DEVICE constexpr int f8_group(int pitch) { return (4 * pitch + 127) / 128 * 128; }
// one partial-score exchange buffer: 128 rows x 32 fp32, rows padded to 36 floats so that the eight threads of a
// quarter warp reading 16 bytes of eight consecutive rows hit eight different 4-bank groups
constexpr int X_LD = KT + 4;
constexpr int X_BYTES = HM * X_LD * 4;
// TMEM: O [128 x 256] fp32 at columns [0, 256); two S buffers of 64 columns at 256 and 320 (P overwrites the first
// KT/2 columns of its S buffer as packed 16-bit values and is read there by the P·V MMA)
constexpr int TM_O = 0, TM_S = 256, TM_S_STRIDE = 64;
template <bool F8>
constexpr int smem_bytes() {
  return 1024 + NAC_MAX * Q_ATOM + (F8 ? F8_STAGES * F8_KV_STAGE + F8_SLOTS * F8_SLOT : STAGES * KV_STAGE) +
         2 * X_BYTES + 256;
}
constexpr float kRescaleThresh = 8.0f;

struct Params {
  const int* idx;          // [T, K]
  int K;                   // keys per token in idx
  int H;
  int n_splits, chunk;     // keys [split*chunk, (split+1)*chunk) of each token's list
  float scale_log2;
  float* part_o;           // [T, n_splits, H, 512] fp32 (n_splits > 1)
  float* part_ml;          // [T, n_splits, H, 2]  (m in log2 units, l)
  __nv_bfloat16* out;      // [T, H, 512] when n_splits == 1
  int* status;
  const float* sink;       // optional [H]: per-head sink logit (softmax units; one extra denominator term)
};

CB_DEVICE uint64_t desc_mn_sw128(const void* p, uint32_t lbo, uint32_t sbo) {
  const uint64_t addr = smem_u32(p);
  return ((addr >> 4) & 0x3FFFull) | (uint64_t((lbo >> 4) & 0x3FFF) << 16) | (uint64_t((sbo >> 4) & 0x3FFF) << 32) |
         (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

CB_DEVICE void tma_gather4(void* dst, const void* tmap, uint64_t* bar, int col, int r0, int r1, int r2, int r3) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(col), "r"(r0), "r"(r1),
      "r"(r2), "r"(r3)
      : "memory");
}

// Two e4m3 values (low byte first) -> two fp16 (exact conversion).
CB_DEVICE uint32_t e4m3x2_to_f16x2(uint32_t v) {
  uint32_t r;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(uint16_t(v)));
  return r;
}
CB_DEVICE uint32_t hmul2_u32(uint32_t a, uint32_t s) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(s));
  return r;
}
CB_DEVICE uint32_t pack_f16x2(float a, float b) {
  __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Global atom index of local atom `la` in CTA `hh` of the pair: the CTA's value half (atoms 4hh .. 4hh+3) first,
// then (MLA rows, CTA 0) the RoPE-key atom 8.
CB_DEVICE int atom_of(int hh, int la) { return la < 4 ? hh * 4 + la : 8; }

// One token's keys [split*chunk, ...) are handled by a cluster of two CTAs (blockIdx.y = cluster rank hh).  The row
// of a cached key is split between them by 64-dim atoms: CTA hh gathers only its value half (and CTA 0 the RoPE
// atom), so no byte of a key row is read twice.  Each CTA computes the partial S over its atoms; the two partials
// are exchanged through distributed shared memory every tile, so both CTAs hold the same S and the same softmax
// (addition is commutative: identical m, l and P), and each accumulates P·V for its own value half.
//   TMA   Q atoms once; then per 32-key tile the CTA's pieces of the gathered rows (bf16: into operand stage j % 5
//         once P·V(j-5) released it; fp8: into staging slot j % 4 once its conversion and Q·Kᵀ(j-4) are done)
//   CVT   (fp8 rows, warps 2-3) staging slot j % 4 -> fp16 value atoms of operand stage j % 3, scaled per atom
//   MMA   QK(0) QK(1) | PV(0) QK(2) | PV(1) QK(3) | ...   S(j) goes to buffer j % 2; PV(j) reads P(j) from the same
//         columns and QK(j+2) overwrites them afterwards (tcgen05 MMAs of one thread execute in issue order)
//   softmax (one head row per thread): partial S -> peer's exchange buffer, peer's partial + own = S, online
//         softmax with lazy O rescale (only when the running max grows by more than 2^8), P over S in TMEM
// fp8 rows run the MMAs in fp16 (q arrives as fp16; fp16 holds every e4m3 value times its power-of-two scale).
template <int NA, bool F8>
__global__ void __launch_bounds__(256, 1) sparse_mla_kernel(const __grid_constant__ CUtensorMap tm_q,
                                                            const __grid_constant__ CUtensorMap tm_kv,
                                                            const __grid_constant__ CUtensorMap tm_sc,
                                                            const __grid_constant__ CUtensorMap tm_pe,
                                                            const Params p) {
  cb::pdl_entry();
#if defined(__CUDA_ARCH__) && __CUDA_ARCH__ >= 1000
  constexpr int NST = F8 ? F8_STAGES : STAGES;               // operand stages
  constexpr int STAGE_B = F8 ? F8_KV_STAGE : KV_STAGE;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sKV = sQ + NAC_MAX * Q_ATOM;
  uint8_t* sST = sKV + NST * STAGE_B;                         // fp8 staging slots
  float* xbuf = reinterpret_cast<float*>(sST + (F8 ? F8_SLOTS * F8_SLOT : 0));   // [2][128][X_LD]: the PEER's partial S
  uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(xbuf) + 2 * X_BYTES);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;              // [NST]
  uint64_t* kv_empty = kv_full + NST;        // [NST]
  uint64_t* s_full = kv_empty + NST;         // [2]
  uint64_t* p_full = s_full + 2;             // [2]
  uint64_t* pv_done = p_full + 2;            // [2]: PV(j) completes phase j >> 1 of pv_done[j & 1]
  uint64_t* x_full = pv_done + 2;            // [2]: the peer's partial of tile j landed in xbuf[j & 1] (tx bytes)
  uint64_t* x_empty = x_full + 2;            // [2]: the peer consumed this CTA's partial of tile j
  uint64_t* st_full = x_empty + 2;           // [F8_SLOTS] fp8: a slot's gathers landed (tx bytes)
  uint64_t* st_empty = st_full + F8_SLOTS;   // [F8_SLOTS] fp8: both converter warps are done with a slot
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(st_empty + F8_SLOTS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int t = blockIdx.x, hh = int(cluster_ctarank()), split = blockIdx.z;
  const uint32_t peer = uint32_t(hh ^ 1);
  const bool rope = NA == 9 && hh == (F8 ? 1 : 0);   // this CTA owns the RoPE-key atom
  const int nac = rope ? 5 : 4;
  const int k_begin = split * p.chunk;
  const int k_end = min(p.K, k_begin + p.chunk);
  const int n_tiles = k_end > k_begin ? (k_end - k_begin + KT - 1) / KT : 0;   // the same in both CTAs
  const int* idx_t = p.idx + size_t(t) * p.K;
  const uint32_t warp = warp_id(), lane = lane_id();

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < NST; ++i) { mbar_init(&kv_full[i], F8 ? 2 : 1); mbar_init(&kv_empty[i], 1); }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1); mbar_init(&p_full[i], 128); mbar_init(&pv_done[i], 1);
      mbar_init(&x_full[i], 1); mbar_init(&x_empty[i], 128);
    }
    if (F8)
      for (int i = 0; i < F8_SLOTS; ++i) { mbar_init(&st_full[i], 1); mbar_init(&st_empty[i], 2); }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 2) { tmem_alloc(tmem_slot, 512); tmem_relinquish(); }
  tc_fence_before();
  cluster_sync();                            // both CTAs' barriers are initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto fail = [&](int code) { if (p.status) atomicCAS(p.status, 0, code); *abort_flag = 1; };

  if (warp == 0) {
    // ---------------- TMA: this CTA's Q atoms once, then its pieces of the gathered KV rows ----------------
    if (lane == 0 && n_tiles > 0) {
      tma_prefetch_desc(&tm_q); tma_prefetch_desc(&tm_kv);
      if (F8) tma_prefetch_desc(&tm_sc);
      mbar_arrive_expect_tx(q_full, nac * Q_ATOM);
      for (int la = 0; la < nac; ++la) tma_load_3d(sQ + la * Q_ATOM, &tm_q, q_full, atom_of(hh, la) * 64, 0, t);
    }
    // KT == 32: one key per lane; the next tile's slot is loaded while this tile's gathers are issued
    int next = k_begin + lane < k_end ? idx_t[k_begin + lane] : 0;
    for (int j = 0; j < n_tiles; ++j) {
      int slot = next;
      const int nk = k_begin + (j + 1) * KT + lane;
      next = (j + 1 < n_tiles && nk < k_end) ? idx_t[nk] : 0;
      if (slot < 0) slot = 0;                                  // masked in softmax; keep the address valid
      const int s = F8 ? j % F8_SLOTS : j % STAGES;
      uint64_t* full = F8 ? &st_full[s] : &kv_full[s];
      int ok = 1;
      if (lane == 0) {
        ok = (F8 ? mbar_wait(&st_empty[s], ((j / F8_SLOTS) & 1) ^ 1)
                 : mbar_wait(&kv_empty[s], ((j / STAGES) & 1) ^ 1)) ? 1 : 0;
        if (ok) mbar_arrive_expect_tx(full, F8 ? KT * (hh ? f8_pitch1(NA) : F8_PITCH0) : nac * KV_ATOM);
        else fail(kErrTimeoutEmpty);
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok || *abort_flag) break;
      if (lane == 0) CB_ATTN_TRACE(0, j);
      // lane (part, g): part = lane / 8, row group g = lane % 8 (rows 4g..4g+3)
      const int part = int(lane >> 3), g = int(lane & 7);
      const int r0 = __shfl_sync(0xffffffffu, slot, 4 * g), r1 = __shfl_sync(0xffffffffu, slot, 4 * g + 1);
      const int r2 = __shfl_sync(0xffffffffu, slot, 4 * g + 2), r3 = __shfl_sync(0xffffffffu, slot, 4 * g + 3);
      if constexpr (F8) {
        // one gather4 of this CTA's contiguous piece of four rows (16-bit elements: CTA 1 starts at byte 256)
        if (part == 0)
          tma_gather4(sST + s * F8_SLOT + g * f8_group(hh ? f8_pitch1(NA) : F8_PITCH0), hh ? &tm_sc : &tm_kv, full,
                      hh * 128, r0, r1, r2, r3);
      } else {
        if (part < 4)
          tma_gather4(sKV + s * KV_STAGE + part * KV_ATOM + g * 4 * 128, &tm_kv, full, atom_of(hh, part) * 64, r0, r1,
                      r2, r3);
        if (rope && part == 0)                                 // the RoPE atom (CTA 0 of MLA rows)
          tma_gather4(sKV + s * KV_STAGE + 4 * KV_ATOM + g * 4 * 128, &tm_kv, full, 8 * 64, r0, r1, r2, r3);
      }
      __syncwarp();
    }
  } else if (F8 && (warp == 2 || warp == 3)) {
    // ---------------- fp8 -> fp16 value atoms (each warp converts 16 of the tile's 32 rows) ----------------
    const int cw = int(warp) - 2;
    for (int j = 0; j < n_tiles; ++j) {
      const int s8 = j % F8_SLOTS, s = j % F8_STAGES;
      int ok = 1;
      if (lane == 0) {
        ok = (mbar_wait(&st_full[s8], (j / F8_SLOTS) & 1) && mbar_wait(&kv_empty[s], ((j / F8_STAGES) & 1) ^ 1)) ? 1
                                                                                                             : 0;
        if (!ok) fail(kErrTimeoutFull);
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok || *abort_flag) break;
      const uint8_t* sl = sST + s8 * F8_SLOT;
      uint8_t* dst = sKV + s * F8_KV_STAGE;
      const int pitch = hh ? f8_pitch1(NA) : F8_PITCH0, grp = f8_group(pitch);
      const int voff = hh ? 16 : 0, soff = hh ? 0 : 256;      // values / scale bytes within this CTA's piece
#pragma unroll 2
      for (int i = 0; i < 8; ++i) {
        // task: row, local atom la, 16-value chunk c (a warp's lanes cover two rows' 256 value bytes)
        const int id = cw * 256 + i * 32 + int(lane);
        const int row = id >> 4, la = (id >> 2) & 3, c = id & 3;
        const uint8_t* rp = sl + (row >> 2) * grp + (row & 3) * pitch;
        const uint4 v = *reinterpret_cast<const uint4*>(rp + voff + la * 64 + c * 16);
        const uint32_t sb = rp[soff + hh * 4 + la];
        const __half hs = __float2half_rn(ue8m0_to_float(sb));
        const uint32_t s2 = uint32_t(*reinterpret_cast<const uint16_t*>(&hs)) * 0x10001u;
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        uint32_t h[8];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          h[2 * k] = hmul2_u32(e4m3x2_to_f16x2(w[k] & 0xffffu), s2);
          h[2 * k + 1] = hmul2_u32(e4m3x2_to_f16x2(w[k] >> 16), s2);
        }
        uint8_t* rowp = dst + la * KV_ATOM + row * 128;
        const int sw = row & 7;
        *reinterpret_cast<uint4*>(rowp + (((2 * c) ^ sw) << 4)) = make_uint4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<uint4*>(rowp + (((2 * c + 1) ^ sw) << 4)) = make_uint4(h[4], h[5], h[6], h[7]);
      }
      if (rope) {                            // fp16 RoPE key (bytes 272..399 of CTA 1's piece) -> operand atom 4
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int id = cw * 128 + i * 32 + int(lane);
          const int row = id >> 3, c8 = id & 7;
          const uint4 v = *reinterpret_cast<const uint4*>(sl + (row >> 2) * grp + (row & 3) * pitch + 272 + c8 * 16);
          *reinterpret_cast<uint4*>(dst + 4 * KV_ATOM + row * 128 + ((c8 ^ (row & 7)) << 4)) = v;
        }
      }
      fence_proxy_async();                   // generic-proxy stores -> visible to the tensor core's operand reads
      __syncwarp();
      if (lane == 0) { mbar_arrive(&kv_full[s]); mbar_arrive(&st_empty[s8]); }
      if (lane == 0 && cw == 0) CB_ATTN_TRACE(1, j);
    }
  } else if (warp == 1) {
    // ---------------- MMA ----------------
    if (elect_one() && n_tiles > 0) {
      const uint32_t id_qk = F8 ? idesc_f16(HM, KT) : idesc_bf16(HM, KT);
      const uint32_t id_pv = (F8 ? idesc_f16(HM, DHALF) : idesc_bf16(HM, DHALF)) | (1u << 16);   // B (V) MN-major
      bool ok = mbar_wait(q_full, 0);
      if (!ok) fail(kErrTimeoutFull);
      auto issue_qk = [&](int j) -> bool {
        const int s = j % NST, b = j & 1;
        if (!mbar_wait(&kv_full[s], (j / NST) & 1)) { fail(kErrTimeoutFull); return false; }
        tc_fence_after();
        for (int la = 0; la < nac; ++la) {
          const uint8_t* kb = sKV + s * STAGE_B + la * KV_ATOM;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_f16_ss(tmem + TM_S + b * TM_S_STRIDE, smem_desc_sw128(sQ + la * Q_ATOM + kk * 32),
                       smem_desc_sw128(kb + kk * 32), id_qk, (la | kk) > 0);
        }
        mma_commit(&s_full[b]);
        CB_ATTN_TRACE(2, j);
        return true;
      };
      auto issue_pv = [&](int j) -> bool {
        const int s = j % NST, b = j & 1;
        if (!mbar_wait(&p_full[b], (j >> 1) & 1)) { fail(kErrTimeoutFull); return false; }
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < KT / 16; ++k)
          mma_f16_ts(tmem + TM_O, tmem + TM_S + b * TM_S_STRIDE + 8 * k,
                     desc_mn_sw128(sKV + s * STAGE_B + k * 16 * 128, KV_ATOM, 1024), id_pv,
                     (j > 0 || k > 0) ? 1u : 0u);
        mma_commit(&pv_done[b]);
        mma_commit(&kv_empty[s]);
        CB_ATTN_TRACE(3, j);
        return true;
      };
      if (ok) ok = issue_qk(0);
      if (ok && n_tiles > 1) ok = issue_qk(1);
      for (int j = 0; ok && j < n_tiles && !*abort_flag; ++j) {
        ok = issue_pv(j);
        if (ok && j + 2 < n_tiles) ok = issue_qk(j + 2);
      }
    }
  } else if (warp >= 4) {
    // ---------------- partial-score exchange, softmax / rescale / epilogue ----------------
    const uint32_t q = warp & 3;
    const int row = q * 32 + lane;               // head
    const uint32_t t_lane = tmem + ((q * 32) << 16);
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    // validity of a tile's keys (one per lane): the slot of the next tile is loaded one tile ahead, so its global
    // load latency stays off the per-tile chain
    int next_slot = k_begin + lane < k_end ? idx_t[k_begin + lane] : -1;
    for (int j = 0; j < n_tiles; ++j) {
      const int b = j & 1;
      const int my_slot = next_slot;
      const int nk = k_begin + (j + 1) * KT + lane;
      next_slot = nk < k_end ? idx_t[nk] : -1;
      if (!mbar_wait(&s_full[b], (j >> 1) & 1)) { fail(kErrTimeoutTmem); ok = false; break; }
      if (row == 0) CB_ATTN_TRACE(4, j);
      tc_fence_after();
      uint32_t r[KT];
      tmem_ld_32x32b_x32(t_lane + TM_S + b * TM_S_STRIDE, r);
      const uint32_t vmask = __ballot_sync(0xffffffffu, my_slot >= 0);
      tmem_ld_wait();
      // arm this CTA's receive barrier for the peer's partial of tile j (its stores count down the bytes)
      if (row == 0) mbar_arrive_expect_tx(&x_full[b], HM * KT * 4);    // 128 rows x 32 fp32 (no padding)
      // my partial -> the peer's exchange buffer b (once the peer has consumed what I wrote there two tiles ago):
      // asynchronous stores whose bytes complete the peer's x_full[b], no fence on this side
      if (!mbar_wait(&x_empty[b], ((j >> 1) & 1) ^ 1)) { fail(kErrTimeoutPeer); ok = false; break; }
      if (row == 0) CB_ATTN_TRACE(7, j);
      const uint32_t xrow = mapa_shared(smem_u32(xbuf + (b * HM + row) * X_LD), peer);
      const uint32_t xbar = mapa_shared(smem_u32(&x_full[b]), peer);
#pragma unroll
      for (int c = 0; c < KT / 4; ++c)
        st_async_v4(xrow + 16 * c, r[4 * c], r[4 * c + 1], r[4 * c + 2], r[4 * c + 3], xbar);
      // the peer's partial of this tile
      if (!mbar_wait(&x_full[b], (j >> 1) & 1)) { fail(kErrTimeoutPeer); ok = false; break; }
      if (row == 0) CB_ATTN_TRACE(5, j);
      const float4* xr = reinterpret_cast<const float4*>(xbuf + (b * HM + row) * X_LD);
      float sv[KT];
#pragma unroll
      for (int c = 0; c < KT / 4; ++c) {
        const float4 v = xr[c];
        sv[4 * c + 0] = __uint_as_float(r[4 * c + 0]) + v.x;
        sv[4 * c + 1] = __uint_as_float(r[4 * c + 1]) + v.y;
        sv[4 * c + 2] = __uint_as_float(r[4 * c + 2]) + v.z;
        sv[4 * c + 3] = __uint_as_float(r[4 * c + 3]) + v.w;
      }
      float mt = -INFINITY;
#pragma unroll
      for (int i = 0; i < KT; ++i) {
        sv[i] = ((vmask >> i) & 1u) ? sv[i] * p.scale_log2 : -INFINITY;
        mt = fmaxf(mt, sv[i]);
      }
      const bool need = (j > 0) && (mt > m_used + kRescaleThresh);
      const float m_new = (need || j == 0) ? fmaxf(m_used, mt) : m_used;
      const float m_ref = m_new == -INFINITY ? 0.f : m_new;
      float alpha = 1.f;
      if (need && m_used != -INFINITY) alpha = exp2f(m_used - m_ref);
      if (j > 0 && __any_sync(0xffffffffu, need)) {
        // O holds the sums of earlier tiles at the old max: wait for the last PV, then rescale it in TMEM
        if (!mbar_wait(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1)) { fail(kErrTimeoutTmem); ok = false; break; }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < DHALF; c += 32) {
          uint32_t o[32];
          tmem_ld_32x32b_x32(t_lane + TM_O + c, o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st_32x32b_x32(t_lane + TM_O + c, o);
        }
      }
      float rs0 = 0.f, rs1 = 0.f;
      uint32_t pk[KT / 2];
#pragma unroll
      for (int i = 0; i < KT; i += 2) {
        const float a0 = exp2f(sv[i] - m_ref), a1 = exp2f(sv[i + 1] - m_ref);
        rs0 += a0;
        rs1 += a1;
        pk[i / 2] = F8 ? pack_f16x2(a0, a1) : pack_bf16x2(a0, a1);
      }
      tmem_st_32x32b_x16(t_lane + TM_S + b * TM_S_STRIDE, pk);   // P over the first KT/2 columns of S(j)
      // my exchange buffer b is free again: P (issued above) is computed from its values, so their loads are done
      mbar_arrive_cluster_relaxed(mapa_shared(smem_u32(&x_empty[b]), peer));
      l = l * alpha + (rs0 + rs1);
      m_used = m_new;
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_full[b]);
      if (row == 0) CB_ATTN_TRACE(6, j);
    }
    if (ok && n_tiles > 0) {
      if (!mbar_wait(&pv_done[(n_tiles - 1) & 1], ((n_tiles - 1) >> 1) & 1)) { fail(kErrTimeoutTmem); ok = false; }
      tc_fence_after();
    }
    const bool head_ok = row < p.H;
    if (p.n_splits > 1) {
      if (ok && head_ok && hh == 0) {
        float* ml = p.part_ml + ((size_t(t) * p.n_splits + split) * p.H + row) * 2;
        ml[0] = m_used == -INFINITY ? -INFINITY : m_used;
        ml[1] = l;
      }
    }
    if (ok) {
      float lt = l;
      if (p.sink && head_ok) {   // extra denominator term 2^(sink - m) relative to this row's running max
        const float m_ref = m_used == -INFINITY ? 0.f : m_used;
        lt += exp2f(p.sink[row] * 1.4426950408889634f - m_ref);
      }
      const float inv = (p.n_splits == 1 && lt > 0.f) ? 1.f / lt : 1.f;
#pragma unroll 1
      for (int c = 0; c < DHALF; c += 32) {
        uint32_t v[32];
        if (n_tiles > 0) {
          tmem_ld_32x32b_x32(t_lane + TM_O + c, v);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = 0u;
        }
        if (!head_ok) continue;
        if (p.n_splits == 1) {
          __nv_bfloat16* o = p.out + (size_t(t) * p.H + row) * DL + hh * DHALF + c;
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            uint4 u;
            u.x = pack_bf16x2(__uint_as_float(v[8 * w + 0]) * inv, __uint_as_float(v[8 * w + 1]) * inv);
            u.y = pack_bf16x2(__uint_as_float(v[8 * w + 2]) * inv, __uint_as_float(v[8 * w + 3]) * inv);
            u.z = pack_bf16x2(__uint_as_float(v[8 * w + 4]) * inv, __uint_as_float(v[8 * w + 5]) * inv);
            u.w = pack_bf16x2(__uint_as_float(v[8 * w + 6]) * inv, __uint_as_float(v[8 * w + 7]) * inv);
            reinterpret_cast<uint4*>(o)[w] = u;
          }
        } else {
          float* o = p.part_o + ((size_t(t) * p.n_splits + split) * p.H + row) * DL + hh * DHALF + c;
#pragma unroll
          for (int w = 0; w < 8; ++w)
            reinterpret_cast<uint4*>(o)[w] = make_uint4(v[4 * w], v[4 * w + 1], v[4 * w + 2], v[4 * w + 3]);
        }
      }
    }
  }
  __syncthreads();
  cluster_sync();          // the peer no longer writes into this CTA's exchange buffers or arrives on its barriers
  if (warp == 2) { tc_fence_after(); tmem_dealloc(tmem, 512); }
#endif
}

// out[t, h, :] = Σ_s 2^(m_s - M) O_s / Σ_s 2^(m_s - M) l_s.  One CTA of 128 threads per (token, head): the split
// weights are computed once, each thread then combines one float4 of the 512-wide row.
constexpr int kMaxSplits = 128;
__global__ void mla_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml, int n_splits,
                                   int H, __nv_bfloat16* __restrict__ out, const float* __restrict__ sink) {
  cb::pdl_entry();
  __shared__ float wts[kMaxSplits];
  __shared__ float s_inv;
  const int t = blockIdx.x, h = blockIdx.y;
  if (threadIdx.x == 0) {
    float M = -INFINITY;
    for (int s = 0; s < n_splits; ++s) M = fmaxf(M, part_ml[((size_t(t) * n_splits + s) * H + h) * 2]);
    const float sk = sink ? sink[h] * 1.4426950408889634f : -INFINITY;
    M = fmaxf(M, sk);
    float L = sink ? exp2f(sk - M) : 0.f;
    for (int s = 0; s < n_splits; ++s) {
      const float* ml = part_ml + ((size_t(t) * n_splits + s) * H + h) * 2;
      const float wv = ml[0] == -INFINITY ? 0.f : exp2f(ml[0] - M);
      wts[s] = wv;
      if (ml[0] != -INFINITY) L += wv * ml[1];
    }
    s_inv = L > 0.f ? 1.f / L : 0.f;
  }
  __syncthreads();
  const float inv = s_inv;
  for (int c = threadIdx.x * 4; c < DL; c += blockDim.x * 4) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s = 0; s < n_splits; ++s) {
      const float wv = wts[s];
      if (wv == 0.f) continue;
      const float4 o = *reinterpret_cast<const float4*>(part_o + ((size_t(t) * n_splits + s) * H + h) * DL + c);
      acc.x += wv * o.x; acc.y += wv * o.y; acc.z += wv * o.z; acc.w += wv * o.w;
    }
    uint2 w2;
    w2.x = pack_bf16x2(acc.x * inv, acc.y * inv);
    w2.y = pack_bf16x2(acc.z * inv, acc.w * inv);
    *reinterpret_cast<uint2*>(out + (size_t(t) * H + h) * DL + c) = w2;
  }
}

// ---------------------------------------------------------------------------------------------------------------
// fp8 latent rows.  A cached token row of the fp8 format holds r = 512 e4m3 latent values quantised per 64-dim atom
// (UE8M0 power-of-two scale, the smallest 2^e with amax / 2^e <= 448), the 8 scale bytes padded to 16, and for MLA
// the 64 RoPE-key dims as fp16: 656 bytes per MLA token (1152 in bf16), 528 per latent-MQA token (its RoPE dims are
// the last latent atom).  Byte layout: values of dims 0..255 | scales | values of dims 256..511 | RoPE key.
// One warp per row: lane l quantises dims [16 l, 16 l + 16), lanes 4a..4a+3 form atom a.
// ---------------------------------------------------------------------------------------------------------------
__global__ void latent_store_fp8_kernel(const __nv_bfloat16* __restrict__ rows, int n, int ld, int D,
                                        const int* __restrict__ slots, uint8_t* __restrict__ cache, int RB) {
  cb::pdl_entry();
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (w >= n) return;
  const int slot = slots[w];
  if (slot < 0) return;                                   // uniform per warp
  const __nv_bfloat16* x = rows + size_t(w) * ld;
  uint8_t* dst = cache + size_t(slot) * RB;
  const uint4 raw0 = *reinterpret_cast<const uint4*>(x + lane * 16);
  const uint4 raw1 = *reinterpret_cast<const uint4*>(x + lane * 16 + 8);
  const uint32_t u[8] = {raw0.x, raw0.y, raw0.z, raw0.w, raw1.x, raw1.y, raw1.z, raw1.w};
  float v[16];
#pragma unroll
  for (int i = 0; i < 8; ++i) { v[2 * i] = bf16_lo(u[i]); v[2 * i + 1] = bf16_hi(u[i]); }
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
  const uint32_t sb = ue8m0_for_amax(amax);
  const float inv = ue8m0_inv(sb);
  uint4 q;
  q.x = pack_fp8x4(v[0] * inv, v[1] * inv, v[2] * inv, v[3] * inv);
  q.y = pack_fp8x4(v[4] * inv, v[5] * inv, v[6] * inv, v[7] * inv);
  q.z = pack_fp8x4(v[8] * inv, v[9] * inv, v[10] * inv, v[11] * inv);
  q.w = pack_fp8x4(v[12] * inv, v[13] * inv, v[14] * inv, v[15] * inv);
  *reinterpret_cast<uint4*>(dst + lane * 16 + (lane >= 16 ? 16 : 0)) = q;   // dims 256.. follow the scale bytes
  // scale bytes of atoms 0..7 (lanes 0, 4, ..., 28) -> bytes [256, 272), the last 8 zero
  uint32_t lo = 0, hi = 0;
#pragma unroll
  for (int a = 0; a < 8; ++a) {
    const uint32_t b = __shfl_sync(0xffffffffu, sb, 4 * a);
    if (a < 4) lo |= b << (8 * a); else hi |= b << (8 * (a - 4));
  }
  if (lane == 0) *reinterpret_cast<uint4*>(dst + 256) = make_uint4(lo, hi, 0u, 0u);
  if (D == 576 && lane < 16) {                            // RoPE key dims 512..575 -> fp16 at bytes [528, 656)
    const uint2 r2 = *reinterpret_cast<const uint2*>(x + 512 + lane * 4);
    __half2 h0 = __floats2half2_rn(bf16_lo(r2.x), bf16_hi(r2.x));
    __half2 h1 = __floats2half2_rn(bf16_lo(r2.y), bf16_hi(r2.y));
    uint2 o;
    o.x = *reinterpret_cast<uint32_t*>(&h0);
    o.y = *reinterpret_cast<uint32_t*>(&h1);
    reinterpret_cast<uint2*>(dst + 528)[lane] = o;
  }
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

}  // namespace mla

namespace {

CUresult make_map(CUtensorMap* m, CUtensorMapDataType dt, int rank, const void* base, const cuuint64_t* dims,
                  const cuuint64_t* strides, const cuuint32_t* box, CUtensorMapSwizzle sw) {
  const cuuint32_t es[3] = {1, 1, 1};
  return mla::encode_fn()(m, dt, rank, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

template <int NA, bool F8>
cudaError_t launch_sparse_mla(const CUtensorMap& tq, const CUtensorMap& tkv, const CUtensorMap& tsc,
                              const CUtensorMap& tpe, const mla::Params& p, int T, int n_splits, cudaStream_t s) {
  using namespace mla;
  cudaError_t e = smem_optin(sparse_mla_kernel<NA, F8>, smem_bytes<F8>());
  if (e != cudaSuccess) return e;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1; attr[0].val.clusterDim.y = 2; attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;     // see cb::pdl_entry
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(T, 2, n_splits);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = smem_bytes<F8>();
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, sparse_mla_kernel<NA, F8>, tq, tkv, tsc, tpe, p);
}

// Shared by the bf16 and fp8 entry points: q [T, H, D] (bf16, or fp16 for fp8 rows); kv rows [S, row_bytes].
cudaError_t sparse_mla_any(bool f8, const void* q, int T, int H, const void* kv, int S, const int* idx, int K,
                           float scale, int n_splits, float* part_o, float* part_ml, void* out, int* status,
                           cudaStream_t s, const float* sink, int D) {
  using namespace mla;
  if (T == 0) return cudaSuccess;
  if (H > HM || H < 1 || n_splits < 1 || n_splits > kMaxSplits || (D != 576 && D != 512)) return cudaErrorInvalidValue;
  if (!encode_fn()) return cudaErrorInvalidValue;
  const int RB = f8 ? (D == 576 ? 656 : 528) : D * 2;        // bytes of one cached row
  CUtensorMap tq, tkv, tsc, tpe;
  {
    const cuuint64_t dims[3] = {cuuint64_t(D), cuuint64_t(H), cuuint64_t(T)};
    const cuuint64_t str[2] = {cuuint64_t(D) * 2, cuuint64_t(H) * D * 2};
    const cuuint32_t box[3] = {64, HM, 1};
    if (make_map(&tq, f8 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, q, dims, str, box,
                 CU_TENSOR_MAP_SWIZZLE_128B) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  if (!f8) {
    const cuuint64_t dims[2] = {cuuint64_t(D), cuuint64_t(S)};
    const cuuint64_t str[1] = {cuuint64_t(RB)};
    const cuuint32_t box[2] = {64, 1};
    if (make_map(&tkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, kv, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B) !=
        CUDA_SUCCESS)
      return cudaErrorInvalidValue;
    tsc = tkv;
    tpe = tkv;
  } else {
    // 16-bit elements over each row: CTA 0 reads [0, 272) bytes, CTA 1 [256, RB)
    const cuuint64_t dims[2] = {cuuint64_t(RB / 2), cuuint64_t(S)};
    const cuuint64_t str[1] = {cuuint64_t(RB)};
    const cuuint32_t box0[2] = {F8_PITCH0 / 2, 1}, box1[2] = {uint32_t(RB - 256) / 2, 1};
    if (make_map(&tkv, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, kv, dims, str, box0, CU_TENSOR_MAP_SWIZZLE_NONE) !=
            CUDA_SUCCESS ||
        make_map(&tsc, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, kv, dims, str, box1, CU_TENSOR_MAP_SWIZZLE_NONE) !=
            CUDA_SUCCESS)
      return cudaErrorInvalidValue;
    tpe = tkv;
  }
  Params p;
  p.idx = idx; p.K = K; p.H = H; p.n_splits = n_splits;
  p.chunk = ((K + n_splits - 1) / n_splits + KT - 1) / KT * KT;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.part_o = part_o; p.part_ml = part_ml;
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  p.status = status;
  p.sink = sink;
  cudaError_t e;
  if (f8) e = D == 576 ? launch_sparse_mla<9, true>(tq, tkv, tsc, tpe, p, T, n_splits, s)
                       : launch_sparse_mla<8, true>(tq, tkv, tsc, tpe, p, T, n_splits, s);
  else e = D == 576 ? launch_sparse_mla<9, false>(tq, tkv, tsc, tpe, p, T, n_splits, s)
                    : launch_sparse_mla<8, false>(tq, tkv, tsc, tpe, p, T, n_splits, s);
  if (e != cudaSuccess) return e;
  e = cudaGetLastError();
  if (e != cudaSuccess || n_splits == 1) return e;
  cb::launch_k(mla::mla_combine_kernel, dim3(T, H), 128, 0, s, part_o, part_ml, n_splits, H,
               reinterpret_cast<__nv_bfloat16*>(out), sink);
  return cudaGetLastError();
}

}  // namespace

// q [T,H,D], kv [S,D] bf16 with D = 576 (MLA) or 512 (latent MQA); idx [T,K]; out [T,H,512] bf16.
// part_o/part_ml: workspace for n_splits > 1
// (sizes T*n_splits*H*512 and T*n_splits*H*2 floats).
cudaError_t sparse_mla(const void* q, int T, int H, const void* kv, int S, const int* idx, int K, float scale,
                       int n_splits, float* part_o, float* part_ml, void* out, int* status, cudaStream_t s,
                       const float* sink, int D) {
  return sparse_mla_any(false, q, T, H, kv, S, idx, K, scale, n_splits, part_o, part_ml, out, status, s, sink, D);
}

// The same attention over fp8 cache rows (656 bytes per MLA row, 528 per latent-MQA row; see latent_store_fp8),
// with q [T,H,D] in fp16.
cudaError_t sparse_mla_fp8(const void* q, int T, int H, const void* kv, int S, const int* idx, int K, float scale,
                           int n_splits, float* part_o, float* part_ml, void* out, int* status, cudaStream_t s,
                           const float* sink, int D) {
  return sparse_mla_any(true, q, T, H, kv, S, idx, K, scale, n_splits, part_o, part_ml, out, status, s, sink, D);
}

// rows [n, D] bf16 (row stride ld elements, D = 576 or 512) -> fp8 cache rows at slots[i] (slots < 0 skipped).
cudaError_t latent_store_fp8(const void* rows, int n, int ld, int D, const int* slots, void* cache, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  if ((D != 576 && D != 512) || ld < D || (ld % 8) != 0) return cudaErrorInvalidValue;
  const int RB = D == 576 ? 656 : 528;
  cb::launch_k(mla::latent_store_fp8_kernel, dim3((n + 7) / 8), 256, 0, s,
               reinterpret_cast<const __nv_bfloat16*>(rows), n, ld, D, slots, reinterpret_cast<uint8_t*>(cache), RB);
  return cudaGetLastError();
}

}  // namespace cb
