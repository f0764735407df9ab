// NVLink peer-memory kernels for the multi-GPU paths (symmetric heap, see symm.cu):
//
//  * p2p_gather_rows     : every rank writes its rows into every peer's gathered buffer (the all-gather of the
//                          down-projection outputs / DSA selection), 16-byte P2P stores.
//  * p2p_scatter_partials: rank s writes the rows of its o_proj partial sum that token-shard owner r holds into
//                          r's slot [s]; reduce_slots sums the world slots locally in fp32 (the reduce-scatter).
//  * EP MoE: moe_count (per-expert counts -> owners), moe_dispatch (fp8 1x128 quantisation of each token row fused
//    with the P2P stores of the row and its UE8M0 scale bytes into the owner's expert-sorted receive buffer, in
//    the SF-tile layout the grouped GEMM reads), moe_combine_pull (P2P loads of the expert outputs from their
//    owners fused with the weighted top-k reduction and the shared-expert add).
//  * embed_peer: vocab-parallel embedding — each token's row is read straight from its owner's table.
//
// Every kernel here only loads/stores peer memory with ordinary (non-TMA) instructions; the cross-rank ordering is
// done by the signal/wait kernels of symm.cu (release/acquire at system scope, bounded waits).
// Reference: MegaMoE dispatch/combine over SymBuffer (king_v10/bundle_v9/cuda_moe_prefill.py:4343-4660,
// 5542-5681), Engram peer reads (cuda_peer_read.py:64-126).
#include "common.cuh"

namespace cb {

// ---------------------------------------------------------------------------------------------------------------
// all-gather of rows: src [n, row_bytes] -> dst_ptrs[r] + (row0 + i) * row_bytes for every rank r
// ---------------------------------------------------------------------------------------------------------------
template <typename V>
__global__ void p2p_gather_kernel(const uint8_t* __restrict__ src, int n, int row_bytes,
                                  const uint64_t* __restrict__ dst_ptrs, int world, int row0) {
  cb::pdl_entry();
  const int chunks = row_bytes / int(sizeof(V));
  const int64_t total = int64_t(n) * chunks;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t row = i / chunks, c = i % chunks;
    const V v = reinterpret_cast<const V*>(src + row * row_bytes)[c];
    for (int r = 0; r < world; ++r) {
      uint8_t* dst = reinterpret_cast<uint8_t*>(dst_ptrs[r]) + (row0 + row) * row_bytes;
      reinterpret_cast<V*>(dst)[c] = v;
    }
  }
  publish_peer_stores();    // the peer stores are performed before any later barrier publishes them
}

cudaError_t p2p_gather_rows(const void* src, int n, int row_bytes, const uint64_t* dst_ptrs, int world, int row0,
                            cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  if (row_bytes % 4) return cudaErrorInvalidValue;
  const bool wide = (row_bytes % 16) == 0;
  const int64_t total = int64_t(n) * (row_bytes / (wide ? 16 : 4));
  const int blocks = int(total / 256 + 1 < 4 * 148 ? total / 256 + 1 : 4 * 148);
  if (wide)
    cb::launch_k(p2p_gather_kernel<uint4>, blocks, 256, 0, s, reinterpret_cast<const uint8_t*>(src), n, row_bytes, dst_ptrs,
                                                    world, row0);
  else
    cb::launch_k(p2p_gather_kernel<uint32_t>, blocks, 256, 0, s, reinterpret_cast<const uint8_t*>(src), n, row_bytes,
                                                       dst_ptrs, world, row0);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------------------------------
// head <-> token all-to-all around the decode attention core (tensor-parallel attention, `world` ranks own
// contiguous token shards bounds[r]..bounds[r+1] and `C`-byte blocks of heads):
//   mode 0, heads -> tokens: src [T, C] (all tokens, this rank's heads) -> peer d's [n_d, world * C] at column
//           block my_rank, rows of d's tokens;
//   mode 1, tokens -> heads: src [n_me, world * C] (this rank's tokens, all heads) -> peer d's [T, C] at the rows
//           of this rank's tokens, column block d.
// One CTA per (row, destination); every warp store writes 512 contiguous bytes of a destination row.
// ---------------------------------------------------------------------------------------------------------------
__global__ void p2p_a2a_heads_kernel(const uint8_t* __restrict__ src, const int* __restrict__ bounds, int world,
                                     int my_rank, const uint64_t* __restrict__ dst_ptrs, int C, int mode) {
  cb::pdl_entry();
  const int i = blockIdx.x, d = blockIdx.y;
  const uint8_t* s;
  uint8_t* t;
  if (mode == 0) {
    const int lo = bounds[d], n = bounds[d + 1] - lo;
    if (i >= n) return;
    s = src + size_t(lo + i) * C;
    t = reinterpret_cast<uint8_t*>(dst_ptrs[d]) + (size_t(i) * world + my_rank) * C;
  } else {
    const int lo = bounds[my_rank], n = bounds[my_rank + 1] - lo;
    if (i >= n) return;
    s = src + (size_t(i) * world + d) * C;
    t = reinterpret_cast<uint8_t*>(dst_ptrs[d]) + size_t(lo + i) * C;
  }
  for (int c = threadIdx.x; c < C / 16; c += blockDim.x)
    reinterpret_cast<uint4*>(t)[c] = reinterpret_cast<const uint4*>(s)[c];
  publish_peer_stores();
}

cudaError_t p2p_a2a_heads(const void* src, const int* bounds_dev, int world, int my_rank, const uint64_t* dst_ptrs,
                          int C, int mode, int max_rows, cudaStream_t s) {
  if (max_rows <= 0) return cudaSuccess;
  if (C % 16 || (mode != 0 && mode != 1)) return cudaErrorInvalidValue;
  cb::launch_k(p2p_a2a_heads_kernel, dim3(max_rows, world), 256, 0, s, reinterpret_cast<const uint8_t*>(src), bounds_dev,
                                                             world, my_rank, dst_ptrs, C, mode);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------------------------------
// reduce-scatter: partial [T, D] bf16 -> owner r's slot buffer rows [my_rank][i] for rows of r's shard;
// reduce_slots: out[i] = sum_s slots[s][i] (fp32 accumulate, bf16 out)
// ---------------------------------------------------------------------------------------------------------------
__global__ void p2p_scatter_kernel(const __nv_bfloat16* __restrict__ part, int D, const int* __restrict__ bounds,
                                   int world, int my_rank, const uint64_t* __restrict__ slot_ptrs, int slot_rows,
                                   int T) {
  cb::pdl_entry();
  const int chunks = D / 8;
  const int64_t total = int64_t(T) * chunks;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int row = int(i / chunks), c = int(i % chunks);
    int r = 0;
    while (r + 1 < world && row >= bounds[r + 1]) ++r;
    const int li = row - bounds[r];
    const uint4 v = reinterpret_cast<const uint4*>(part + size_t(row) * D)[c];
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(slot_ptrs[r]) + (size_t(my_rank) * slot_rows + li) * D;
    reinterpret_cast<uint4*>(dst)[c] = v;
  }
  publish_peer_stores();
}

__global__ void reduce_slots_kernel(const __nv_bfloat16* __restrict__ slots, int world, int slot_rows, int n, int D,
                                    __nv_bfloat16* __restrict__ out) {
  cb::pdl_entry();
  const int chunks = D / 8;
  const int64_t total = int64_t(n) * chunks;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int row = int(i / chunks), c = int(i % chunks);
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int s = 0; s < world; ++s) {
      const uint4 v = reinterpret_cast<const uint4*>(slots + (size_t(s) * slot_rows + row) * D)[c];
      acc[0] += bf16_lo(v.x); acc[1] += bf16_hi(v.x); acc[2] += bf16_lo(v.y); acc[3] += bf16_hi(v.y);
      acc[4] += bf16_lo(v.z); acc[5] += bf16_hi(v.z); acc[6] += bf16_lo(v.w); acc[7] += bf16_hi(v.w);
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]); o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]); o.w = pack_bf16x2(acc[6], acc[7]);
    reinterpret_cast<uint4*>(out + size_t(row) * D)[c] = o;
  }
}

cudaError_t p2p_scatter_partials(const void* part, int T, int D, const int* bounds_dev, int world, int my_rank,
                                 const uint64_t* slot_ptrs, int slot_rows, cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  if (D % 8) return cudaErrorInvalidValue;
  const int64_t total = int64_t(T) * (D / 8);
  const int blocks = int(total / 256 + 1 < 4 * 148 ? total / 256 + 1 : 4 * 148);
  cb::launch_k(p2p_scatter_kernel, blocks, 256, 0, s, reinterpret_cast<const __nv_bfloat16*>(part), D, bounds_dev, world,
                                            my_rank, slot_ptrs, slot_rows, T);
  return cudaGetLastError();
}

cudaError_t reduce_slots(const void* slots, int world, int slot_rows, int n, int D, void* out, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  const int64_t total = int64_t(n) * (D / 8);
  const int blocks = int(total / 256 + 1 < 4 * 148 ? total / 256 + 1 : 4 * 148);
  cb::launch_k(reduce_slots_kernel, blocks, 256, 0, s, reinterpret_cast<const __nv_bfloat16*>(slots), world, slot_rows, n, D,
                                             reinterpret_cast<__nv_bfloat16*>(out));
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------------------------------
// EP MoE
// ---------------------------------------------------------------------------------------------------------------
// counts: one CTA per global expert scans this rank's (token, slot) pairs in order; pair_rank[i] = rank of pair i
// among the pairs of its expert (token order, deterministic), and the expert's count is written into EVERY rank's
// count matrix cnt_ptrs[r] -> int32 [world(src)][E], so that after one barrier each rank can lay out every owner's
// receive buffer by itself (no second exchange of offsets).
__global__ void moe_count_kernel(const int* __restrict__ ids, int Tk, int E, int world, int my_rank,
                                 const uint64_t* __restrict__ cnt_ptrs, int* __restrict__ pair_rank) {
  cb::pdl_entry();
  constexpr int kPer = 8;                  // consecutive pairs per thread per pass
  __shared__ int sw[32];
  const int e = blockIdx.x;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int base = 0;
  for (int i0 = 0; i0 < Tk; i0 += blockDim.x * kPer) {
    const int b0 = i0 + threadIdx.x * kPer;
    uint32_t mask = 0;
#pragma unroll
    for (int u = 0; u < kPer; ++u)
      if (b0 + u < Tk && ids[b0 + u] == e) mask |= 1u << u;
    const int hits = __popc(mask);
    // inclusive block scan of hits
    int v = hits;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += n;
    }
    if (lane == 31) sw[wid] = v;
    __syncthreads();
    if (wid == 0) {
      int x = lane < nw ? sw[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += n;
      }
      if (lane < nw) sw[lane] = x;
    }
    __syncthreads();
    int r = base + v + (wid > 0 ? sw[wid - 1] : 0) - hits;
    while (mask) {
      const int u = __ffs(mask) - 1;
      mask &= mask - 1;
      pair_rank[b0 + u] = r++;
    }
    base += sw[nw - 1];
    __syncthreads();
  }
  if (threadIdx.x < world) {
    int* dst = reinterpret_cast<int*>(cnt_ptrs[threadIdx.x]) + my_rank * E + e;
    *dst = base;
    __threadfence_system();
  }
}

cudaError_t moe_count(const int* ids, int Tk, int E, int world, int my_rank, const uint64_t* cnt_ptrs,
                      int* pair_rank, cudaStream_t s) {
  if (world > 512) return cudaErrorInvalidValue;
  cb::launch_k(moe_count_kernel, E, 512, 0, s, ids, Tk, E, world, my_rank, cnt_ptrs, pair_rank);
  return cudaGetLastError();
}

// Layout of every owner's receive buffer from the full count matrix cnt [world(src)][E] (identical on every rank
// after the count barrier).  Owner o holds experts [o*El, (o+1)*El); each expert's segment is padded to `align`
// rows.  my_off[e]: the row of expert e's segment at its owner where this rank's rows start (sources in rank order).
// For this rank's own experts: m_block_expert (expert of each 128-row block, -1 beyond) and num_blocks.
// One thread per global expert: its row count over all sources and the rows of lower-ranked sources, then a
// block-wide inclusive scan of the 128-row block counts; each owner's segment starts at row 0 of its buffer.
__global__ void moe_layout_kernel(const int* __restrict__ cnt, int world, int E, int my_rank, int max_blocks,
                                  int align, int* __restrict__ my_off, int* __restrict__ m_block_expert,
                                  int* __restrict__ num_blocks) {
  cb::pdl_entry();
  __shared__ int s_incl[1024];
  __shared__ int s_warp[32];
  const int e = threadIdx.x;
  const int lane = e & 31, wid = e >> 5, nw = blockDim.x >> 5;
  const int El = E / world;
  int n = 0, before = 0;
  if (e < E) {
#pragma unroll 8
    for (int sr = 0; sr < world; ++sr) {
      const int c = cnt[sr * E + e];
      if (sr < my_rank) before += c;
      n += c;
    }
  }
  const int nb = e < E ? (n + align - 1) / align * (align / 128) : 0;   // segment padded to `align` rows
  int v = nb;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int u = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += u;
  }
  if (lane == 31) s_warp[wid] = v;
  __syncthreads();
  if (wid == 0) {
    int x = lane < nw ? s_warp[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += u;
    }
    if (lane < nw) s_warp[lane] = x;
  }
  __syncthreads();
  const int incl = v + (wid > 0 ? s_warp[wid - 1] : 0);
  if (e < E) s_incl[e] = incl;
  __syncthreads();
  const int mine0 = my_rank * El, mine1 = mine0 + El;
  const int mine_base = mine0 > 0 ? s_incl[mine0 - 1] : 0;
  const int total = s_incl[mine1 - 1] - mine_base;              // 128-row blocks of this rank's experts
  if (e < E) {
    const int o = e / El;
    const int seg_base = o * El > 0 ? s_incl[o * El - 1] : 0;
    const int local = incl - nb - seg_base;                      // blocks before e inside its owner's buffer
    my_off[e] = local * 128 + before;
    if (o == my_rank)
      for (int j = 0; j < nb && local + j < max_blocks; ++j) m_block_expert[local + j] = e - mine0;
  }
  for (int j = total + e; j < max_blocks; j += blockDim.x) m_block_expert[j] = -1;
  if (e == 0) num_blocks[0] = total < max_blocks ? total : max_blocks;
}

cudaError_t moe_layout(const int* cnt, int world, int E, int my_rank, int max_blocks, int align, int* my_off,
                       int* m_block_expert, int* num_blocks, cudaStream_t s) {
  if ((align != 128 && align != 256) || world > 1024 || E % world || E > 1024) return cudaErrorInvalidValue;
  cb::launch_k(moe_layout_kernel, 1, ((E + 31) / 32) * 32, 0, s, cnt, world, E, my_rank, max_blocks, align, my_off,
                                                           m_block_expert, num_blocks);
  return cudaGetLastError();
}

constexpr int kDispatchCols = 1024;      // columns of a token row per dispatch CTA (a multiple of 512)
constexpr int kSplitRowsBelow = 1024;    // token counts below this split each row over several CTAs

// Dispatch: one CTA per local token (for decode batches, one per 1024 columns of it); the row is quantised once
// (1x128 UE8M0 blocks), then written to each selected expert's owner at row  my_off[e] + pair_rank.  Destination
// rows are stored in pos_out [T, k] (row index inside the owner's buffer, -1 if it did not fit) for a pull combine; with rinfo_ptrs the owner also
// learns where each received row goes back to: rinfo_owner[row] = (my_rank << 24) | (t * k + j), the slot of this
// token's j-th expert in this rank's combine buffer (push combine from the owner's GEMM epilogue).
// recv_ptrs[r]: fp8 rows [cap, D]; sf_ptrs[r]: SF tiles of those rows (row blocks = cap/128).
__global__ void moe_dispatch_kernel(const __nv_bfloat16* __restrict__ x, int D, const int* __restrict__ ids, int k,
                                    int El, int my_rank, const int* __restrict__ pair_rank,
                                    const uint64_t* __restrict__ recv_ptrs, const uint64_t* __restrict__ sf_ptrs,
                                    const int* __restrict__ my_off, const uint64_t* __restrict__ rinfo_ptrs,
                                    int cap, int* __restrict__ pos_out, int* __restrict__ status) {
  cb::pdl_entry();
  const int t = blockIdx.x;
  const int span = gridDim.y == 1 ? D : kDispatchCols;
  const int c0 = blockIdx.y * span, c1 = min(D, c0 + span);    // this CTA's columns
  const int row_blocks = cap / 128;
  __shared__ int s_dst[16], s_owner[16];
  __shared__ uint32_t s_sf[64];            // UE8M0 scale of each 128-column block, four per word
  if (threadIdx.x < k) {
    const int e = ids[t * k + threadIdx.x];
    const int owner = e / El;
    int row = my_off[e] + pair_rank[t * k + threadIdx.x];
    if (row >= cap) { if (status) atomicCAS(status, 0, kErrBadArg); row = -1; }
    s_dst[threadIdx.x] = row;
    s_owner[threadIdx.x] = owner;
    if (blockIdx.y == 0) {
      pos_out[t * k + threadIdx.x] = row;
      if (rinfo_ptrs && row >= 0)
        reinterpret_cast<int*>(rinfo_ptrs[owner])[row] = (my_rank << 24) | (t * k + threadIdx.x);
    }
  }
  if (threadIdx.x < 64) s_sf[threadIdx.x] = 0x7f7f7f7fu;
  __syncthreads();
  // each group of 16 threads quantises one 128-column block (8 values per thread); every warp store writes 256
  // contiguous bytes of a destination row
  for (int col = c0 + threadIdx.x * 8; col < c1; col += blockDim.x * 8) {
    const uint4 raw = *reinterpret_cast<const uint4*>(x + size_t(t) * D + col);
    float v[8] = {bf16_lo(raw.x), bf16_hi(raw.x), bf16_lo(raw.y), bf16_hi(raw.y),
                  bf16_lo(raw.z), bf16_hi(raw.z), bf16_lo(raw.w), bf16_hi(raw.w)};
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[j]));
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const uint32_t sb = ue8m0_for_amax(amax);
    const float inv = ue8m0_inv(sb);
    uint2 q;
    q.x = pack_fp8x4(v[0] * inv, v[1] * inv, v[2] * inv, v[3] * inv);
    q.y = pack_fp8x4(v[4] * inv, v[5] * inv, v[6] * inv, v[7] * inv);
    const int kb = col / 128;
    if ((threadIdx.x & 15) == 0) reinterpret_cast<uint8_t*>(s_sf)[kb] = uint8_t(sb);
    for (int j = 0; j < k; ++j) {
      const int row = s_dst[j];
      if (row < 0) continue;
      uint8_t* dst = reinterpret_cast<uint8_t*>(recv_ptrs[s_owner[j]]) + size_t(row) * D + col;
      *reinterpret_cast<uint2*>(dst) = q;
    }
  }
  __syncthreads();
  // scale words: word g of a row holds the scales of column blocks 4g..4g+3 (SF tile layout of the owner)
  const int g0 = c0 / 512, words = (c1 + 511) / 512 - g0;       // scale words covering this CTA's columns
  for (int i = threadIdx.x; i < k * words; i += blockDim.x) {
    const int j = i / words, g = g0 + i - j * words;
    const int row = s_dst[j];
    if (row < 0) continue;
    const int rb = row >> 7, r = row & 127;
    uint32_t* sfw = reinterpret_cast<uint32_t*>(sf_ptrs[s_owner[j]]) +
                    (size_t(g) * row_blocks + rb) * 128 + (r & 31) * 4 + (r >> 5);
    *sfw = s_sf[g];
  }
  publish_peer_stores();
}

cudaError_t moe_dispatch(const void* x, int T, int D, const int* ids, int k, int El, int my_rank,
                         const int* pair_rank, const uint64_t* recv_ptrs, const uint64_t* sf_ptrs,
                         const int* my_off, const uint64_t* rinfo_ptrs, int cap, int* pos_out, int* status,
                         cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  if (D % 128 || D > 64 * 512 || k > 16 || cap % 128 || (rinfo_ptrs && T * k > (1 << 24))) return cudaErrorInvalidValue;
  // decode batches: a token row is split over D/1024 CTAs (one 8-column chunk per thread) so the few tokens
  // spread their peer stores over the SMs; prefill batches: one 256-thread CTA per token
  const bool split = T < kSplitRowsBelow;
  cb::launch_k(moe_dispatch_kernel, dim3(T, split ? (D + kDispatchCols - 1) / kDispatchCols : 1),
               split ? kDispatchCols / 8 : 256, 0, s,
               reinterpret_cast<const __nv_bfloat16*>(x), D, ids, k, El, my_rank, pair_rank,
                                        recv_ptrs, sf_ptrs, my_off, rinfo_ptrs, cap, pos_out, status);
  return cudaGetLastError();
}

// Push combine, home side: the owners' expert GEMMs stored every routed row into this rank's slots [T*k, D];
// out[t] = add[t] + sum_j w[t,j] * slots[t*k + j] over the slots that were dispatched (pos >= 0).  Local reads only.
template <int KMAX>
__global__ void moe_combine_slots_kernel(const __nv_bfloat16* __restrict__ slots, int D, const int* __restrict__ pos,
                                         const float* __restrict__ w, int k, const __nv_bfloat16* __restrict__ add,
                                         __nv_bfloat16* __restrict__ out) {
  cb::pdl_entry();
  const int t = blockIdx.x;
  __shared__ float s_w[KMAX];
  if (threadIdx.x < KMAX) {
    const int j = threadIdx.x;
    s_w[j] = (j < k && pos[t * k + j] >= 0) ? w[t * k + j] : 0.f;
  }
  __syncthreads();
  const uint4* src = reinterpret_cast<const uint4*>(slots + size_t(t) * k * D);
  for (int c = blockIdx.y * blockDim.x + threadIdx.x; c < D / 8; c += gridDim.y * blockDim.x) {
    float acc[8];
    if (add) {
      const uint4 a = *reinterpret_cast<const uint4*>(add + size_t(t) * D + 8 * c);
      acc[0] = bf16_lo(a.x); acc[1] = bf16_hi(a.x); acc[2] = bf16_lo(a.y); acc[3] = bf16_hi(a.y);
      acc[4] = bf16_lo(a.z); acc[5] = bf16_hi(a.z); acc[6] = bf16_lo(a.w); acc[7] = bf16_hi(a.w);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.f;
    }
#pragma unroll
    for (int j = 0; j < KMAX; ++j) {
      if (j >= k) break;
      const float wv = s_w[j];
      if (wv == 0.f) continue;
      const uint4 v = src[size_t(j) * (D / 8) + c];
      acc[0] += wv * bf16_lo(v.x); acc[1] += wv * bf16_hi(v.x); acc[2] += wv * bf16_lo(v.y);
      acc[3] += wv * bf16_hi(v.y); acc[4] += wv * bf16_lo(v.z); acc[5] += wv * bf16_hi(v.z);
      acc[6] += wv * bf16_lo(v.w); acc[7] += wv * bf16_hi(v.w);
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]); o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]); o.w = pack_bf16x2(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(out + size_t(t) * D + 8 * c) = o;
  }
}

cudaError_t moe_combine_slots(const void* slots, int T, int D, const int* pos, const float* w, int k, const void* add,
                              void* out, cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  if (D % 8 || k > 16) return cudaErrorInvalidValue;
  const auto* sl = reinterpret_cast<const __nv_bfloat16*>(slots);
  const auto* a = reinterpret_cast<const __nv_bfloat16*>(add);
  auto* o = reinterpret_cast<__nv_bfloat16*>(out);
  if (k <= 8)
    cb::launch_k(moe_combine_slots_kernel<8>, T, 128, 0, s, sl, D, pos, w, k, a, o);
  else
    cb::launch_k(moe_combine_slots_kernel<16>, T, 128, 0, s, sl, D, pos, w, k, a, o);
  return cudaGetLastError();
}

// Combine: out[t] = add[t] + sum_j w[t,j] * y_owner(j)[pos[t,j]] — P2P loads from the owners' output buffers.
// The k remote loads of a column chunk are issued together (KMAX unrolled, predicated) so that each thread keeps k
// NVLink reads in flight instead of one.
template <int KMAX>
__global__ void moe_combine_pull_kernel(const uint64_t* __restrict__ y_ptrs, int D, const int* __restrict__ ids,
                                        const int* __restrict__ pos, const float* __restrict__ w, int k, int El,
                                        const __nv_bfloat16* __restrict__ add, __nv_bfloat16* __restrict__ out) {
  cb::pdl_entry();
  const int t = blockIdx.x;                // token; blockIdx.y: 1024-column slice of its row
  __shared__ const uint4* s_src[KMAX];
  __shared__ float s_w[KMAX];
  if (threadIdx.x < KMAX) {
    const int j = threadIdx.x;
    const int row = j < k ? pos[t * k + j] : -1;
    s_src[j] = row < 0 ? nullptr
                       : reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(
                                                            y_ptrs[ids[t * k + j] / El]) + size_t(row) * D);
    s_w[j] = row < 0 ? 0.f : w[t * k + j];
  }
  __syncthreads();
  for (int c = blockIdx.y * blockDim.x + threadIdx.x; c < D / 8; c += gridDim.y * blockDim.x) {
    float acc[8];
    if (add) {
      const uint4 a = *reinterpret_cast<const uint4*>(add + size_t(t) * D + 8 * c);
      acc[0] = bf16_lo(a.x); acc[1] = bf16_hi(a.x); acc[2] = bf16_lo(a.y); acc[3] = bf16_hi(a.y);
      acc[4] = bf16_lo(a.z); acc[5] = bf16_hi(a.z); acc[6] = bf16_lo(a.w); acc[7] = bf16_hi(a.w);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.f;
    }
    uint4 v[KMAX];
#pragma unroll
    for (int j = 0; j < KMAX; ++j) v[j] = s_src[j] ? s_src[j][c] : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int j = 0; j < KMAX; ++j) {
      const float wv = s_w[j];
      acc[0] += wv * bf16_lo(v[j].x); acc[1] += wv * bf16_hi(v[j].x); acc[2] += wv * bf16_lo(v[j].y);
      acc[3] += wv * bf16_hi(v[j].y); acc[4] += wv * bf16_lo(v[j].z); acc[5] += wv * bf16_hi(v[j].z);
      acc[6] += wv * bf16_lo(v[j].w); acc[7] += wv * bf16_hi(v[j].w);
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]); o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]); o.w = pack_bf16x2(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(out + size_t(t) * D + 8 * c) = o;
  }
}

cudaError_t moe_combine_pull(const uint64_t* y_ptrs, int T, int D, const int* ids, const int* pos, const float* w,
                             int k, int El, const void* add, void* out, cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  if (D % 8 || k > 16) return cudaErrorInvalidValue;
  const auto* a = reinterpret_cast<const __nv_bfloat16*>(add);
  auto* o = reinterpret_cast<__nv_bfloat16*>(out);
  // decode batches: a token row is split over D/1024 CTAs so every SM keeps loads in flight (one column chunk per
  // thread: its k NVLink reads are issued together); prefill batches: one CTA per token
  const dim3 grid(T, T < kSplitRowsBelow ? (D / 8 + 127) / 128 : 1);
  if (k <= 8)
    cb::launch_k(moe_combine_pull_kernel<8>, grid, 128, 0, s, y_ptrs, D, ids, pos, w, k, El, a, o);
  else
    cb::launch_k(moe_combine_pull_kernel<16>, grid, 128, 0, s, y_ptrs, D, ids, pos, w, k, El, a, o);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------------------------------
// vocab-parallel embedding from peer HBM: X[t, s, :] = table_owner(id)[id - owner*per] for all hc streams
// ---------------------------------------------------------------------------------------------------------------
__global__ void embed_peer_kernel(const uint64_t* __restrict__ table_ptrs, int per, int world,
                                  const int* __restrict__ ids, int D, int hc, __nv_bfloat16* __restrict__ X,
                                  float* __restrict__ sumsq) {
  cb::pdl_entry();
  __shared__ float red[32];
  const int t = blockIdx.x;
  int id = ids[t];
  if (!cb_check_index(id, (long long)per * world, "embed_peer")) id = 0;   // bad token id: row 0, no wild read
  int owner = id / per;
  if (owner >= world) owner = world - 1;
  const __nv_bfloat16* row = reinterpret_cast<const __nv_bfloat16*>(table_ptrs[owner]) + size_t(id - owner * per) * D;
  float ss = 0.f;
  for (int col = threadIdx.x * 8; col < D; col += blockDim.x * 8) {
    const uint4 raw = *reinterpret_cast<const uint4*>(row + col);
    ss += bf16_lo(raw.x) * bf16_lo(raw.x) + bf16_hi(raw.x) * bf16_hi(raw.x) + bf16_lo(raw.y) * bf16_lo(raw.y) +
          bf16_hi(raw.y) * bf16_hi(raw.y) + bf16_lo(raw.z) * bf16_lo(raw.z) + bf16_hi(raw.z) * bf16_hi(raw.z) +
          bf16_lo(raw.w) * bf16_lo(raw.w) + bf16_hi(raw.w) * bf16_hi(raw.w);
    for (int s = 0; s < hc; ++s) *reinterpret_cast<uint4*>(X + (size_t(t) * hc + s) * D + col) = raw;
  }
  ss = block_sum(ss, red);
  if (threadIdx.x == 0 && sumsq) sumsq[t] = ss * hc;
}

cudaError_t embed_peer(const uint64_t* table_ptrs, int per, int world, const int* ids, int T, int D, int hc,
                       void* X, float* sumsq, cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  cb::launch_k(embed_peer_kernel, T, 128, 0, s, table_ptrs, per, world, ids, D, hc, reinterpret_cast<__nv_bfloat16*>(X),
                                      sumsq);
  return cudaGetLastError();
}

}  // namespace cb
