// Host launchers of the CUDA-core kernels (raw pointers + stream; no torch types, so they can be called from
// plain C/C++ as well as from the Python bindings).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace cb {

// x_rows: rows of x; gather sources outside [0, x_rows) give zero rows (-1: not checked).
cudaError_t act_quant(const void* x, int ldx, void* q, int ldq, uint32_t* sf, int M, int K, const int* src_rows,
                      cudaStream_t s, const int* n_blocks = nullptr, int x_rows = -1);
cudaError_t gather_fp8_rows(const void* src, const uint32_t* src_sf, int src_rows_n, int K, const int* src_rows,
                            int M, const int* n_blocks, void* dst, uint32_t* dst_sf, cudaStream_t s);
cudaError_t rms_norm(const void* x, int ldx, const float* w, void* y, int ldy, void* q, uint32_t* sf, int M, int D,
                     float eps, cudaStream_t s);
cudaError_t sf_pad(uint32_t* sf, int M, int K, cudaStream_t s);
cudaError_t rope_inplace(void* x, int T, int64_t stride_t, int64_t stride_h, int H, int off, int dim,
                         const float* cos_sin, const int* pos, bool inverse, cudaStream_t s);
// n_groups > 1: group-limited routing (experts only from the topk_groups groups with the best top-2 key sums)
cudaError_t router_topk(const float* logits, const float* bias, int T, int E, int k, int score, bool norm,
                        float route_scale, float* w, int* ids, cudaStream_t s,
                        const float* bias_img = nullptr, const int* tok = nullptr, int img_id = -1,
                        int n_groups = 1, int topk_groups = 1);
cudaError_t moe_layout(const int* ids, int T, int k, int E, int max_blocks, int* slot_pos, int* row_src,
                       int* m_block_expert, int* num_blocks, int* counts, cudaStream_t s, int align, int* scratch);
cudaError_t moe_combine(const void* Y, int ldy, const float* w, const int* slot_pos, int T, int k, const void* add,
                        void* out, int D, cudaStream_t s);
// mHC statistics for few tokens: mix[t, r] = X[t] · fn[r] for r < R, fp32 (CUDA cores; decode batches)
cudaError_t mhc_stats_small(const void* X, int ldx, const void* fn, int R, int K, int T, float* out, int ldo,
                            cudaStream_t s);
cudaError_t mhc_coeffs(const float* mix, int ld_mix, const float* sumsq, const float* base, const float* scale, int T,
                       int flat_dim, int iters, float hc_eps, float rms_eps, float* pre, float* post, float* comb,
                       cudaStream_t s);
cudaError_t mhc_head_coeffs(const float* mix, int ld_mix, const float* sumsq, const float* base, const float* scale,
                            int T, int flat_dim, float hc_eps, float rms_eps, float* pre, cudaStream_t s);
cudaError_t mhc_pre_norm(const void* X, const float* pre, const float* w, int T, int D, float eps, void* y, void* q,
                         uint32_t* sf, const int* rows, cudaStream_t s);
// DSA indexer post-processing of the fused [wk | weights_proj] fp32 projection kw [T, ld >= Di + Hi]: k [T, Di] bf16
// = RoPE(LayerNorm(kw[:, :Di])) (RoPE on dims [0, dr)), w [T, Hi] fp32 = kw[:, Di:] * wscale
// Per-head matmul for decode batches (swap-AB tcgen05): out[t, h, n] = sum_k x[t, h, k] w[h, n, k] for n < N, then
// out[t, h, N + j] = x[t, h, K + j] for j < tail.  x bf16 (strides xs_t, xs_h; unit stride along k), w bf16
// [H, N, K] contiguous, out bf16 or fp16 (strides os_t, os_h).  T <= 256, N % 128 == 0, K % 64 == 0.
cudaError_t head_bmm(const void* x, long long xs_t, long long xs_h, const void* w, int T, int H, int N, int K,
                     void* out, bool out_f16, long long os_t, long long os_h, int tail, int* status, cudaStream_t s);
int head_bmm_smem_bytes(int T, int K);
cudaError_t indexer_kw_post(const float* kw, int ld, int T, int Di, int Hi, const float* ln_w, const float* ln_b,
                            float eps, const float* cos_sin, const int* pos, int dr, float wscale, void* k, float* w,
                            cudaStream_t s);
// Fused decode-size mHC boundary (post-mix of `out` when given, the next sublayer's statistics and coefficients,
// pre-mix + RMSNorm + bf16 / fp8 outputs); X [T, 4, D] bf16 updated in place; D a multiple of 1024, at most 8192
cudaError_t mhc_boundary_small(void* X, int T, int D, const void* out, const float* post_in, const float* comb_in,
                               const void* fn, const float* base, const float* scale, int iters, float hc_eps,
                               float rms_eps, const float* w, void* y, void* q, uint32_t* sf, float* pre_out,
                               float* post_out, float* comb_out, cudaStream_t s);
cudaError_t mhc_post_mix(const void* X, const void* out, const float* post, const float* comb, int T, int D, void* Xn,
                         float* sumsq, cudaStream_t s);
cudaError_t embed_hc(const void* table, int row_lo, int rows, const int* ids, int T, int D, int hc, void* X,
                     float* sumsq, cudaStream_t s);
cudaError_t row_sumsq(const void* x, int T, int64_t n, float* out, cudaStream_t s);
cudaError_t silu_mul(const void* gu, int T, int I, float limit, void* out, cudaStream_t s);

// tcgen05 GEMMs (gemm.cu)
enum GemmEpiHost { GEMM_OUT_BF16 = 0, GEMM_OUT_SWIGLU_FP8 = 1, GEMM_OUT_F32 = 2 };
// fp8 block-scaled: A [M,K] e4m3 + SF tiles, B [Nb,K] e4m3 + SF tiles. Dense when m_block_expert == nullptr.
cudaError_t gemm_fp8(const void* A, const void* B, const uint32_t* sfa, const uint32_t* sfb, int M, int N, int K,
                     int Nb, void* out, int ldo, int epi, uint32_t* out_sf, float swiglu_limit,
                     const int* m_block_expert, const int* num_m_blocks_dev, int max_m_blocks, int* status,
                     int num_sms, cudaStream_t s, int pair = -1, float* work = nullptr,
                     const int* row_valid = nullptr);
// K splits gemm_fp8 uses for a dense small-M GEMM (work must then hold splits * M * N floats).
int gemm_fp8_splits(int M, int N, int K, bool grouped, int epi, int num_sms);
cudaError_t gemm_bf16(const void* A, int lda, const void* B, int ldb, int M, int N, int K, int Nb, void* out, int ldo,
                      int epi, const int* m_block_expert, const int* num_m_blocks_dev, int max_m_blocks, int* status,
                      int num_sms, cudaStream_t s, int k_splits = 1, float* work = nullptr);

// tcgen05 MLA prefill attention (attn_prefill.cu)
// sink (optional, [H] fp32): per-head attention-sink logit
cudaError_t attn_prefill(const void* q, const void* kvb, const void* kpe, int T, int H, const int* tiles,
                         int n_tiles, const uint32_t* mask, int mask_words, float scale, void* out, int* status,
                         cudaStream_t s, const float* sink = nullptr);

// trace (optional, int64 [1 + 2*trace_cap], zeroed): event timeline of CTA (0,0), see attn_prefill.cu
cudaError_t attn_prefill2(const void* q, const void* kvb, const void* kpe, int T, int H, const int* tiles,
                          int n_tiles, const uint32_t* mask, int mask_words, float scale, void* out, int* status,
                          cudaStream_t s, int64_t* trace = nullptr, int trace_cap = 0, const float* sink = nullptr);
cudaError_t attn_prefill3(const void* q, const void* kvb, const void* kpe, int T, int H, const int* tiles,
                          int n_tiles, const uint32_t* mask, int mask_words, float scale, void* out, int* status,
                          cudaStream_t s, int64_t* trace = nullptr, int trace_cap = 0, const float* sink = nullptr);

// DSA indexer: logits GEMM with fused relu/weight/head-sum epilogue (gemm.cu) and exact top-k bitmask (topk.cu)
cudaError_t indexer_logits(const void* keys, int L, const void* q, int Tq, int H, int Di, const float* w, float* out,
                           int ldo, bool causal, int* status, int num_sms, cudaStream_t s);
// fp8 e4m3 keys [L, Di] / queries [Tq*H, Di] with 1x128 UE8M0 SF tiles (block-scaled tcgen05)
cudaError_t indexer_logits_fp8(const void* keys, const uint32_t* keys_sf, int L, const void* q, const uint32_t* q_sf,
                               int Tq, int H, int Di, const float* w, float* out, int ldo, bool causal, int* status,
                               int num_sms, cudaStream_t s);
cudaError_t topk_mask(const float* logits, int ldo, int Tq, int k, uint32_t* mask, int mask_words, int row0,
                      cudaStream_t s);
// tcgen05 decode indexer (indexer_decode.cu): q [T,H,128] bf16, w [T,H], indexer-key cache kc [S,128] bf16
cudaError_t indexer_decode_logits(const void* q, const float* w, const void* kc, int S, const int* key_slots,
                                  const int* n_keys, int T, int Lmax, int H, int D, float* out, int* status,
                                  cudaStream_t s);
cudaError_t topk_index(const float* logits, const int* key_slots, const int* n_keys, int T, int Lmax, int k,
                       int* out, cudaStream_t s);
// general form: logits row stride ldo, slot row stride (0 = one shared slot list), n_keys or causal row0 + t + 1
cudaError_t topk_slots(const float* logits, int ldo, const int* key_slots, int slot_stride, const int* n_keys,
                       int row0, int T, int Lmax, int k, int* out, cudaStream_t s);

// tcgen05 absorbed-MLA sparse attention over the latent cache (attn_decode.cu)
// sink (optional, [H] fp32): per-head attention-sink logit; D: row width, 576 (MLA: 512 latent + 64 RoPE key) or
// 512 (latent MQA: the RoPE dims are the last 64 of the 512); the value is the first 512 dims either way
cudaError_t sparse_mla(const void* q, int T, int H, const void* kv, int S, const int* idx, int K, float scale,
                       int n_splits, float* part_o, float* part_ml, void* out, int* status, cudaStream_t s,
                       const float* sink = nullptr, int D = 576);
// fp8 cache rows (656 bytes per MLA row, 528 per latent-MQA row), q [T, H, D] fp16
cudaError_t sparse_mla_fp8(const void* q, int T, int H, const void* kv, int S, const int* idx, int K, float scale,
                           int n_splits, float* part_o, float* part_ml, void* out, int* status, cudaStream_t s,
                           const float* sink, int D);
// bf16 latent rows [n, D] (row stride ld) -> fp8 cache rows at slots (D = 576 or 512)
cudaError_t latent_store_fp8(const void* rows, int n, int ld, int D, const int* slots, void* cache, cudaStream_t s);

// Engram (engram.cu): fp8 row gather (UE8M0 per 32; table split over ranks by row ranges `bounds`, peer pointers)
// and the fused per-stream gate + residual update + new sum of squares
cudaError_t engram_gather(const int* ids, int T, int C, int dim, const uint64_t* data_ptrs, const uint64_t* sf_ptrs,
                          const int* bounds, int world, void* out, cudaStream_t s);
cudaError_t engram_gate(void* X, const void* kv, const float* qw, const float* kw, int T, int hc, int D, float eps,
                        float clamp, float* sumsq, cudaStream_t s, const int* tok = nullptr, int img_id = -1);

}  // namespace cb
