// Python bindings of the CUDA kernels. Shape / dtype / device checks live here; kernels take raw pointers.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <atomic>
#include "small_ops.h"

namespace {

#define CHECK_CUDA(t) TORCH_CHECK((t).is_cuda(), #t " must be a CUDA tensor")
#define CHECK_CONTIG(t) TORCH_CHECK((t).is_contiguous(), #t " must be contiguous")
#define CHECK_DT(t, d) TORCH_CHECK((t).scalar_type() == (d), #t " has dtype ", (t).scalar_type(), ", expected ", (d))
std::atomic<int64_t> g_launches{0};   // kernels launched through these bindings (bench.py reports it)

#define CK(expr)                                                                          \
  do {                                                                                    \
    cudaError_t _e = (expr);                                                              \
    TORCH_CHECK(_e == cudaSuccess, #expr " failed: ", cudaGetErrorString(_e));            \
    g_launches.fetch_add(1, std::memory_order_relaxed);                                   \
  } while (0)

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

int num_sms() {
  static int n = 0;
  if (!n) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

template <typename T>
T* ptr_or_null(const c10::optional<torch::Tensor>& t) {
  return t.has_value() && t->defined() ? reinterpret_cast<T*>(t->data_ptr()) : nullptr;
}

int64_t sf_words(int64_t M, int64_t K) { return ((K + 511) / 512) * ((M + 127) / 128) * 128; }

// ---------------------------------------------------------------------------------------------------------------
void act_quant(torch::Tensor x, torch::Tensor q, torch::Tensor sf, c10::optional<torch::Tensor> src_rows, int64_t M,
               c10::optional<torch::Tensor> n_blocks) {
  CHECK_CUDA(x); CHECK_DT(x, at::kBFloat16); CHECK_DT(q, at::kFloat8_e4m3fn); CHECK_DT(sf, at::kInt);
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1);
  const int K = x.size(1);
  TORCH_CHECK(q.size(0) >= M && q.size(1) == K && q.is_contiguous());
  TORCH_CHECK(sf.numel() >= sf_words(M, K));
  if (!src_rows.has_value()) TORCH_CHECK(x.size(0) >= M);
  c10::cuda::CUDAGuard g(x.device());
  CK(cb::act_quant(x.data_ptr(), x.stride(0), q.data_ptr(), K, reinterpret_cast<uint32_t*>(sf.data_ptr()), M, K,
                   ptr_or_null<const int>(src_rows), cur_stream(), ptr_or_null<const int>(n_blocks), int(x.size(0))));
}

void gather_fp8_rows(torch::Tensor src, torch::Tensor src_sf, torch::Tensor src_rows, torch::Tensor dst,
                     torch::Tensor dst_sf, c10::optional<torch::Tensor> n_blocks) {
  CHECK_CUDA(src); CHECK_DT(src, at::kFloat8_e4m3fn); CHECK_DT(dst, at::kFloat8_e4m3fn); CHECK_CONTIG(src);
  CHECK_CONTIG(dst); CHECK_DT(src_rows, at::kInt);
  const int K = src.size(1), M = dst.size(0);
  TORCH_CHECK(dst.size(1) == K && src_rows.numel() >= M && dst_sf.numel() >= sf_words(M, K));
  c10::cuda::CUDAGuard g(src.device());
  CK(cb::gather_fp8_rows(src.data_ptr(), reinterpret_cast<const uint32_t*>(src_sf.data_ptr()), src.size(0), K,
                         src_rows.data_ptr<int>(), M, ptr_or_null<const int>(n_blocks), dst.data_ptr(),
                         reinterpret_cast<uint32_t*>(dst_sf.data_ptr()), cur_stream()));
}

void rms_norm(torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> y, c10::optional<torch::Tensor> q,
              c10::optional<torch::Tensor> sf, double eps) {
  CHECK_CUDA(x); CHECK_DT(x, at::kBFloat16); CHECK_DT(w, at::kFloat);
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1);
  const int M = x.size(0), D = x.size(1);
  int ldy = D;
  if (y.has_value()) { CHECK_DT((*y), at::kBFloat16); TORCH_CHECK(y->stride(1) == 1); ldy = y->stride(0); }
  if (q.has_value()) { TORCH_CHECK(sf.has_value()); TORCH_CHECK(sf->numel() >= sf_words(M, D)); }
  if (M == 0) return;                         // a rank without rows this step (empty shard): nothing to launch
  c10::cuda::CUDAGuard g(x.device());
  CK(cb::rms_norm(x.data_ptr(), x.stride(0), w.data_ptr<float>(), ptr_or_null<void>(y), ldy, ptr_or_null<void>(q),
                  ptr_or_null<uint32_t>(sf), M, D, float(eps), cur_stream()));
  if (q.has_value()) CK(cb::sf_pad(reinterpret_cast<uint32_t*>(sf->data_ptr()), M, D, cur_stream()));
}

void rope(torch::Tensor x, int64_t off, int64_t dim, torch::Tensor cos_sin, torch::Tensor pos, bool inverse) {
  CHECK_CUDA(x); CHECK_DT(x, at::kBFloat16); CHECK_DT(cos_sin, at::kFloat); CHECK_DT(pos, at::kInt);
  TORCH_CHECK(x.dim() == 3 && x.stride(2) == 1, "rope expects [T, H, d] with unit inner stride");
  TORCH_CHECK(cos_sin.size(1) == dim);
  c10::cuda::CUDAGuard g(x.device());
  CK(cb::rope_inplace(x.data_ptr(), x.size(0), x.stride(0), x.stride(1), x.size(1), off, dim,
                      cos_sin.data_ptr<float>(), pos.data_ptr<int>(), inverse, cur_stream()));
}

// bias_img / tok / img_id (optional): tokens with tok[t] == img_id rank with bias_img instead of bias
void router_topk(torch::Tensor logits, c10::optional<torch::Tensor> bias, int64_t k, int64_t score, bool norm,
                 double route_scale, torch::Tensor w, torch::Tensor ids, c10::optional<torch::Tensor> bias_img,
                 c10::optional<torch::Tensor> tok, int64_t img_id, int64_t n_groups, int64_t topk_groups) {
  CHECK_CUDA(logits); CHECK_DT(logits, at::kFloat); CHECK_CONTIG(logits);
  CHECK_DT(w, at::kFloat); CHECK_DT(ids, at::kInt);
  if (tok.has_value() && tok->defined()) { CHECK_DT((*tok), at::kInt); CHECK_CONTIG((*tok)); }
  c10::cuda::CUDAGuard g(logits.device());
  CK(cb::router_topk(logits.data_ptr<float>(), ptr_or_null<const float>(bias), logits.size(0), logits.size(1), k,
                     score, norm, float(route_scale), w.data_ptr<float>(), ids.data_ptr<int>(), cur_stream(),
                     ptr_or_null<const float>(bias_img), ptr_or_null<const int>(tok), int(img_id), int(n_groups),
                     int(topk_groups)));
}

void moe_layout(torch::Tensor ids, int64_t E, torch::Tensor slot_pos, torch::Tensor row_src,
                torch::Tensor m_block_expert, torch::Tensor num_blocks, torch::Tensor counts, int64_t align,
                torch::Tensor scratch) {
  TORCH_CHECK(counts.numel() >= E && scratch.numel() >= 2 * E && scratch.scalar_type() == at::kInt);
  CHECK_CUDA(ids); CHECK_DT(ids, at::kInt); CHECK_CONTIG(ids);
  TORCH_CHECK(row_src.numel() >= m_block_expert.numel() * 128);
  c10::cuda::CUDAGuard g(ids.device());
  CK(cb::moe_layout(ids.data_ptr<int>(), ids.size(0), ids.size(1), E, m_block_expert.numel(),
                    slot_pos.data_ptr<int>(), row_src.data_ptr<int>(), m_block_expert.data_ptr<int>(),
                    num_blocks.data_ptr<int>(), counts.data_ptr<int>(), cur_stream(), int(align),
                    scratch.data_ptr<int>()));
}

void moe_combine(torch::Tensor Y, torch::Tensor w, torch::Tensor slot_pos, c10::optional<torch::Tensor> add,
                 torch::Tensor out) {
  CHECK_CUDA(Y); CHECK_DT(Y, at::kBFloat16); CHECK_DT(out, at::kBFloat16); CHECK_CONTIG(out);
  TORCH_CHECK(Y.stride(1) == 1);
  c10::cuda::CUDAGuard g(Y.device());
  CK(cb::moe_combine(Y.data_ptr(), Y.stride(0), w.data_ptr<float>(), slot_pos.data_ptr<int>(), out.size(0),
                     slot_pos.size(1), ptr_or_null<const void>(add), out.data_ptr(), out.size(1), cur_stream()));
}

void mhc_coeffs(torch::Tensor mix, torch::Tensor sumsq, torch::Tensor base, torch::Tensor scale, int64_t flat_dim,
                int64_t iters, double hc_eps, double rms_eps, torch::Tensor pre, torch::Tensor post,
                torch::Tensor comb) {
  CHECK_CUDA(mix); CHECK_DT(mix, at::kFloat);
  TORCH_CHECK(mix.size(1) >= 48 && mix.stride(1) == 1);
  c10::cuda::CUDAGuard g(mix.device());
  CK(cb::mhc_coeffs(mix.data_ptr<float>(), mix.stride(0), sumsq.data_ptr<float>(), base.data_ptr<float>(),
                    scale.data_ptr<float>(), mix.size(0), flat_dim, iters, hc_eps, rms_eps, pre.data_ptr<float>(),
                    post.data_ptr<float>(), comb.data_ptr<float>(), cur_stream()));
}

void mhc_head_coeffs(torch::Tensor mix, torch::Tensor sumsq, torch::Tensor base, torch::Tensor scale,
                     int64_t flat_dim, double hc_eps, double rms_eps, torch::Tensor pre) {
  CHECK_CUDA(mix); CHECK_DT(mix, at::kFloat);
  c10::cuda::CUDAGuard g(mix.device());
  CK(cb::mhc_head_coeffs(mix.data_ptr<float>(), mix.stride(0), sumsq.data_ptr<float>(), base.data_ptr<float>(),
                         scale.data_ptr<float>(), mix.size(0), flat_dim, hc_eps, rms_eps, pre.data_ptr<float>(),
                         cur_stream()));
}

void mhc_pre_norm(torch::Tensor X, torch::Tensor pre, torch::Tensor w, double eps, c10::optional<torch::Tensor> y,
                  c10::optional<torch::Tensor> q, c10::optional<torch::Tensor> sf, c10::optional<torch::Tensor> rows) {
  CHECK_CUDA(X); CHECK_DT(X, at::kBFloat16); CHECK_CONTIG(X);
  TORCH_CHECK(X.dim() == 3 && X.size(1) == 4);
  const int T = rows.has_value() ? rows->numel() : X.size(0);
  const int D = X.size(2);
  if (q.has_value()) { TORCH_CHECK(sf.has_value() && sf->numel() >= sf_words(T, D)); }
  c10::cuda::CUDAGuard g(X.device());
  CK(cb::mhc_pre_norm(X.data_ptr(), pre.data_ptr<float>(), w.data_ptr<float>(), T, D, eps, ptr_or_null<void>(y),
                      ptr_or_null<void>(q), ptr_or_null<uint32_t>(sf), ptr_or_null<const int>(rows), cur_stream()));
  if (q.has_value()) CK(cb::sf_pad(reinterpret_cast<uint32_t*>(sf->data_ptr()), T, D, cur_stream()));
}

void mhc_post_mix(torch::Tensor X, torch::Tensor out, torch::Tensor post, torch::Tensor comb, torch::Tensor Xn,
                  torch::Tensor sumsq) {
  CHECK_CUDA(X); CHECK_DT(X, at::kBFloat16); CHECK_CONTIG(X); CHECK_CONTIG(out); CHECK_CONTIG(Xn);
  TORCH_CHECK(X.size(1) == 4);
  c10::cuda::CUDAGuard g(X.device());
  CK(cb::mhc_post_mix(X.data_ptr(), out.data_ptr(), post.data_ptr<float>(), comb.data_ptr<float>(), X.size(0),
                      X.size(2), Xn.data_ptr(), sumsq.data_ptr<float>(), cur_stream()));
}

// Fused decode-size mHC boundary: X [T, 4, D] bf16 in place; out (optional) the previous sublayer's output [T, D]
// with its post [T, 4] / comb [T, 16]; fn [48, 4D] bf16 (hi; lo), base [24], scale [3] and norm weight w [D] of the
// next sublayer -> y [T, D] bf16, q [T, D] fp8 + sf (SF tiles), and that sublayer's pre / post / comb
void mhc_boundary_small(torch::Tensor X, c10::optional<torch::Tensor> out, c10::optional<torch::Tensor> post_in,
                        c10::optional<torch::Tensor> comb_in, torch::Tensor fn, torch::Tensor base, torch::Tensor scale,
                        int64_t iters, double hc_eps, double rms_eps, torch::Tensor w, torch::Tensor y,
                        c10::optional<torch::Tensor> q, c10::optional<torch::Tensor> sf, torch::Tensor pre_out,
                        torch::Tensor post_out, torch::Tensor comb_out) {
  CHECK_CUDA(X); CHECK_DT(X, at::kBFloat16); CHECK_CONTIG(X); CHECK_DT(fn, at::kBFloat16); CHECK_CONTIG(fn);
  CHECK_DT(w, at::kFloat); CHECK_DT(y, at::kBFloat16); CHECK_CONTIG(y);
  TORCH_CHECK(X.dim() == 3 && X.size(1) == 4, "mhc_boundary_small: X [T, 4, D]");
  const int T = X.size(0), D = X.size(2);
  TORCH_CHECK(fn.size(0) == 48 && fn.size(1) == 4 * D, "mhc_boundary_small: fn [48, 4D]");
  if (out.has_value()) {
    CHECK_DT((*out), at::kBFloat16); CHECK_CONTIG((*out));
    TORCH_CHECK(post_in.has_value() && comb_in.has_value(), "mhc_boundary_small: post / comb of the output");
  }
  c10::cuda::CUDAGuard g(X.device());
  CK(cb::mhc_boundary_small(X.data_ptr(), T, D, ptr_or_null<const void>(out), ptr_or_null<const float>(post_in),
                            ptr_or_null<const float>(comb_in), fn.data_ptr(), base.data_ptr<float>(),
                            scale.data_ptr<float>(), int(iters), float(hc_eps), float(rms_eps), w.data_ptr<float>(),
                            y.data_ptr(), ptr_or_null<void>(q), ptr_or_null<uint32_t>(sf), pre_out.data_ptr<float>(),
                            post_out.data_ptr<float>(), comb_out.data_ptr<float>(), cur_stream()));
  if (q.has_value()) CK(cb::sf_pad(reinterpret_cast<uint32_t*>(sf->data_ptr()), T, D, cur_stream()));
}

// per-head matmul of a decode batch: x [T, H, >= K + tail] bf16, w [H, N, K] bf16 -> out [T, H, N + tail]
void head_bmm(torch::Tensor x, torch::Tensor w, int64_t tail, torch::Tensor out, c10::optional<torch::Tensor> status) {
  CHECK_CUDA(x); CHECK_DT(x, at::kBFloat16); CHECK_DT(w, at::kBFloat16); CHECK_CONTIG(w);
  TORCH_CHECK(x.dim() == 3 && w.dim() == 3 && out.dim() == 3 && x.stride(2) == 1 && out.stride(2) == 1,
              "head_bmm: x [T, H, K], w [H, N, K], out [T, H, N + tail]");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 || out.scalar_type() == at::kHalf, "head_bmm: bf16 or fp16 out");
  const int T = x.size(0), H = x.size(1), N = w.size(1), K = w.size(2);
  TORCH_CHECK(w.size(0) == H && x.size(2) >= K + tail && out.size(0) == T && out.size(1) == H &&
              out.size(2) == N + tail, "head_bmm: shapes");
  c10::cuda::CUDAGuard g(x.device());
  CK(cb::head_bmm(x.data_ptr(), x.stride(0), x.stride(1), w.data_ptr(), T, H, N, K, out.data_ptr(),
                  out.scalar_type() == at::kHalf, out.stride(0), out.stride(1), int(tail), ptr_or_null<int>(status),
                  cur_stream()));
}

// DSA indexer key / head-weight post-processing (LayerNorm + RoPE of the key, scaled head weights) in one launch
void indexer_kw_post(torch::Tensor kw, int64_t Di, torch::Tensor ln_w, torch::Tensor ln_b, double eps,
                     torch::Tensor cos_sin, torch::Tensor pos, int64_t dr, double wscale, torch::Tensor k,
                     torch::Tensor w) {
  CHECK_CUDA(kw); CHECK_DT(kw, at::kFloat); CHECK_DT(ln_w, at::kFloat); CHECK_DT(ln_b, at::kFloat);
  CHECK_DT(cos_sin, at::kFloat); CHECK_DT(pos, at::kInt); CHECK_DT(k, at::kBFloat16); CHECK_DT(w, at::kFloat);
  CHECK_CONTIG(k); CHECK_CONTIG(w); CHECK_CONTIG(pos); CHECK_CONTIG(cos_sin);
  TORCH_CHECK(kw.dim() == 2 && kw.stride(1) == 1, "indexer_kw_post: kw [T, Di + Hi]");
  const int T = kw.size(0), Hi = kw.size(1) - int(Di);
  TORCH_CHECK(k.numel() == int64_t(T) * Di && w.numel() == int64_t(T) * Hi && pos.numel() >= T, "shapes");
  c10::cuda::CUDAGuard g(kw.device());
  CK(cb::indexer_kw_post(kw.data_ptr<float>(), kw.stride(0), T, int(Di), Hi, ln_w.data_ptr<float>(),
                         ln_b.data_ptr<float>(), float(eps), cos_sin.data_ptr<float>(), pos.data_ptr<int>(), int(dr),
                         float(wscale), k.data_ptr(), w.data_ptr<float>(), cur_stream()));
}

void embed_hc(torch::Tensor table, int64_t row_lo, torch::Tensor ids, torch::Tensor X,
              c10::optional<torch::Tensor> sumsq) {
  CHECK_CUDA(table); CHECK_DT(table, at::kBFloat16); CHECK_CONTIG(table); CHECK_DT(ids, at::kInt);
  c10::cuda::CUDAGuard g(table.device());
  CK(cb::embed_hc(table.data_ptr(), row_lo, table.size(0), ids.data_ptr<int>(), ids.numel(), table.size(1),
                  X.size(1), X.data_ptr(), ptr_or_null<float>(sumsq), cur_stream()));
}

void row_sumsq(torch::Tensor x, torch::Tensor out) {
  CHECK_CUDA(x); CHECK_CONTIG(x); CHECK_DT(x, at::kBFloat16);
  c10::cuda::CUDAGuard g(x.device());
  CK(cb::row_sumsq(x.data_ptr(), x.size(0), x.numel() / std::max<int64_t>(x.size(0), 1), out.data_ptr<float>(),
                   cur_stream()));
}

void silu_mul(torch::Tensor gu, double limit, torch::Tensor out) {
  CHECK_CUDA(gu); CHECK_CONTIG(gu); CHECK_CONTIG(out);
  c10::cuda::CUDAGuard g(gu.device());
  CK(cb::silu_mul(gu.data_ptr(), gu.size(0), out.size(1), float(limit), out.data_ptr(), cur_stream()));
}

// ---------------------------------------------------------------------------------------------------------------
// GEMMs
// ---------------------------------------------------------------------------------------------------------------
void gemm_fp8(torch::Tensor A, torch::Tensor sfa, torch::Tensor B, torch::Tensor sfb, torch::Tensor out, int64_t epi,
              c10::optional<torch::Tensor> out_sf, double swiglu_limit, c10::optional<torch::Tensor> m_block_expert,
              c10::optional<torch::Tensor> num_m_blocks, int64_t N_per_group, c10::optional<torch::Tensor> status,
              int64_t pair, c10::optional<torch::Tensor> row_valid) {
  CHECK_CUDA(A); CHECK_DT(A, at::kFloat8_e4m3fn); CHECK_DT(B, at::kFloat8_e4m3fn); CHECK_CONTIG(A); CHECK_CONTIG(B);
  CHECK_DT(sfa, at::kInt); CHECK_DT(sfb, at::kInt);
  const int M = A.size(0), K = A.size(1);
  const int Nb = B.size(0);
  TORCH_CHECK(B.size(1) == K, "K mismatch");
  const bool grouped = m_block_expert.has_value();
  const int N = grouped ? int(N_per_group) : Nb;
  TORCH_CHECK(sfa.numel() >= sf_words(M, K), "sfa too small");
  TORCH_CHECK(sfb.numel() >= sf_words(Nb, K), "sfb too small");
  TORCH_CHECK(out.stride(-1) == 1);
  if (epi == cb::GEMM_OUT_SWIGLU_FP8) {
    CHECK_DT(out, at::kFloat8_e4m3fn);
    TORCH_CHECK(out_sf.has_value() && out_sf->numel() >= sf_words(M, N / 2));
  } else if (epi == cb::GEMM_OUT_F32) {
    CHECK_DT(out, at::kFloat);
  } else {
    CHECK_DT(out, at::kBFloat16);
  }
  if (grouped) TORCH_CHECK(m_block_expert->numel() * 128 <= M, "grouped rows must cover all m blocks");
  c10::cuda::CUDAGuard g(A.device());
  torch::Tensor work;
  const bool pair_path = epi != cb::GEMM_OUT_F32 && (pair == 1 || (pair < 0 && !grouped && M >= 512));
  const int splits = pair_path ? 1 : cb::gemm_fp8_splits(M, N, K, grouped, int(epi), num_sms());
  if (splits > 1) work = torch::empty({int64_t(splits) * M * N}, A.options().dtype(at::kFloat));
  if (pair == 2 && grouped && epi == cb::GEMM_OUT_SWIGLU_FP8)
    work = torch::empty({int64_t(M) * N}, A.options().dtype(at::kFloat));
  CK(cb::gemm_fp8(A.data_ptr(), B.data_ptr(), reinterpret_cast<uint32_t*>(sfa.data_ptr()),
                  reinterpret_cast<uint32_t*>(sfb.data_ptr()), M, N, K, Nb, out.data_ptr(), out.stride(0), epi,
                  ptr_or_null<uint32_t>(out_sf), float(swiglu_limit), ptr_or_null<const int>(m_block_expert),
                  ptr_or_null<const int>(num_m_blocks), grouped ? m_block_expert->numel() : 0,
                  ptr_or_null<int>(status), num_sms(), cur_stream(), int(pair),
                  work.defined() ? work.data_ptr<float>() : nullptr, ptr_or_null<const int>(row_valid)));
}

void gemm_bf16(torch::Tensor A, torch::Tensor B, torch::Tensor out, int64_t epi,
               c10::optional<torch::Tensor> m_block_expert, c10::optional<torch::Tensor> num_m_blocks,
               int64_t N_per_group, c10::optional<torch::Tensor> status, int64_t k_splits) {
  torch::Tensor work;
  CHECK_CUDA(A); CHECK_DT(A, at::kBFloat16); CHECK_DT(B, at::kBFloat16);
  TORCH_CHECK(A.stride(1) == 1 && B.stride(1) == 1 && out.stride(-1) == 1);
  const int M = A.size(0), K = A.size(1), Nb = B.size(0);
  TORCH_CHECK(B.size(1) == K);
  const bool grouped = m_block_expert.has_value();
  const int N = grouped ? int(N_per_group) : Nb;
  if (epi == cb::GEMM_OUT_F32) { CHECK_DT(out, at::kFloat); } else { CHECK_DT(out, at::kBFloat16); }
  if (k_splits > 1) {
    TORCH_CHECK(epi == cb::GEMM_OUT_F32 && !grouped, "split-K needs fp32 output and a dense GEMM");
    work = torch::empty({k_splits * int64_t(M) * out.stride(0)}, A.options().dtype(at::kFloat));
  }
  c10::cuda::CUDAGuard g(A.device());
  CK(cb::gemm_bf16(A.data_ptr(), A.stride(0), B.data_ptr(), B.stride(0), M, N, K, Nb, out.data_ptr(), out.stride(0),
                   epi, ptr_or_null<const int>(m_block_expert), ptr_or_null<const int>(num_m_blocks),
                   grouped ? m_block_expert->numel() : 0, ptr_or_null<int>(status), num_sms(), cur_stream(),
                   int(k_splits), k_splits > 1 ? work.data_ptr<float>() : nullptr));
}

// q [T, H, 192], kvb [T, H, 256] (k_nope | v), kpe [T, 64] -> out [T, H, 128]
void attn_prefill(torch::Tensor q, torch::Tensor kvb, torch::Tensor kpe, torch::Tensor tiles,
                  c10::optional<torch::Tensor> mask, double scale, torch::Tensor out,
                  c10::optional<torch::Tensor> status, int64_t version, c10::optional<torch::Tensor> trace,
                  c10::optional<torch::Tensor> sink) {
  if (sink.has_value() && sink->defined()) {
    CHECK_DT((*sink), at::kFloat); CHECK_CONTIG((*sink)); TORCH_CHECK(sink->numel() >= q.size(1));
  }
  CHECK_CUDA(q); CHECK_DT(q, at::kBFloat16); CHECK_DT(kvb, at::kBFloat16); CHECK_DT(kpe, at::kBFloat16);
  CHECK_CONTIG(q); CHECK_CONTIG(kvb); CHECK_CONTIG(kpe); CHECK_CONTIG(out); CHECK_DT(tiles, at::kInt);
  TORCH_CHECK(q.size(2) == 192 && kvb.size(2) == 256 && kpe.size(-1) == 64, "attn_prefill: MLA dims 192/128");
  TORCH_CHECK(tiles.dim() == 2 && tiles.size(1) == 4);
  const int T = q.size(0), H = q.size(1);
  TORCH_CHECK(kvb.size(0) == T && kvb.size(1) == H && kpe.numel() == int64_t(T) * 64);
  int words = 0;
  if (mask.has_value()) { CHECK_DT((*mask), at::kInt); TORCH_CHECK(mask->size(0) == T); words = mask->size(1); }
  c10::cuda::CUDAGuard g(q.device());
  if (version >= 2) {
    int64_t* tr = nullptr;
    int cap = 0;
    if (trace.has_value() && trace->defined()) {
      TORCH_CHECK(trace->scalar_type() == at::kLong && trace->is_contiguous() && trace->numel() >= 3);
      tr = trace->data_ptr<int64_t>();
      cap = int((trace->numel() - 1) / 2);
    }
    auto fn = version == 3 ? cb::attn_prefill3 : cb::attn_prefill2;
    CK(fn(q.data_ptr(), kvb.data_ptr(), kpe.data_ptr(), T, H, tiles.data_ptr<int>(), tiles.size(0),
          ptr_or_null<const uint32_t>(mask), words, float(scale), out.data_ptr(), ptr_or_null<int>(status),
          cur_stream(), tr, cap, ptr_or_null<const float>(sink)));
  } else {
    CK(cb::attn_prefill(q.data_ptr(), kvb.data_ptr(), kpe.data_ptr(), T, H, tiles.data_ptr<int>(), tiles.size(0),
                        ptr_or_null<const uint32_t>(mask), words, float(scale), out.data_ptr(),
                        ptr_or_null<int>(status), cur_stream(), ptr_or_null<const float>(sink)));
  }
}

// keys [L, Di] bf16, q [Tq, H, Di] bf16, w [Tq, H] fp32 -> logits [Tq, ldo] fp32
void indexer_logits(torch::Tensor keys, torch::Tensor q, torch::Tensor w, torch::Tensor out, bool causal) {
  CHECK_CUDA(keys); CHECK_DT(keys, at::kBFloat16); CHECK_DT(q, at::kBFloat16); CHECK_DT(w, at::kFloat);
  CHECK_CONTIG(keys); CHECK_CONTIG(q); CHECK_CONTIG(w); CHECK_DT(out, at::kFloat);
  TORCH_CHECK(out.stride(1) == 1 && out.size(0) >= q.size(0) && out.stride(0) >= keys.size(0));
  c10::cuda::CUDAGuard g(keys.device());
  CK(cb::indexer_logits(keys.data_ptr(), keys.size(0), q.data_ptr(), q.size(0), q.size(1), q.size(2),
                        w.data_ptr<float>(), out.data_ptr<float>(), out.stride(0), causal, nullptr, num_sms(),
                        cur_stream()));
}

// fp8 keys kq [L, Di] + ksf, queries qq [Tq*H, Di] + qsf (act_quant SF tiles), w [Tq, H] -> logits [Tq, ldo] fp32
void indexer_logits_fp8(torch::Tensor kq, torch::Tensor ksf, torch::Tensor qq, torch::Tensor qsf, int64_t H,
                        torch::Tensor w, torch::Tensor out, bool causal) {
  CHECK_CUDA(kq); CHECK_CONTIG(kq); CHECK_CONTIG(qq); CHECK_CONTIG(w); CHECK_DT(w, at::kFloat);
  CHECK_DT(out, at::kFloat);
  TORCH_CHECK(kq.element_size() == 1 && qq.element_size() == 1 && kq.size(1) == qq.size(1));
  const int Tq = int(qq.size(0) / H);
  TORCH_CHECK(out.stride(1) == 1 && out.size(0) >= Tq && out.stride(0) >= kq.size(0));
  c10::cuda::CUDAGuard g(kq.device());
  CK(cb::indexer_logits_fp8(kq.data_ptr(), reinterpret_cast<const uint32_t*>(ksf.data_ptr()), kq.size(0),
                            qq.data_ptr(), reinterpret_cast<const uint32_t*>(qsf.data_ptr()), Tq, int(H),
                            int(kq.size(1)), w.data_ptr<float>(), out.data_ptr<float>(), out.stride(0), causal,
                            nullptr, num_sms(), cur_stream()));
}

void topk_mask(torch::Tensor logits, int64_t Tq, int64_t k, torch::Tensor mask, int64_t row0) {
  CHECK_CUDA(logits); CHECK_DT(logits, at::kFloat); CHECK_DT(mask, at::kInt); CHECK_CONTIG(mask);
  TORCH_CHECK(logits.stride(1) == 1 && row0 + Tq <= mask.size(0) && mask.size(1) * 32 >= Tq);
  c10::cuda::CUDAGuard g(logits.device());
  CK(cb::topk_mask(logits.data_ptr<float>(), logits.stride(0), Tq, k, reinterpret_cast<uint32_t*>(mask.data_ptr()),
                   mask.size(1), row0, cur_stream()));
}

// q [T, H, D], kv [S, D] bf16 (D = 576 MLA latent + RoPE key, or 512 latent MQA), idx [T, K] int32
// -> out [T, H, 512] bf16
// Absorbed sparse attention over cached latent rows.  kv bf16 [S, D] with q bf16, or kv uint8 [S, 656 | 528] (the
// fp8 cache format) with q fp16.
void sparse_mla(torch::Tensor q, torch::Tensor kv, torch::Tensor idx, double scale, int64_t n_splits,
                c10::optional<torch::Tensor> work, torch::Tensor out, c10::optional<torch::Tensor> sink) {
  if (sink.has_value() && sink->defined()) {
    CHECK_DT((*sink), at::kFloat); CHECK_CONTIG((*sink)); TORCH_CHECK(sink->numel() >= q.size(1));
  }
  const bool f8 = kv.scalar_type() == at::kByte;
  CHECK_CUDA(q); CHECK_DT(idx, at::kInt); CHECK_DT(out, at::kBFloat16);
  if (f8) { CHECK_DT(q, at::kHalf); } else { CHECK_DT(q, at::kBFloat16); CHECK_DT(kv, at::kBFloat16); }
  CHECK_CONTIG(q); CHECK_CONTIG(kv); CHECK_CONTIG(idx); CHECK_CONTIG(out);
  const int D = q.size(2);
  TORCH_CHECK((D == 576 || D == 512) && out.size(2) == 512, "sparse_mla: q width 576 or 512, out width 512");
  TORCH_CHECK(kv.size(1) == (f8 ? (D == 576 ? 656 : 528) : D), "sparse_mla: cache row width");
  const int T = q.size(0), H = q.size(1);
  float* po = nullptr;
  float* pml = nullptr;
  if (n_splits > 1) {
    TORCH_CHECK(work.has_value() && work->numel() >= int64_t(T) * n_splits * H * 514, "sparse_mla: workspace");
    po = work->data_ptr<float>();
    pml = po + int64_t(T) * n_splits * H * 512;
  }
  c10::cuda::CUDAGuard g(q.device());
  auto fn = f8 ? cb::sparse_mla_fp8 : cb::sparse_mla;
  CK(fn(q.data_ptr(), T, H, kv.data_ptr(), kv.size(0), idx.data_ptr<int>(), idx.size(1), float(scale), n_splits, po,
        pml, out.data_ptr(), nullptr, cur_stream(), ptr_or_null<const float>(sink), D));
}

// bf16 latent rows [n, D] (row stride free, unit column stride) -> fp8 cache rows [S, 656 | 528] at slots [n]
void latent_store_fp8(torch::Tensor rows, torch::Tensor slots, torch::Tensor cache) {
  CHECK_CUDA(rows); CHECK_DT(rows, at::kBFloat16); CHECK_DT(slots, at::kInt); CHECK_CONTIG(slots);
  CHECK_DT(cache, at::kByte); CHECK_CONTIG(cache);
  TORCH_CHECK(rows.dim() == 2 && rows.stride(1) == 1, "latent_store_fp8: rows [n, D] with unit column stride");
  const int D = rows.size(1);
  TORCH_CHECK((D == 576 || D == 512) && cache.size(1) == (D == 576 ? 656 : 528), "latent_store_fp8: widths");
  TORCH_CHECK(slots.numel() == rows.size(0), "latent_store_fp8: one slot per row");
  c10::cuda::CUDAGuard g(rows.device());
  CK(cb::latent_store_fp8(rows.data_ptr(), rows.size(0), rows.stride(0), D, slots.data_ptr<int>(), cache.data_ptr(),
                          cur_stream()));
}

// Engram row gather: ids [T, C] int32 global rows; data_ptrs / sf_ptrs uint64 [world] (fp8 rows [R_r, dim], UE8M0
// bytes [R_r, dim/32] of each rank's shard); bounds int32 [world + 1] global row ranges -> out [T, C*dim] bf16
void engram_gather(torch::Tensor ids, torch::Tensor data_ptrs, torch::Tensor sf_ptrs, torch::Tensor bounds,
                   int64_t dim, torch::Tensor out) {
  CHECK_CUDA(ids); CHECK_DT(ids, at::kInt); CHECK_CONTIG(ids); CHECK_DT(bounds, at::kInt); CHECK_CONTIG(out);
  CHECK_DT(out, at::kBFloat16);
  TORCH_CHECK(out.numel() == ids.numel() * dim, "engram_gather: out size");
  c10::cuda::CUDAGuard g(ids.device());
  CK(cb::engram_gather(ids.data_ptr<int>(), ids.size(0), ids.size(1), dim,
                       reinterpret_cast<const uint64_t*>(data_ptrs.data_ptr()),
                       reinterpret_cast<const uint64_t*>(sf_ptrs.data_ptr()), bounds.data_ptr<int>(),
                       data_ptrs.numel(), out.data_ptr(), cur_stream()));
}

// Engram gate, in place on X [T, hc, D] bf16 with kv [T, (hc+1)*D] bf16; sumsq [T] fp32 <- new sum of squares
void engram_gate(torch::Tensor X, torch::Tensor kv, torch::Tensor qw, torch::Tensor kw, double eps, double clamp,
                 torch::Tensor sumsq, c10::optional<torch::Tensor> tok, int64_t img_id) {
  CHECK_CUDA(X); CHECK_DT(X, at::kBFloat16); CHECK_DT(kv, at::kBFloat16); CHECK_CONTIG(X); CHECK_CONTIG(kv);
  CHECK_DT(qw, at::kFloat); CHECK_DT(kw, at::kFloat); CHECK_DT(sumsq, at::kFloat);
  const int T = X.size(0), hc = X.size(1), D = X.size(2);
  TORCH_CHECK(kv.size(0) == T && kv.size(1) == (hc + 1) * D, "engram_gate: kv shape");
  c10::cuda::CUDAGuard g(X.device());
  CK(cb::engram_gate(X.data_ptr(), kv.data_ptr(), qw.data_ptr<float>(), kw.data_ptr<float>(), T, hc, D, float(eps),
                     float(clamp), sumsq.data_ptr<float>(), cur_stream(), ptr_or_null<const int>(tok),
                     int(img_id)));
}

// decode-side DSA: q [T, H, 128] bf16, w [T, H] fp32, kc [S, 128] bf16, key_slots [T, L], n_keys [T] -> out [T, k]
void mhc_stats_small(torch::Tensor X, torch::Tensor fn, int64_t rows, torch::Tensor out) {
  CHECK_CUDA(X); CHECK_DT(X, at::kBFloat16); CHECK_DT(fn, at::kBFloat16); CHECK_DT(out, at::kFloat);
  CHECK_CONTIG(fn); TORCH_CHECK(X.dim() == 2 && X.stride(1) == 1 && out.stride(1) == 1);
  TORCH_CHECK(fn.size(1) == X.size(1) && rows <= fn.size(0) && out.size(1) >= rows && out.size(0) == X.size(0));
  c10::cuda::CUDAGuard g(X.device());
  CK(cb::mhc_stats_small(X.data_ptr(), X.stride(0), fn.data_ptr(), int(rows), X.size(1), X.size(0),
                         out.data_ptr<float>(), out.stride(0), cur_stream()));
}

void indexer_decode_logits(torch::Tensor q, torch::Tensor w, torch::Tensor kc, torch::Tensor key_slots,
                           torch::Tensor n_keys, torch::Tensor logits) {
  CHECK_CUDA(q); CHECK_CONTIG(q); CHECK_CONTIG(kc); CHECK_CONTIG(key_slots); CHECK_CONTIG(logits);
  CHECK_DT(q, at::kBFloat16); CHECK_DT(kc, at::kBFloat16); CHECK_DT(w, at::kFloat); CHECK_DT(logits, at::kFloat);
  CHECK_DT(key_slots, at::kInt); CHECK_DT(n_keys, at::kInt);
  const int T = q.size(0), L = key_slots.size(1);
  TORCH_CHECK(logits.size(0) == T && logits.size(1) == L && kc.size(1) == q.size(2));
  c10::cuda::CUDAGuard g(q.device());
  CK(cb::indexer_decode_logits(q.data_ptr(), w.contiguous().data_ptr<float>(), kc.data_ptr(), kc.size(0),
                               key_slots.data_ptr<int>(), n_keys.data_ptr<int>(), T, L, q.size(1), q.size(2),
                               logits.data_ptr<float>(), nullptr, cur_stream()));
}

// Causal top-k of one prefill sequence block: logits [Tq, ldo] (row t: keys 0..row0+t), seq_slots [L] -> out [Tq, k].
void topk_causal_slots(torch::Tensor logits, torch::Tensor seq_slots, int64_t row0, torch::Tensor out) {
  CHECK_CUDA(logits); CHECK_DT(logits, at::kFloat); CHECK_DT(seq_slots, at::kInt); CHECK_DT(out, at::kInt);
  CHECK_CONTIG(seq_slots); CHECK_CONTIG(out);
  TORCH_CHECK(logits.stride(1) == 1 && out.size(0) == logits.size(0));
  const int T = logits.size(0), L = seq_slots.numel();
  TORCH_CHECK(row0 + T <= L && logits.size(1) >= row0 + T, "causal rows beyond the sequence");
  c10::cuda::CUDAGuard g(logits.device());
  CK(cb::topk_slots(logits.data_ptr<float>(), logits.stride(0), seq_slots.data_ptr<int>(), 0, nullptr, int(row0), T,
                    L, out.size(1), out.data_ptr<int>(), cur_stream()));
}

void indexer_topk(torch::Tensor q, torch::Tensor w, torch::Tensor kc, torch::Tensor key_slots, torch::Tensor n_keys,
                  torch::Tensor out) {
  CHECK_CUDA(q); CHECK_CONTIG(out); CHECK_DT(out, at::kInt);
  const int T = q.size(0), L = key_slots.size(1);
  auto logits = torch::empty({T, L}, q.options().dtype(at::kFloat));
  indexer_decode_logits(q, w, kc, key_slots, n_keys, logits);
  c10::cuda::CUDAGuard g(q.device());
  CK(cb::topk_index(logits.data_ptr<float>(), key_slots.data_ptr<int>(), n_keys.data_ptr<int>(), T, L, out.size(1),
                    out.data_ptr<int>(), cur_stream()));
}

}  // namespace

void register_runtime(pybind11::module_& m);
void register_p2p(pybind11::module_& m);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  register_runtime(m);
  register_p2p(m);
  m.doc() = "carbon_b200 sm_100a kernels";
  m.def("act_quant", &act_quant);
  m.def("rms_norm", &rms_norm);
  m.def("rope", &rope);
  m.def("router_topk", &router_topk);
  m.def("moe_layout", &moe_layout);
  m.def("gather_fp8_rows", &gather_fp8_rows);
  m.def("moe_combine", &moe_combine);
  m.def("mhc_coeffs", &mhc_coeffs);
  m.def("mhc_head_coeffs", &mhc_head_coeffs);
  m.def("mhc_pre_norm", &mhc_pre_norm);
  m.def("mhc_boundary_small", &mhc_boundary_small);
  m.def("indexer_kw_post", &indexer_kw_post);
  m.def("head_bmm", &head_bmm);
  m.def("mhc_post_mix", &mhc_post_mix);
  m.def("embed_hc", &embed_hc);
  m.def("row_sumsq", &row_sumsq);
  m.def("silu_mul", &silu_mul);
  m.def("gemm_fp8", &gemm_fp8);
  m.def("gemm_bf16", &gemm_bf16);
  m.def("sf_words", &sf_words);
  m.def("launch_count", []() { return g_launches.load(); });
  m.def("attn_prefill", &attn_prefill);
  m.def("indexer_logits", &indexer_logits);
  m.def("indexer_logits_fp8", &indexer_logits_fp8);
  m.def("topk_mask", &topk_mask);
  m.def("sparse_mla", &sparse_mla);
  m.def("latent_store_fp8", &latent_store_fp8);
  m.def("engram_gather", &engram_gather);
  m.def("engram_gate", &engram_gate);
  m.def("indexer_topk", &indexer_topk);
  m.def("indexer_decode_logits", &indexer_decode_logits);
  m.def("topk_causal_slots", &topk_causal_slots);
  m.def("mhc_stats_small", &mhc_stats_small);
}
