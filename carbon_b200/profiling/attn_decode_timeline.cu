// Timeline of the sparse decode attention kernel: 32 tokens x 128 heads x the top-2048 of 4096 cached rows each (in
// key order, as the DSA top-k hands them over), 2 key splits.  Compiles the kernel's translation unit with
// -DCB_DECODE_TRACE, which makes the first CTA pair record the SM clock of every pipeline event of every 32-key tile
// (TMA issue, conversion done, QK / PV issue, S observed, peer partial observed, P written, exchange slot free), and
// prints the table for both CTAs.  Build and run on a B200:
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 --expt-relaxed-constexpr -DCB_DECODE_TRACE \
//        -Icarbon_b200/csrc carbon_b200/profiling/attn_decode_timeline.cu -o attn_timeline -lcuda
//   ./attn_timeline          (fp8 cache rows)      ./attn_timeline bf16   (bf16 rows)
#include "../csrc/attn_decode.cu"
#include <cstdio>
#include <vector>
#include <algorithm>
#include <random>

int main(int argc, char** argv) {
  const int T = 32, H = 128, K = 2048, CTX = 4096, S = T * CTX, D = 576, RB = 656;
  const bool f8 = argc < 2 || argv[1][0] != 'b';
  const int splits = 2;
  std::mt19937 rng(1);
  std::vector<uint16_t> hq(size_t(T) * H * D);
  std::normal_distribution<float> nd(0.f, 0.5f);
  for (auto& v : hq) { __half h = __float2half(nd(rng)); v = *reinterpret_cast<uint16_t*>(&h); }
  std::vector<uint16_t> hrows(size_t(S) * D);
  for (auto& v : hrows) { __nv_bfloat16 b = __float2bfloat16(nd(rng) * 2.f); v = *reinterpret_cast<uint16_t*>(&b); }
  std::vector<int> hidx(size_t(T) * K);
  for (int t = 0; t < T; ++t) {
    std::vector<int> p(CTX);
    for (int i = 0; i < CTX; ++i) p[i] = i;
    std::shuffle(p.begin(), p.end(), rng);
    std::sort(p.begin(), p.begin() + K);
    for (int i = 0; i < K; ++i) hidx[size_t(t) * K + i] = t * CTX + p[i];
  }
  void *q, *rows, *kv, *out;
  int *idx, *slots;
  float* work;
  long long* tr;
  cudaMalloc(&q, hq.size() * 2);
  cudaMalloc(&rows, hrows.size() * 2);
  cudaMalloc(&kv, size_t(S) * (f8 ? RB : D * 2));
  cudaMalloc(&idx, hidx.size() * 4);
  cudaMalloc(&slots, S * 4);
  cudaMalloc(&out, size_t(T) * H * 512 * 2);
  cudaMalloc(&work, size_t(T) * splits * H * 514 * 4);
  cudaMalloc(&tr, 2 * 8 * 64 * 8);
  cudaMemset(tr, 0, 2 * 8 * 64 * 8);
  std::vector<int> hs(S);
  for (int i = 0; i < S; ++i) hs[i] = i;
  cudaMemcpy(q, hq.data(), hq.size() * 2, cudaMemcpyHostToDevice);
  cudaMemcpy(rows, hrows.data(), hrows.size() * 2, cudaMemcpyHostToDevice);
  cudaMemcpy(idx, hidx.data(), hidx.size() * 4, cudaMemcpyHostToDevice);
  cudaMemcpy(slots, hs.data(), S * 4, cudaMemcpyHostToDevice);
  if (f8) cb::latent_store_fp8(rows, S, D, D, slots, kv, 0);
  else cudaMemcpy(kv, rows, hrows.size() * 2, cudaMemcpyDeviceToDevice);
  cudaMemcpyToSymbol(cb::mla::g_attn_trace, &tr, sizeof(tr));
  float* po = work;
  float* pml = work + size_t(T) * splits * H * 512;
  cudaEvent_t a, b;
  cudaEventCreate(&a); cudaEventCreate(&b);
  float best = 1e9;
  for (int it = 0; it < 5; ++it) {
    cudaEventRecord(a);
    cudaError_t e = f8 ? cb::sparse_mla_fp8(q, T, H, kv, S, idx, K, 0.07f, splits, po, pml, out, nullptr, 0, nullptr, D)
                       : cb::sparse_mla(q, T, H, kv, S, idx, K, 0.07f, splits, po, pml, out, nullptr, 0, nullptr, D);
    cudaEventRecord(b);
    cudaEventSynchronize(b);
    float ms;
    cudaEventElapsedTime(&ms, a, b);
    if (ms < best) best = ms;
    if (e != cudaSuccess) printf("launch error %s\n", cudaGetErrorString(e));
  }
  printf("%s: best %.1f us, err=%s\n", f8 ? "fp8" : "bf16", best * 1e3, cudaGetErrorString(cudaDeviceSynchronize()));
  std::vector<long long> h(2 * 8 * 64);
  cudaMemcpy(h.data(), tr, h.size() * 8, cudaMemcpyDeviceToHost);
  const char* names[8] = {"tma_issue", "cvt_done", "qk_issue", "pv_issue", "s_full", "x_full", "p_arrive", "x_empty"};
  for (int c = 0; c < 2; ++c) {
    long long t0 = h[(c * 8 + 0) * 64 + 0];
    for (int ev = 0; ev < 8; ++ev) if (h[(c * 8 + ev) * 64] && h[(c * 8 + ev) * 64] < t0) t0 = h[(c * 8 + ev) * 64];
    printf("CTA %d (clock cycles from its first event)\n tile", c);
    for (int ev = 0; ev < 8; ++ev) printf(" %10s", names[ev]);
    printf("\n");
    for (int j = 0; j < 34; ++j) {
      printf(" %4d", j);
      for (int ev = 0; ev < 8; ++ev) {
        const long long v = h[(c * 8 + ev) * 64 + j];
        printf(" %10lld", v ? v - t0 : -1);
      }
      printf("\n");
    }
  }
  return 0;
}
