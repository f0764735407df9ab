// Native host runtime: the KV page allocator and the per-step batch metadata builder.
//
// The decode loop rebuilds, every step, the slot of each new token and the slot list of every key the batch
// attends to.  Doing that in Python costs O(batch x context) interpreter work per step; here it is one C++ pass
// writing straight into (pinned) tensors that are then copied to the device.  This replaces the sealed engine's
// scheduler bookkeeping that the reference relies on (req_to_token / token_to_kv_pool maps,
// king_v10/bundle_v9/dec/index_reuse.py:10-17) and its host-side DP-count plumbing (replay_counts.py:40).
#include <torch/extension.h>
#include <torch/cuda.h>
#include <algorithm>
#include <mutex>
#include <stdexcept>
#include <vector>

namespace {

// Free-list page allocator with reference counts (a page may be shared by requests with a common prefix).
class BlockAllocator {
 public:
  explicit BlockAllocator(int64_t num_pages) : refs_(num_pages, 0) {
    free_.reserve(num_pages);
    for (int64_t p = num_pages - 1; p >= 0; --p) free_.push_back(int32_t(p));
  }
  std::vector<int32_t> alloc(int64_t n) {
    std::lock_guard<std::mutex> g(mu_);
    if (n > int64_t(free_.size())) throw std::runtime_error("KV cache out of pages");
    std::vector<int32_t> out(n);
    for (int64_t i = 0; i < n; ++i) {
      out[i] = free_.back();
      free_.pop_back();
      refs_[out[i]] = 1;
    }
    return out;
  }
  void share(const std::vector<int32_t>& pages) {
    std::lock_guard<std::mutex> g(mu_);
    for (int32_t p : pages) {
      check(p);
      if (refs_[p] <= 0) throw std::runtime_error("share of a free page");
      ++refs_[p];
    }
  }
  void free(const std::vector<int32_t>& pages) {
    std::lock_guard<std::mutex> g(mu_);
    for (int32_t p : pages) {
      check(p);
      if (refs_[p] <= 0) throw std::runtime_error("double free of a KV page");
      if (--refs_[p] == 0) free_.push_back(p);
    }
  }
  int64_t num_free() const { return int64_t(free_.size()); }
  int64_t num_pages() const { return int64_t(refs_.size()); }
  int32_t refcount(int32_t p) const { check(p); return refs_[p]; }

 private:
  void check(int32_t p) const {
    if (p < 0 || p >= int32_t(refs_.size())) throw std::runtime_error("page id out of range");
  }
  std::vector<int32_t> refs_;
  std::vector<int32_t> free_;
  std::mutex mu_;
};

inline int32_t slot_of(const std::vector<int32_t>& pages, int64_t pos, int64_t page_size) {
  const int64_t pi = pos / page_size;
  if (pi >= int64_t(pages.size())) throw std::runtime_error("position beyond the request's pages");
  return int32_t(int64_t(pages[pi]) * page_size + pos % page_size);
}

// Decode step: request b has `seq_lens[b]` tokens including the new one.
// Returns (out_loc [B], key_slots [B, Lmax] (-1 padded), n_keys [B], pos [B]) as int32 CPU tensors.
std::vector<torch::Tensor> decode_metadata(const std::vector<std::vector<int32_t>>& page_tables,
                                           const std::vector<int64_t>& seq_lens, int64_t page_size,
                                           int64_t pad_to_batch, int64_t min_lmax) {
  const int64_t B = int64_t(seq_lens.size());
  const int64_t Bp = std::max(B, pad_to_batch);
  int64_t Lmax = std::max<int64_t>(1, min_lmax);
  for (auto l : seq_lens) Lmax = std::max(Lmax, l);
  auto opt = torch::TensorOptions().dtype(torch::kInt32).pinned_memory(torch::cuda::is_available());
  auto out_loc = torch::empty({Bp}, opt);
  auto key_slots = torch::full({Bp, Lmax}, -1, opt);
  auto n_keys = torch::zeros({Bp}, opt);
  auto pos = torch::zeros({Bp}, opt);
  int32_t* ol = out_loc.data_ptr<int32_t>();
  int32_t* ks = key_slots.data_ptr<int32_t>();
  int32_t* nk = n_keys.data_ptr<int32_t>();
  int32_t* ps = pos.data_ptr<int32_t>();
  for (int64_t b = 0; b < B; ++b) {
    const auto& pt = page_tables[b];
    const int64_t L = seq_lens[b];
    for (int64_t p = 0; p < L; ++p) ks[b * Lmax + p] = slot_of(pt, p, page_size);
    ol[b] = slot_of(pt, L - 1, page_size);
    nk[b] = int32_t(L);
    ps[b] = int32_t(L - 1);
  }
  // padding rows (CUDA-graph buckets): attend to their own scratch slot 0 only, write to slot 0
  for (int64_t b = B; b < Bp; ++b) { ol[b] = 0; ks[b * Lmax] = 0; nk[b] = 1; ps[b] = 0; }
  return {out_loc, key_slots, n_keys, pos};
}

// Prefill: request b contributes tokens [start_b, start_b + len_b) of its sequence.
// Returns (out_loc [T], pos [T]) int32 CPU tensors.
std::vector<torch::Tensor> prefill_metadata(const std::vector<std::vector<int32_t>>& page_tables,
                                            const std::vector<int64_t>& starts, const std::vector<int64_t>& lens,
                                            int64_t page_size) {
  int64_t T = 0;
  for (auto l : lens) T += l;
  auto opt = torch::TensorOptions().dtype(torch::kInt32).pinned_memory(torch::cuda::is_available());
  auto out_loc = torch::empty({T}, opt);
  auto pos = torch::empty({T}, opt);
  int32_t* ol = out_loc.data_ptr<int32_t>();
  int32_t* ps = pos.data_ptr<int32_t>();
  int64_t t = 0;
  for (size_t b = 0; b < lens.size(); ++b)
    for (int64_t p = starts[b]; p < starts[b] + lens[b]; ++p, ++t) {
      ol[t] = slot_of(page_tables[b], p, page_size);
      ps[t] = int32_t(p);
    }
  return {out_loc, pos};
}

}  // namespace

void register_runtime(pybind11::module_& m) {
  pybind11::class_<BlockAllocator>(m, "BlockAllocator")
      .def(pybind11::init<int64_t>())
      .def("alloc", &BlockAllocator::alloc)
      .def("share", &BlockAllocator::share)
      .def("free", &BlockAllocator::free)
      .def("num_free", &BlockAllocator::num_free)
      .def("num_pages", &BlockAllocator::num_pages)
      .def("refcount", &BlockAllocator::refcount);
  m.def("decode_metadata", &decode_metadata);
  m.def("prefill_metadata", &prefill_metadata);
}
